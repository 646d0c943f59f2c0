// Gather-rate ceiling for the sparse-attention access pattern (a measurement aid,
// not part of the operator).
//
// The attention kernel at the headline shape reads every retrieved key's K and V
// rows (H*D contiguous elements of one token, 1 KB at H=8, D=64 bf16) with 16-byte
// non-coherent loads, one warp per query, several rows in flight per lane.  When
// K/V fit in L2 that stream, not HBM, bounds the kernel.  This kernel issues the
// same loads over the same indices and does nothing else (the loaded words are
// folded into one word per warp so the loads stay live), so its rate is the
// ceiling the attention kernel can approach with this load scheme.
#include "wf_kernels.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace wf {
namespace {

constexpr int kWarps = 8;
constexpr int kInFlight = 4;  // retrieved rows per lane in flight, as the attention kernel keeps

// FULL: rows of exactly 64 vectors (1 KB), two per lane, no per-load predicate.
template <bool FULL>
__global__ void __launch_bounds__(kWarps * 32) gather_rows_kernel(const uint4* __restrict__ k,
                                                                const uint4* __restrict__ v, int64_t row_vecs,
                                                                int64_t stride_vecs, const int32_t* __restrict__ idx,
                                                                int64_t n_query, int K, int64_t n_rows,
                                                                uint32_t* __restrict__ sink) {
  const int lane = threadIdx.x & 31;
  const int64_t qi = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (qi >= n_query) return;
  const int32_t* row = idx + qi * K;
  uint32_t acc = 0;
  for (int s0 = 0; s0 < K; s0 += 32) {
    const int my = s0 + lane < K ? row[s0 + lane] : 0;
    const int n = K - s0 < 32 ? K - s0 : 32;
    for (int j0 = 0; j0 < n; j0 += kInFlight) {
      uint4 a[kInFlight][2], b[kInFlight][2];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        int j = __shfl_sync(0xffffffffu, my, (j0 + u) & 31);
        if (!FULL) j = (j0 + u < n && j >= 0 && j < n_rows) ? j : 0;
        else j = (j >= 0 && j < n_rows) ? j : 0;
        const int64_t base = (int64_t)j * stride_vecs;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int64_t e = lane + 32 * c;
          const bool in = FULL || e < row_vecs;
          a[u][c] = in ? __ldg(k + base + e) : make_uint4(0, 0, 0, 0);
          b[u][c] = in ? __ldg(v + base + e) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kInFlight; ++u)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          acc ^= a[u][c].x ^ a[u][c].y ^ a[u][c].z ^ a[u][c].w ^ b[u][c].x ^ b[u][c].y ^ b[u][c].z ^ b[u][c].w;
    }
  }
  acc = __reduce_xor_sync(0xffffffffu, acc);
  if (lane == 0) sink[qi] = acc;
}

}  // namespace

int launch_gather_rows_bench(const void* k, const void* v, int64_t row_bytes, int64_t stride_bytes,
                             const int32_t* idx, int64_t n_query, int K, int64_t n_rows, uint32_t* sink,
                             cudaStream_t stream) {
  if (row_bytes <= 0 || row_bytes > 1024 || row_bytes % 16 || stride_bytes % 16 || K < 1 || n_query < 1)
    return -1;
  const unsigned blocks = (unsigned)((n_query + kWarps - 1) / kWarps);
  auto kern = (row_bytes == 1024 && K % 32 == 0) ? gather_rows_kernel<true> : gather_rows_kernel<false>;
  kern<<<blocks, kWarps * 32, 0, stream>>>(static_cast<const uint4*>(k), static_cast<const uint4*>(v), row_bytes / 16,
                                          stride_bytes / 16, idx, n_query, K, n_rows, sink);
  return (int)cudaGetLastError();
}

}  // namespace wf
