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
#include "wf_sm100.cuh"

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

// The alternative the attention kernel does not use: the same rows moved by the
// bulk-copy engine (cp.async.bulk, global -> shared, completion on an mbarrier).
// One warp per query; lane 0 issues the K and V rows of kBulkKeys keys per stage
// into a two-stage ring of this warp's shared memory and the warp waits for each
// stage (bounded).  READ: the warp then reads every staged byte back with 16-byte
// shared loads, as a kernel consuming the rows would; otherwise it reads nothing.
constexpr int kBulkWarps = 4;
constexpr int kBulkKeys = 4;
constexpr int kBulkStage = 2 * kBulkKeys * 1024;  // K and V rows of kBulkKeys keys
constexpr uint64_t kBulkWaitNs = 1000000000ull;

template <bool READ>
__global__ void __launch_bounds__(kBulkWarps * 32) gather_rows_bulk_kernel(const char* __restrict__ k,
                                                                         const char* __restrict__ v,
                                                                         int64_t stride_bytes,
                                                                         const int32_t* __restrict__ idx,
                                                                         int64_t n_query, int K, int64_t n_rows,
                                                                         uint32_t* __restrict__ sink) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bars[kBulkWarps][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qi = (int64_t)blockIdx.x * kBulkWarps + warp;
  unsigned char* ring = smem + (size_t)warp * 2 * kBulkStage;
  if (lane == 0) {
    sm100::mbar_init(&bars[warp][0], 1);
    sm100::mbar_init(&bars[warp][1], 1);
    sm100::fence_mbarrier_init();
  }
  __syncwarp();
  if (qi >= n_query) return;
  const int32_t* row = idx + qi * K;
  const int nchunk = K / kBulkKeys;
  auto issue = [&](int ch) {
    if (lane != 0) return;
    uint64_t* bar = &bars[warp][ch & 1];
    unsigned char* dst = ring + (ch & 1) * kBulkStage;
    sm100::mbar_arrive_expect_tx(bar, kBulkStage);
    for (int u = 0; u < kBulkKeys; ++u) {
      int j = row[ch * kBulkKeys + u];
      j = (j >= 0 && j < n_rows) ? j : 0;
      const char* srcs[2] = {k + (int64_t)j * stride_bytes, v + (int64_t)j * stride_bytes};
      for (int t = 0; t < 2; ++t)
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                sm100::smem_u32(dst + (2 * u + t) * 1024)),
            "l"(srcs[t]), "r"(1024), "r"(sm100::smem_u32(bar))
            : "memory");
    }
  };
  uint32_t acc = 0;
  bool ok = true;
  issue(0);
  for (int ch = 0; ch < nchunk; ++ch) {
    if (ch + 1 < nchunk) issue(ch + 1);  // the other stage was consumed in iteration ch - 1
    ok = __all_sync(0xffffffffu, sm100::mbar_wait(&bars[warp][ch & 1], (uint32_t)(ch >> 1) & 1u, kBulkWaitNs));
    if (!ok) {
      // give the copies in flight (stages ch and ch + 1) one more bounded wait, then stop
      for (int c = ch; c <= ch + 1 && c < nchunk; ++c)
        sm100::mbar_wait(&bars[warp][c & 1], (uint32_t)(c >> 1) & 1u, kBulkWaitNs);
      break;
    }
    if (READ) {
      const uint4* st = reinterpret_cast<const uint4*>(ring + (ch & 1) * kBulkStage);
#pragma unroll
      for (int i = 0; i < kBulkStage / 16 / 32; ++i) {
        const uint4 x = st[i * 32 + lane];
        acc ^= x.x ^ x.y ^ x.z ^ x.w;
      }
    }
    __syncwarp();
  }
  acc = __reduce_xor_sync(0xffffffffu, acc);
  if (lane == 0) sink[qi] = ok ? acc : 0xffffffffu;  // a wait that gave up marks the query
}

}  // namespace

int launch_gather_rows_bulk_bench(const void* k, const void* v, int64_t stride_bytes, const int32_t* idx,
                                  int64_t n_query, int K, int64_t n_rows, int read_back, uint32_t* sink,
                                  cudaStream_t stream) {
  if (K < kBulkKeys || K % kBulkKeys || n_query < 1 || stride_bytes % 16) return -1;
  const unsigned blocks = (unsigned)((n_query + kBulkWarps - 1) / kBulkWarps);
  const int smem = kBulkWarps * 2 * kBulkStage;
  auto kern = read_back ? gather_rows_bulk_kernel<true> : gather_rows_bulk_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  kern<<<blocks, kBulkWarps * 32, smem, stream>>>(static_cast<const char*>(k), static_cast<const char*>(v),
                                                   stride_bytes, idx, n_query, K, n_rows, sink);
  return (int)cudaGetLastError();
}

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
