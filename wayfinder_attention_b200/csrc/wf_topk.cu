// Exact causal top-K retrieval over learned addresses (CUDA-core scorer).
//
// Semantics follow routing_attention/kernels/causal_topk.py of the reference:
//   * scores s[i, j] = <q_addr[i], k_addr[j]> in fp32 (inputs upcast exactly,
//     causal_topk.py:150-151), keys j <= i only (mask, causal_topk.py:111-129);
//   * K_eff = min(top_k, T) slots per row (causal_topk.py:495);
//   * rows with fewer than K_eff causal keys get pad indices (i + K + s + 1) % T
//     in their empty slots (causal_topk.py:37-57), using the sorted-slot
//     convention (valid entries first), or -1 when pad_mode == 1.
// Slots are ordered by descending score; equal scores break to the lower key
// index, which makes the result a deterministic function of the inputs.
//
// Design: one CTA owns 64 consecutive query rows.  Keys stream through shared
// memory in chunks of 64; a 16x16 thread grid computes the 64x64 fp32 score
// tile with a fixed summation order (d = 0..R-1).  The T x T score matrix never
// leaves the SM.  Each warp owns 8 rows and keeps, per row, a candidate buffer
// in shared memory plus a strict admission threshold (the current K-th best
// key).  Because keys arrive in increasing index order, a later key that ties
// the threshold always loses, so "admit iff key > threshold" is exact.  When a
// buffer overflows, the warp runs a 32-step radix select on the ordered keys to
// find the exact K-th value and compacts the buffer back to K entries.
#include "wf_common.cuh"
#include "wf_kernels.h"
#include "wf_select.cuh"

#include <climits>
#include <cstdlib>
#include <cstring>

namespace wf {
namespace {

using select::merge_row;
using select::bitonic_sort_desc;

constexpr int kRows = 64;      // query rows per CTA
constexpr int kChunk = 64;     // keys per streamed chunk
constexpr int kThreads = 256;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxDevices = 64;

template <typename TI, int RP, int EPL, int SE>
__global__ void __launch_bounds__(kThreads, 1) causal_topk_kernel(const TopkParams p) {
  constexpr int CAP = 32 * EPL;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* qs = reinterpret_cast<float*>(smem_raw);     // [RP][kRows]
  float* ks = qs + RP * kRows;                        // [RP][kChunk]
  float* sc = ks + RP * kChunk;                       // [kRows][kChunk]
  uint32_t* thr = reinterpret_cast<uint32_t*>(sc + kRows * kChunk);
  int* cnt = reinterpret_cast<int*>(thr + kRows);
  uint32_t* bkey = reinterpret_cast<uint32_t*>(cnt + kRows);  // [kRows][CAP]
  int* bidx = reinterpret_cast<int*>(bkey + kRows * CAP);     // [kRows][CAP]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntile = (p.Tq + kRows - 1) / kRows;
  const int tile = ntile - 1 - (int)blockIdx.x;  // heaviest (latest) rows first
  const int b = blockIdx.y;
  const int l0 = tile * kRows;
  const int nrows = min(kRows, p.Tq - l0);
  const int g0 = p.lim ? 0 : ((l0 / p.rt) * p.rs + p.r0) * p.rt + (l0 % p.rt);
  const int32_t* lrow = p.lim ? p.lim + (int64_t)b * p.Tq + l0 : nullptr;  // per-row key limits
  const int key_end = min(lrow ? lrow[nrows - 1] : g0 + nrows, p.Tk);

  const TI* qb = reinterpret_cast<const TI*>(p.q) + (int64_t)b * p.qsb;
  const TI* kb = reinterpret_cast<const TI*>(p.k) + (int64_t)b * p.ksb;

  for (int e = tid; e < RP * kRows; e += kThreads) {
    const int r = e % kRows, d = e / kRows;
    float v = 0.f;
    if (r < nrows && d < p.R) v = to_f32(qb[(int64_t)(l0 + r) * p.qst + (int64_t)d * p.qsr]);
    qs[d * kRows + r] = v;
  }
  if (tid < kRows) {
    thr[tid] = 0u;
    cnt[tid] = 0;
  }

  const int tx = tid & 15, ty = tid >> 4;
  for (int c0 = 0; c0 < key_end; c0 += kChunk) {
    __syncthreads();
    for (int e = tid; e < RP * kChunk; e += kThreads) {
      const int c = e % kChunk, d = e / kChunk;
      float v = 0.f;
      if (c0 + c < key_end && d < p.R) v = to_f32(kb[(int64_t)(c0 + c) * p.kst + (int64_t)d * p.ksr]);
      ks[d * kChunk + c] = v;
    }
    __syncthreads();
    {
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 8
      for (int d = 0; d < RP; ++d) {
        const float4 a = *reinterpret_cast<const float4*>(&qs[d * kRows + ty * 4]);
        const float4 k4 = *reinterpret_cast<const float4*>(&ks[d * kChunk + tx * 4]);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], kv[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(&sc[(ty * 4 + i) * kChunk + tx * 4]) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
    __syncthreads();

#pragma unroll 1
    for (int rr = 0; rr < kRows / 8; ++rr) {
      const int r = warp * (kRows / 8) + rr;
      if (r >= nrows) break;
      const int g = lrow ? lrow[r] - 1 : g0 + r;
      if (c0 > g) continue;
      uint32_t* bk = bkey + r * CAP;
      int* bi = bidx + r * CAP;
      int n = cnt[r];
      uint32_t t = thr[r];
#pragma unroll
      for (int h = 0; h < kChunk / 32; ++h) {
        const int j = c0 + h * 32 + lane;
        const uint32_t key = ordered_key(sc[r * kChunk + h * 32 + lane]);
        const bool valid = j <= g;
        bool pass = valid && key > t;
        unsigned m = __ballot_sync(kFull, pass);
        if (m == 0u) continue;
        if (n + __popc(m) > CAP) {
          t = merge_row<EPL>(bk, bi, n, p.K, lane);
          n = p.K;
          pass = valid && key > t;
          m = __ballot_sync(kFull, pass);
        }
        if (pass) {
          const int pos = n + __popc(m & lanemask_lt());
          bk[pos] = key;
          bi[pos] = j;
        }
        n += __popc(m);
      }
      __syncwarp();
      if (lane == 0) {
        cnt[r] = n;
        thr[r] = t;
      }
      __syncwarp();
    }
  }
  __syncthreads();

  // Finalise: exact top-K, sort descending (ties -> lower index), pads.
#pragma unroll 1
  for (int rr = 0; rr < kRows / 8; ++rr) {
    const int r = warp * (kRows / 8) + rr;
    if (r >= nrows) break;
    const int g = lrow ? lrow[r] - 1 : g0 + r;
    uint32_t* bk = bkey + r * CAP;
    int* bi = bidx + r * CAP;
    int n = cnt[r];
    if (n > p.K) {
      merge_row<EPL>(bk, bi, n, p.K, lane);
      n = p.K;
    }
    uint64_t c[SE];
#pragma unroll
    for (int i = 0; i < SE; ++i) {
      const int e = i * 32 + lane;
      c[i] = (e < n) ? (((uint64_t)bk[e] << 32) | (uint32_t)(~(uint32_t)bi[e])) : 0ull;
    }
    bitonic_sort_desc<SE>(c, lane);
    int32_t* out = p.idx + ((int64_t)b * p.Tq + l0 + r) * p.K;
#pragma unroll
    for (int i = 0; i < SE; ++i) {
      const int s = i * 32 + lane;
      if (s < p.K) {
        int v;
        if (s < n) {
          v = (int)(~(uint32_t)c[i]);
        } else {
          v = p.pad_mode == 0 ? (int)(((int64_t)g + p.K + s + 1) % p.Tk) : -1;
        }
        out[s] = v;
      }
    }
  }
}

template <int EPL>
constexpr size_t smem_for(int rp) {
  return sizeof(float) * ((size_t)rp * kRows + (size_t)rp * kChunk + (size_t)kRows * kChunk) +
         2 * sizeof(int) * kRows + (size_t)kRows * 32 * EPL * (sizeof(uint32_t) + sizeof(int));
}

template <typename TI, int RP, int EPL, int SE>
int launch_t(const TopkParams& p, cudaStream_t stream) {
  const size_t smem = smem_for<EPL>(RP);
  auto kern = causal_topk_kernel<TI, RP, EPL, SE>;
  static bool configured[kMaxDevices] = {};  // per instantiation and device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev >= kMaxDevices || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    if (dev < kMaxDevices) configured[dev] = true;
  }
  TopkParams q = p;
  q.cap = 32 * EPL;
  dim3 grid((p.Tq + kRows - 1) / kRows, p.B);
  kern<<<grid, kThreads, smem, stream>>>(q);
  return (int)cudaGetLastError();
}

// K classes: (EPL, SE) with CAP = 32*EPL >= K + 64 and 32*SE >= K.
template <typename TI, int RP>
int launch_rp(const TopkParams& p, cudaStream_t s) {
  if (p.K <= 32) return launch_t<TI, RP, 3, 1>(p, s);
  if (p.K <= 64) return launch_t<TI, RP, 4, 2>(p, s);
  if (p.K <= 128) return launch_t<TI, RP, 6, 4>(p, s);
  if (p.K <= 256) return launch_t<TI, RP, 10, 8>(p, s);
  return -1;
}

template <typename TI>
int launch_ti(const TopkParams& p, cudaStream_t s) {
  if (p.R <= 32) return launch_rp<TI, 32>(p, s);
  if (p.R <= 64) return launch_rp<TI, 64>(p, s);
  if (p.R <= 128) return launch_rp<TI, 128>(p, s);
  return -1;
}

int epl_for(int K) { return K <= 32 ? 3 : K <= 64 ? 4 : K <= 128 ? 6 : K <= 256 ? 10 : 0; }
int rp_for(int R) { return R <= 32 ? 32 : R <= 64 ? 64 : R <= 128 ? 128 : 0; }

}  // namespace

size_t topk_smem_bytes(int R, int K) {
  const int epl = epl_for(K), rp = rp_for(R);
  if (!epl || !rp) return 0;
  const size_t bytes = sizeof(float) * ((size_t)rp * kRows + (size_t)rp * kChunk + (size_t)kRows * kChunk) +
                       2 * sizeof(int) * kRows + (size_t)kRows * 32 * epl * 8;
  return bytes <= 227 * 1024 ? bytes : 0;
}

int topk_max_k() { return 256; }

int launch_causal_topk(const TopkParams& p, int dtype, cudaStream_t stream) {
  // WF_TOPK_IMPL=cuda_core forces the CUDA-core scorer (used by the tests to cross-check the two kernels).
  const char* impl = getenv("WF_TOPK_IMPL");
  const bool force_cc = impl && strcmp(impl, "cuda_core") == 0;
  if (!force_cc && topk_tc_supported(p, dtype)) return launch_causal_topk_tc(p, dtype, stream);
  if (topk_smem_bytes(p.R, p.K) == 0) return -1;
  switch (dtype) {
    case kBF16: return launch_ti<__nv_bfloat16>(p, stream);
    case kF16: return launch_ti<__half>(p, stream);
    case kF32: return launch_ti<float>(p, stream);
    default: return -1;
  }
}

}  // namespace wf
