// Warp-cooperative selection primitives shared by the top-K kernels.
#pragma once

#include <climits>
#include <stdint.h>

#include "wf_common.cuh"

namespace wf {
namespace select {

constexpr unsigned kFull = 0xffffffffu;

// Select the exact top-K (by ordered key, ties -> lower index) among the n > K
// entries of one row's buffer and compact them to positions [0, K).
// Returns the K-th key, the new admission threshold.
// Register form: kk/ii hold n > K candidates spread as element e = i*32 + lane
// (empty slots: key 0).  Writes the exact top-K (ties -> lower index) to
// bk/bi[0, K) and returns the K-th key.
template <int EPL, typename IdxT>
__device__ __forceinline__ uint32_t select_compact(const uint32_t (&kk)[EPL], const int (&ii)[EPL], int n, int K,
                                                   int lane, uint32_t* bk, IdxT* bi) {
  // tau = largest value with #(key >= tau) >= K, i.e. the K-th largest key.
  // It shares every bit above the highest bit in which min and max differ.
  uint32_t mn = 0xffffffffu, mx = 0u;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    if (i * 32 + lane < n) {
      mn = min(mn, kk[i]);
      mx = max(mx, kk[i]);
    }
  }
  mn = __reduce_min_sync(kFull, mn);
  mx = __reduce_max_sync(kFull, mx);
  const uint32_t diff = mn ^ mx;
  const int top = diff ? 31 - __clz(diff) : -1;
  uint32_t tau = top >= 0 ? (mn & ~(uint32_t)((2ull << top) - 1)) : mn;
#pragma unroll 1
  for (int bit = top; bit >= 0; --bit) {
    const uint32_t cand = tau | (1u << bit);
    unsigned c = 0;
#pragma unroll
    for (int i = 0; i < EPL; ++i) c += (kk[i] >= cand) ? 1u : 0u;
    c = __reduce_add_sync(kFull, c);
    if (c >= (unsigned)K) tau = cand;
  }
  unsigned gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    gt += (kk[i] > tau) ? 1u : 0u;
    eq += (kk[i] == tau) ? 1u : 0u;
  }
  gt = __reduce_add_sync(kFull, gt);
  eq = __reduce_add_sync(kFull, eq);
  const unsigned need = (unsigned)K - gt;  // 1 <= need <= eq
  int lim = INT_MAX;                        // keep tied entries with index <= lim
  if (need < eq) {
    int last = -1;
#pragma unroll 1
    for (unsigned t = 0; t < need; ++t) {
      int m = INT_MAX;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (kk[i] == tau && ii[i] > last) m = min(m, ii[i]);
      last = __reduce_min_sync(kFull, m);
    }
    lim = last;
  }
  __syncwarp();
  unsigned base = 0;
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const bool take = kk[i] > tau || (kk[i] == tau && ii[i] <= lim);
    const unsigned m = __ballot_sync(kFull, take);
    if (take) {
      const unsigned pos = base + __popc(m & lt);
      bk[pos] = kk[i];
      bi[pos] = (IdxT)ii[i];
    }
    base += __popc(m);
  }
  __syncwarp();
  return tau;
}

template <int EPL, typename IdxT>
__device__ __forceinline__ uint32_t merge_row(uint32_t* bk, IdxT* bi, int n, int K, int lane) {
  uint32_t kk[EPL];
  int ii[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    const bool in = e < n;
    kk[i] = in ? bk[e] : 0u;
    ii[i] = in ? (int)bi[e] : INT_MAX;
  }
  __syncwarp();
  return select_compact<EPL, IdxT>(kk, ii, n, K, lane, bk, bi);
}

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int o) {
  const uint32_t lo = __shfl_xor_sync(kFull, (uint32_t)v, o);
  const uint32_t hi = __shfl_xor_sync(kFull, (uint32_t)(v >> 32), o);
  return ((uint64_t)hi << 32) | lo;
}

// Warp bitonic sort, descending, of 32*SE 64-bit values; element e lives in
// register e / 32 of lane e % 32.
template <int SE>
__device__ __forceinline__ void bitonic_sort_desc(uint64_t (&c)[SE], int lane) {
  constexpr int S = 32 * SE;
#pragma unroll
  for (int size = 2; size <= S; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int rs = stride >> 5;
#pragma unroll
        for (int i = 0; i < SE; ++i) {
          if ((i & rs) == 0) {
            const int j = i | rs;
            const int e = i * 32 + lane;
            const bool desc = (e & size) == 0;
            const uint64_t a = c[i], b = c[j];
            const bool sw = desc ? (a < b) : (a > b);
            c[i] = sw ? b : a;
            c[j] = sw ? a : b;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < SE; ++i) {
          const int e = i * 32 + lane;
          const uint64_t o = shfl_xor64(c[i], stride);
          const bool lower = (lane & stride) == 0;
          const bool desc = (e & size) == 0;
          const bool keep_max = (lower == desc);
          c[i] = keep_max ? (c[i] > o ? c[i] : o) : (c[i] < o ? c[i] : o);
        }
      }
    }
  }
}

}  // namespace select
}  // namespace wf
