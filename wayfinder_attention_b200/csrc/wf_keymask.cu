// Causal top-K retrieval that skips padded keys.
//
// The reference's sparse attention accepts a (B, T) key-padding mask
// (TransformerLM passes `input_ids != pad_token_id`, models/transformer.py:269-284)
// and ignores it (models/attention.py:456-490), while its dense attention masks
// those keys (attention.py:157-167).  This path honours it: a query may retrieve
// only keys j <= t whose mask is set.
//
// Instead of testing a mask bit per score inside the scoring kernels, the valid
// keys of every sequence are compacted first:
//   keymask_scan_kernel     per batch element: inclusive prefix count of the mask
//                           (lim[t] = number of valid keys j <= t) and the map
//                           compacted position -> original position;
//   keymask_compact_kernel  copies the valid key addresses to a dense
//                           (B, T, R) buffer (rows past the count are zeroed);
//   top-K                   the usual kernels on the compacted keys, with query row t
//                           limited to compacted keys c < lim[t] (TopkParams::lim),
//                           pads masked (-1) where fewer than K keys are valid;
//   keymask_remap_kernel    compacted indices back to original positions.
// The mask and the compaction cost two small passes over B*T entries.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {
namespace {

__global__ void __launch_bounds__(1024) keymask_scan_kernel(const uint8_t* mask, int64_t msb, int64_t mst, int T,
                                                            int32_t* lim, int32_t* map) {
  __shared__ int wsum[32];
  const int b = blockIdx.x;
  const uint8_t* m = mask + (int64_t)b * msb;
  int32_t* lb = lim + (int64_t)b * T;
  int32_t* mb = map + (int64_t)b * T;
  const int per = (T + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(lo + per, T);
  int local = 0;
  for (int j = lo; j < hi; ++j) local += m[(int64_t)j * mst] != 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int x = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    wsum[lane] = x;
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? wsum[warp - 1] : 0);
  for (int j = lo; j < hi; ++j) {
    if (m[(int64_t)j * mst] != 0) {
      mb[run] = j;
      ++run;
    }
    lb[j] = run;
  }
}

template <typename T>
__global__ void keymask_compact_kernel(const T* k, int64_t ksb, int64_t kst, int64_t ksr, int B, int Tn, int R,
                                       const int32_t* lim, const int32_t* map, T* kc) {
  const int64_t n = (int64_t)B * Tn * R;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e % R);
    const int64_t bc = e / R;
    const int c = (int)(bc % Tn), b = (int)(bc / Tn);
    const int count = lim[(int64_t)b * Tn + Tn - 1];
    T v = from_f32<T>(0.f);
    if (c < count) v = k[(int64_t)b * ksb + (int64_t)map[(int64_t)b * Tn + c] * kst + (int64_t)r * ksr];
    kc[e] = v;
  }
}

__global__ void keymask_remap_kernel(int32_t* idx, int64_t n, int K, int Tn, const int32_t* map) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int v = idx[e];
    const int64_t b = e / ((int64_t)Tn * K);
    if (v >= 0) idx[e] = map[b * Tn + v];
  }
}

size_t al256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

size_t topk_key_mask_prep_bytes(int64_t B, int64_t T, int R, int esz) {
  return al256((size_t)B * T * R * esz) + 2 * al256((size_t)B * T * 4);
}

int launch_topk_key_mask(TopkParams p, int dtype, const uint8_t* mask, int64_t msb, int64_t mst, void* prep,
                         cudaStream_t stream) {
  const int T = p.Tq;  // Tq == Tk
  const int esz = dtype == kF32 ? 4 : 2;
  unsigned char* c = static_cast<unsigned char*>(prep);
  void* kc = c;
  int32_t* lim = reinterpret_cast<int32_t*>(c + al256((size_t)p.B * T * p.R * esz));
  int32_t* map = lim + al256((size_t)p.B * T * 4) / 4;
  keymask_scan_kernel<<<p.B, 1024, 0, stream>>>(mask, msb, mst, T, lim, map);
  const int64_t n = (int64_t)p.B * T * p.R;
  const unsigned grid = (unsigned)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  if (dtype == kBF16)
    keymask_compact_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(p.k), p.ksb, p.kst,
        p.ksr, p.B, T, p.R, lim, map, static_cast<__nv_bfloat16*>(kc));
  else if (dtype == kF16)
    keymask_compact_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(p.k), p.ksb, p.kst, p.ksr, p.B,
        T, p.R, lim, map, static_cast<__half*>(kc));
  else
    keymask_compact_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(p.k), p.ksb, p.kst, p.ksr, p.B, T,
        p.R, lim, map, static_cast<float*>(kc));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  p.k = kc;
  p.ksb = (int64_t)T * p.R;
  p.kst = p.R;
  p.ksr = 1;
  p.lim = lim;
  p.pad_mode = 1;
  int rc = launch_causal_topk(p, dtype, stream);
  if (rc) return rc;
  const int64_t ni = (int64_t)p.B * T * p.K;
  const unsigned gi = (unsigned)((ni + 255) / 256 < 148 * 16 ? (ni + 255) / 256 : 148 * 16);
  keymask_remap_kernel<<<gi, 256, 0, stream>>>(p.idx, ni, p.K, T, map);
  return (int)cudaGetLastError();
}

}  // namespace wf
