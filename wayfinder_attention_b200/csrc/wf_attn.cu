// Sparse softmax attention over retrieved K/V rows (indices shared by heads).
//
// Semantics follow routing_attention/kernels/fused_sparse.py of the reference
// (sparse_meat_attention_reference, :80-94): for every (b, h, t)
//     s_k   = <q[b,h,t], k[b,h,idx[b,t,k]]> * scale
//     p     = softmax_k(s)
//     out   = sum_k p_k * v[b,h,idx[b,t,k]]
// computed in fp32 and rounded once to the output type.  Nothing of shape
// (B,H,T,K,D) is materialised (the reference gathers it at :64-77).
//
// Design: one warp per (b, t, h); warps of a CTA share (b, t) so the index row
// is read once into L1.  A K or V row of D elements is split across G lanes,
// each loading 16-byte vectors, so 32/G retrieved rows are in flight per warp
// instruction and every 32-byte sector fetched is fully used.  Phase 1 forms
// the K scores (partial dot products reduced by xor-shuffles) into shared
// memory, phase 2 is an exact two-pass softmax over the K scores, phase 3
// accumulates p * v in fp32 registers and reduces across lane groups.
#include "wf_common.cuh"
#include "wf_kernels.h"

#include <math.h>

namespace wf {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kUnroll = 8;  // retrieved rows in flight per lane

// Index slot states after decoding.
constexpr int kMasked = -1;   // pad slot that is excluded from the softmax
constexpr int kBad = -2;      // out-of-range index: output becomes NaN

template <typename TO>
__device__ __forceinline__ void store_out(TO* o, const float* v, int n) {
#pragma unroll
  for (int i = 0; i < n; ++i) o[i] = from_f32<TO>(v[i]);
}

template <typename TI, typename TO, int D>
__global__ void __launch_bounds__(kThreads) sparse_attn_kernel(const AttnParams p) {
  using V16 = Vec16<TI>;
  constexpr int VEC = V16::N;                 // elements per 16-byte vector
  constexpr int NVROW = D / VEC;              // vectors per row
  constexpr int G = NVROW < 32 ? NVROW : 32;  // lanes per retrieved row
  constexpr int NV = NVROW / G;               // vectors per lane
  constexpr int KPP = 32 / G;                 // rows per pass
  constexpr int NE = NV * VEC;                // elements per lane

  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sS = reinterpret_cast<float*>(smem_raw) + (size_t)warp * 2 * p.K;
  int* sI = reinterpret_cast<int*>(sS + p.K);

  const int64_t w = (int64_t)blockIdx.x * kWarps + warp;
  if (w >= (int64_t)p.B * p.Tq * p.H) return;
  const int h = (int)(w % p.H);
  const int64_t bt = w / p.H;
  const int t = (int)(bt % p.Tq);
  const int b = (int)(bt / p.Tq);

  // Decode the index row.
  const int32_t* ip = p.idx + (int64_t)b * p.isb + (int64_t)t * p.ist;
  bool bad = false;
  for (int s = lane; s < p.K; s += 32) {
    int j = ip[(int64_t)s * p.iss];
    if (j < 0) {
      if (p.mask_negative) j = kMasked;
      else if (j >= -p.Tk) j += p.Tk;
      else { j = kBad; bad = true; }
    } else if (j >= p.Tk) {
      j = kBad;
      bad = true;
    }
    sI[s] = j;
  }
  if (__any_sync(kFull, bad) && lane == 0 && p.status) atomicOr(p.status, 1);

  const int sub = lane % G, grp = lane / G;
  float qf[NE];
  {
    const TI* qp = reinterpret_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)h * p.qsh +
                   (int64_t)t * p.qst;
#pragma unroll
    for (int v = 0; v < NV; ++v) V16::unpack(ldg16(qp + (sub * NV + v) * VEC), qf + v * VEC);
  }
  __syncwarp();

  const TI* kbase = reinterpret_cast<const TI*>(p.k) + (int64_t)b * p.ksb + (int64_t)h * p.ksh;
  const TI* vbase = reinterpret_cast<const TI*>(p.v) + (int64_t)b * p.vsb + (int64_t)h * p.vsh;
  const int npass = (p.K + KPP - 1) / KPP;

  // Phase 1: scores.
#pragma unroll 1
  for (int ps = 0; ps < npass; ps += kUnroll) {
    uint4 raw[kUnroll][NV];
    int jj[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int slot = (ps + u) * KPP + grp;
      const int j = (ps + u < npass && slot < p.K) ? sI[slot] : kMasked;
      jj[u] = j;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[u][v] = j >= 0 ? ldg16(kbase + (int64_t)j * p.kst + (sub * NV + v) * VEC) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float d = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float kf[VEC];
        V16::unpack(raw[u][v], kf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) d = fmaf(qf[v * VEC + e], kf[e], d);
      }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(kFull, d, o);
      const int slot = (ps + u) * KPP + grp;
      if (sub == 0 && ps + u < npass && slot < p.K) {
        const int j = jj[u];
        sS[slot] = j >= 0 ? d * p.scale : (j == kMasked ? -INFINITY : NAN);
      }
    }
  }
  __syncwarp();

  // Phase 2: softmax over the K scores (max-subtracted, like F.softmax).
  float m = -INFINITY;
  for (int s = lane; s < p.K; s += 32) m = fmaxf(m, sS[s]);
  m = warp_max(m);
  float sum = 0.f;
  for (int s = lane; s < p.K; s += 32) {
    const float x = sS[s];
    const float e = (x == -INFINITY) ? 0.f : expf(x - m);
    sS[s] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  __syncwarp();
  const float inv = 1.0f / sum;

  // Phase 3: out = sum_k p_k v_k.
  float acc[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) acc[e] = 0.f;
#pragma unroll 1
  for (int ps = 0; ps < npass; ps += kUnroll) {
    uint4 raw[kUnroll][NV];
    float pw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int slot = (ps + u) * KPP + grp;
      const bool in = ps + u < npass && slot < p.K;
      const int j = in ? sI[slot] : kMasked;
      pw[u] = in ? sS[slot] : 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[u][v] = j >= 0 ? ldg16(vbase + (int64_t)j * p.vst + (sub * NV + v) * VEC) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float vf[VEC];
        V16::unpack(raw[u][v], vf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[v * VEC + e] = fmaf(pw[u], vf[e], acc[v * VEC + e]);
      }
    }
  }
#pragma unroll
  for (int o = G; o < 32; o <<= 1)
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[e] += __shfl_xor_sync(kFull, acc[e], o);

  if (grp == 0) {
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[e] *= inv;
    TO* op = reinterpret_cast<TO*>(p.out) + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)t * p.ost;
#pragma unroll
    for (int v = 0; v < NV; ++v) store_out<TO>(op + (sub * NV + v) * VEC, acc + v * VEC, VEC);
  }
}

template <typename TI, typename TO, int D>
int launch_t(const AttnParams& p, cudaStream_t stream) {
  const int64_t work = (int64_t)p.B * p.Tq * p.H;
  const int64_t blocks = (work + kWarps - 1) / kWarps;
  const size_t smem = (size_t)kWarps * 2 * p.K * sizeof(float);
  sparse_attn_kernel<TI, TO, D><<<(unsigned)blocks, kThreads, smem, stream>>>(p);
  return (int)cudaGetLastError();
}

template <typename TI, typename TO>
int launch_d(const AttnParams& p, cudaStream_t s) {
  switch (p.D) {
    case 16: return launch_t<TI, TO, 16>(p, s);
    case 32: return launch_t<TI, TO, 32>(p, s);
    case 64: return launch_t<TI, TO, 64>(p, s);
    case 128: return launch_t<TI, TO, 128>(p, s);
    case 256: return launch_t<TI, TO, 256>(p, s);
    default: return -1;
  }
}

template <typename TI>
int launch_ti(const AttnParams& p, int out_dtype, cudaStream_t s) {
  switch (out_dtype) {
    case kBF16: return launch_d<TI, __nv_bfloat16>(p, s);
    case kF16: return launch_d<TI, __half>(p, s);
    case kF32: return launch_d<TI, float>(p, s);
    default: return -1;
  }
}

}  // namespace

int attn_max_k() { return 512; }

int launch_sparse_attention(const AttnParams& p, int dtype, int out_dtype, cudaStream_t stream) {
  if (p.K < 1 || p.K > attn_max_k()) return -1;
  switch (dtype) {
    case kBF16: return launch_ti<__nv_bfloat16>(p, out_dtype, stream);
    case kF16: return launch_ti<__half>(p, out_dtype, stream);
    case kF32: return launch_ti<float>(p, out_dtype, stream);
    default: return -1;
  }
}

}  // namespace wf
