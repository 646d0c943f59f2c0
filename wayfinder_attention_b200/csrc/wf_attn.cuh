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
// Design.  Indices are shared by the heads, so one warp serves one query and a
// group of heads: each lane owns E consecutive elements (16-byte vectors) of one
// head's row, L = D/E lanes cover a head and 32/L heads share the warp.  For
// every retrieved key the index and row address are computed once for all those
// heads, and the K and V rows of all of them are read with coalesced 16-byte
// loads (lane `sub` of a head owns vectors sub, sub+L, ... so each load
// instruction covers whole sectors) (in the module's (B,T,H,D) layout the heads of one key are contiguous).
//   phase 1: partial dot products over the lane's E elements, reduced over the
//            L lanes of the head by xor-shuffles; one score per (head, key) to
//            shared memory;
//   phase 2: exact two-pass softmax per head (max-subtracted, like F.softmax);
//   phase 3: acc[E] += p * v in fp32 registers; the lane already owns its output
//            elements, so no cross-lane reduction is needed.
// The loop over keys is the same for K and V; a lane keeps U rows in flight.
//
// This header holds the kernel and its launch templates; each input dtype is
// instantiated in its own translation unit (wf_attn_<dtype>.cu) so they compile in parallel.
#pragma once
#include "wf_common.cuh"
#include "wf_kernels.h"

#include <math.h>

namespace wf {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kU = 4;  // retrieved rows in flight per lane

// Index slot states after decoding.
constexpr int kMasked = -1;  // pad slot that is excluded from the softmax
constexpr int kBad = -2;     // out-of-range index: output becomes NaN

template <typename TO>
__device__ __forceinline__ void store_vec(TO* o, const float* v, int n) {
#pragma unroll
  for (int i = 0; i < n; ++i) o[i] = from_f32<TO>(v[i]);
}
template <>
__device__ __forceinline__ void store_vec<__nv_bfloat16>(__nv_bfloat16* o, const float* v, int n) {
  for (int i = 0; i < n; i += 8) {
    uint4 w;
    uint32_t* u = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[i + 2 * e], v[i + 2 * e + 1]);
      u[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(o + i) = w;
  }
}
template <>
__device__ __forceinline__ void store_vec<float>(float* o, const float* v, int n) {
  for (int i = 0; i < n; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}

// Element offset of decoded key slot j (see the decode step) for row stride st.
template <bool CYC>
__device__ __forceinline__ int64_t kv_row_offset(const AttnParams& p, int j, int64_t st, int64_t rank_stride) {
  if (!CYC) return (int64_t)j * st;
  return (int64_t)(j >> 25) * rank_stride + (int64_t)(j & ((1 << 25) - 1)) * st;
}

// CYC: keys live in rank-major gathered blocks (kv_world > 1); a separate
// instantiation keeps the address arithmetic of the plain layout minimal.
template <typename TI, typename TO, int D, int E, bool CYC, bool DROP>
__global__ void __launch_bounds__(256) sparse_attn_kernel(const AttnParams p, int warps_per_block) {
  pdl_wait();
  using V16 = Vec16<TI>;
  constexpr int VEC = V16::N;
  constexpr int NV = E / VEC;       // 16-byte vectors per lane and row
  constexpr int L = D / E;          // lanes per head
  constexpr int HW = 32 / L;        // heads per warp

  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.K;
  // Score row stride: with K a multiple of 32 and L >= 4 lanes per head, K + L puts
  // the heads' rows L banks apart (conflict-free in phase 2) and 16-byte aligned, so
  // phase 3 reads four probabilities (and both phases four indices) per access;
  // otherwise an odd stride keeps the rows in different banks.
  const bool vec = L >= 4 && (K & 31) == 0;
  const int KP = vec ? K + L : (K | 1);
  int* sI = reinterpret_cast<int*>(smem_raw) + (size_t)warp * (K + HW * KP);
  float* sP = reinterpret_cast<float*>(sI + K);  // [HW][KP]

  const int ngroups = (p.H + HW - 1) / HW;
  const int64_t w = (int64_t)blockIdx.x * warps_per_block + warp;
  if (w >= (int64_t)p.B * p.Tq * ngroups) return;
  // Warps walk the queries of one (batch element, head group) before the next: the
  // rows in flight then gather from that group's K/V only (H*D/ngroups of every
  // key row), which stays in L2 far longer than all heads' rows at long T (cfg4:
  // 134 MB per group against 1.07 GB for all 32 heads).
  const int t = (int)(w % p.Tq);
  const int64_t bg = w / p.Tq;
  const int hg = (int)(bg % ngroups);
  const int b = (int)(bg / ngroups);
  const int hl = lane / L;        // head within the warp
  const int sub = lane % L;
  const int h = hg * HW + hl;
  const bool hv = h < p.H;
  const int hc = hv ? h : 0;      // clamp for address arithmetic of idle lanes

  // Decode the index row once for all heads.
  const int32_t* ip = p.idx + (int64_t)b * p.isb + (int64_t)t * p.ist;
  bool bad = false;
  for (int s = lane; s < K; s += 32) {
    int j = ip[(int64_t)s * p.iss];
    if (j < 0) {
      if (p.mask_negative) j = kMasked;
      else if (j >= -p.Tk) j += p.Tk;
      else { j = kBad; bad = true; }
    } else if (j >= p.Tk) {
      j = kBad;
      bad = true;
    }
    if (CYC && j >= 0) {
      // rank-major gathered keys: rank r's rows follow each other, r < kv_world <= 64,
      // stored as r * 2^25 + local row (Tk < 2^25 is checked by the caller)
      const int blk = j / p.kv_tile;
      int blk_id = blk % p.kv_world;
      int lr = (blk / p.kv_world) * p.kv_tile + j % p.kv_tile;
      if (p.kv_chunk_rows > 0) {  // chunk-major: block (chunk, rank)
        const int c = lr / p.kv_chunk_rows;
        lr -= c * p.kv_chunk_rows;
        blk_id += c * p.kv_world;
      }
      j = (blk_id << 25) | lr;
    }
    sI[s] = j;
  }
  if (__any_sync(kFull, bad) && lane == 0 && p.status) atomicOr(p.status, 1);

  float qf[E];
  {
    const TI* qp = reinterpret_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)hc * p.qsh +
                   (int64_t)t * p.qst;
#pragma unroll
    for (int v = 0; v < NV; ++v) V16::unpack(ldg16(qp + (v * L + sub) * VEC), qf + v * VEC);
  }
  __syncwarp();

  // Lane `sub` of a head owns vectors sub, sub + L, ... of the row, so one load
  // instruction reads whole 32-byte sectors.
  const TI* kb = reinterpret_cast<const TI*>(p.k) + (int64_t)b * p.ksb + (int64_t)hc * p.ksh + sub * VEC;
  const TI* vb = reinterpret_cast<const TI*>(p.v) + (int64_t)b * p.vsb + (int64_t)hc * p.vsh + sub * VEC;
  float* myP = sP + hl * KP;

  // Phase 1: scores, and each head's running maximum (every lane of a head holds the
  // reduced scores, so the maximum costs no pass over shared memory).
  float m = -INFINITY;
#pragma unroll 1
  for (int k0 = 0; k0 < K; k0 += kU) {
    uint4 raw[kU][NV];
    int jj[kU];
    if (vec) {
      const int4 j4 = *reinterpret_cast<const int4*>(sI + k0);
      jj[0] = j4.x; jj[1] = j4.y; jj[2] = j4.z; jj[3] = j4.w;
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u) jj[u] = (k0 + u < K) ? sI[k0 + u] : kMasked;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = jj[u];
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[u][v] = (j >= 0 && hv) ? ldg16(kb + kv_row_offset<CYC>(p, j, p.kst, p.k_rank_stride) + v * L * VEC) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float d = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float kf[VEC];
        V16::unpack(raw[u][v], kf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) d = fmaf(qf[v * VEC + e], kf[e], d);
      }
#pragma unroll
      for (int o = L / 2; o > 0; o >>= 1) d += __shfl_xor_sync(kFull, d, o);
      if (k0 + u < K) {
        const int j = jj[u];
        const float sv = j >= 0 ? d * p.scale : (j == kMasked ? -INFINITY : NAN);
        m = fmaxf(m, sv);  // a NaN score (bad index) leaves m alone; the sum below turns NaN
        if (sub == 0) myP[k0 + u] = sv;
      }
    }
  }
  __syncwarp();

  // Phase 2: exponentials and their sum per head; the L lanes of a head share the work.
  float sum = 0.f;
  for (int s = sub; s < K; s += L) {
    const float x = myP[s];
    const float e = (x == -INFINITY) ? 0.f : expf(x - m);
    myP[s] = e;
    sum += e;
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  __syncwarp();
  const float inv = 1.0f / sum;

  // Phase 3: out = sum_k p_k v_k over the lane's own E elements.
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  const uint64_t drow = DROP ? (((uint64_t)b * p.H + (uint64_t)hc) * p.Tq + (uint64_t)t) * (uint64_t)K : 0;
  const float inv_keep = DROP ? 1.0f / (1.0f - p.drop_rate) : 1.0f;
#pragma unroll 1
  for (int k0 = 0; k0 < K; k0 += kU) {
    uint4 raw[kU][NV];
    float pw[kU];
    int jj[kU];
    if (vec) {
      const int4 j4 = *reinterpret_cast<const int4*>(sI + k0);
      const float4 p4 = *reinterpret_cast<const float4*>(myP + k0);
      jj[0] = j4.x; jj[1] = j4.y; jj[2] = j4.z; jj[3] = j4.w;
      pw[0] = p4.x; pw[1] = p4.y; pw[2] = p4.z; pw[3] = p4.w;
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const bool in = k0 + u < K;
        jj[u] = in ? sI[k0 + u] : kMasked;
        pw[u] = in ? myP[k0 + u] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const bool in = k0 + u < K;
      const int j = jj[u];
      if (DROP && in) pw[u] *= dropout_scale(p.drop_seed, drow + (uint64_t)(k0 + u), p.drop_rate, inv_keep);
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[u][v] = (j >= 0 && hv) ? ldg16(vb + kv_row_offset<CYC>(p, j, p.vst, p.v_rank_stride) + v * L * VEC) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float vf[VEC];
        V16::unpack(raw[u][v], vf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[v * VEC + e] = fmaf(pw[u], vf[e], acc[v * VEC + e]);
      }
    }
  }
  if (hv) {
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] *= inv;
    TO* op = reinterpret_cast<TO*>(p.out) + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)t * p.ost;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      TO* o = op + (v * L + sub) * VEC;
      if (p.out_vec_ok) store_vec<TO>(o, acc + v * VEC, VEC);
      else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = from_f32<TO>(acc[v * VEC + e]);
      }
    }
  }
}

constexpr size_t kSmemBudget = 96 * 1024;

template <typename TI, typename TO, int D, int E>
int launch_t(const AttnParams& p, cudaStream_t stream) {
  constexpr int L = D / E;
  constexpr int HW = 32 / L;
  const int ngroups = (p.H + HW - 1) / HW;
  const bool vec = L >= 4 && (p.K & 31) == 0;  // the kernel's score-row stride rule
  const size_t per_warp = ((size_t)p.K + (size_t)HW * (vec ? p.K + L : (p.K | 1))) * sizeof(int);
  int wpb = (int)(kSmemBudget / per_warp);
  wpb = wpb < 1 ? 1 : (wpb > 8 ? 8 : wpb);
  const size_t smem = per_warp * wpb;
  auto kern = p.kv_world > 1 ? sparse_attn_kernel<TI, TO, D, E, true, false>
              : p.drop_rate > 0.f ? sparse_attn_kernel<TI, TO, D, E, false, true>
                                  : sparse_attn_kernel<TI, TO, D, E, false, false>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
  }
  const int64_t work = (int64_t)p.B * p.Tq * ngroups;
  const int64_t blocks = (work + wpb - 1) / wpb;
  const cudaError_t e = launch_pdl(kern, dim3((unsigned)blocks), dim3(wpb * 32), smem, stream, p, wpb);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// E: elements per lane.  16 when the heads of a query span at least 512
// elements (every lane busy), else 8; never more than D.
template <typename TI, typename TO, int D>
int launch_e(const AttnParams& p, cudaStream_t s) {
  constexpr int EMIN = 16 / sizeof(TI);  // one 16-byte vector
  constexpr int E16 = D < 16 ? D : 16;
  constexpr int E8 = D < 8 ? D : 8;
  constexpr int EA = E16 < EMIN ? EMIN : E16;
  constexpr int EB = E8 < EMIN ? EMIN : E8;
  if ((int64_t)p.H * D >= 32 * EA) return launch_t<TI, TO, D, EA>(p, s);
  return launch_t<TI, TO, D, EB>(p, s);
}

template <typename TI, typename TO>
int launch_d(const AttnParams& p, cudaStream_t s) {
  switch (p.D) {
    case 16: return launch_e<TI, TO, 16>(p, s);
    case 32: return launch_e<TI, TO, 32>(p, s);
    case 64: return launch_e<TI, TO, 64>(p, s);
    case 128: return launch_e<TI, TO, 128>(p, s);
    case 256: return launch_e<TI, TO, 256>(p, s);
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
}  // namespace wf
