// Backward of the sparse softmax attention over retrieved rows.
//
// Forward (wf_attn.cuh; reference routing_attention/kernels/fused_sparse.py:80-94):
//   s_k = scale * <q_t, k_{idx_k}>,  p = softmax_k(s),  out_t = sum_k p_k v_{idx_k}
// Gradients for dO = dL/dout (the indices come from top-K and carry none):
//   dp_k = <dO_t, v_{idx_k}>,  D_t = sum_k p_k dp_k,  ds_k = p_k (dp_k - D_t)
//   dq_t      = scale * sum_k ds_k k_{idx_k}
//   dk_j     += scale * ds_k q_t      for every (t, k) with idx_k = j
//   dv_j     += p_k dO_t              for every (t, k) with idx_k = j
// This is the gradient the reference's non-fused training path gets from
// autograd through its gather (models/attention.py:35-56).
//
// Three steps, none of them with floating-point atomics:
//   1. attn_bwd_query_kernel: one warp per (query, group of heads), the lane
//      mapping of the forward kernel.  It recomputes the scores and softmax from a
//      K gather, gathers V for dp, forms ds, writes dq from a second K gather and
//      stores p and scale*ds per (query, slot, head) in the workspace.
//   2. csr_*: the inverse of the index: for every key j the list of (t, k) slots
//      that retrieved it (count, per-batch exclusive scan, fill).
//   3. attn_bwd_key_kernel: one warp per (key, group of heads) walks its list and
//      accumulates dk and dv in fp32 registers, then writes each row once (keys
//      nobody retrieved get zeros).  The order inside a list depends on the fill's
//      atomics, so dk/dv sums may differ in the last bits between runs, like
//      PyTorch's scatter-add backward of a gather.
#include "wf_common.cuh"
#include "wf_kernels.h"

#include <math.h>
#include <type_traits>

namespace wf {
namespace {

constexpr unsigned kFullB = 0xffffffffu;
constexpr int kUB = 4;          // rows in flight per lane
constexpr int kMaskedB = -1;
constexpr int kBadB = -2;

template <typename TO>
__device__ __forceinline__ void store_row(TO* o, const float* v, int n, bool vec_ok) {
  if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
    if (vec_ok) {
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
      return;
    }
  } else if constexpr (std::is_same<TO, float>::value) {
    if (vec_ok) {
      for (int i = 0; i < n; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      return;
    }
  }
  for (int i = 0; i < n; ++i) o[i] = from_f32<TO>(v[i]);
}

__device__ __forceinline__ int decode_slot(int j, const AttnBwdParams& p, bool& bad) {
  if (j < 0) {
    if (p.mask_negative) return kMaskedB;
    if (j >= -p.Tk) return j + p.Tk;
    bad = true;
    return kBadB;
  }
  if (j >= p.Tk) {
    bad = true;
    return kBadB;
  }
  return j;
}

template <typename TI, typename TG, int D, int E>
__global__ void __launch_bounds__(256) attn_bwd_query_kernel(const AttnBwdParams p, int warps_per_block) {
  using V16 = Vec16<TI>;
  constexpr int VEC = V16::N;
  constexpr int NV = E / VEC;
  constexpr int L = D / E;
  constexpr int HW = 32 / L;

  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.K;
  // As in the forward: with K a multiple of 32 and L >= 4, rows K + L apart are
  // 16-byte aligned and bank-disjoint, and indices / coefficients are read 4 at a time.
  const bool vec = L >= 4 && (K & 31) == 0;
  const int KP = vec ? K + L : (K | 1);
  int* sI = reinterpret_cast<int*>(smem_raw) + (size_t)warp * (K + 2 * HW * KP);
  float* sP = reinterpret_cast<float*>(sI + K);  // [HW][KP] scores, then p
  float* sD = sP + HW * KP;                      // [HW][KP] dp, then scale * ds

  const int ngroups = (p.H + HW - 1) / HW;
  const int64_t w = (int64_t)blockIdx.x * warps_per_block + warp;
  if (w >= (int64_t)p.B * p.Tq * ngroups) return;
  // one (batch element, head group) at a time, as in the forward (L2 locality at long T)
  const int t = (int)(w % p.Tq);
  const int64_t bg = w / p.Tq;
  const int hg = (int)(bg % ngroups);
  const int b = (int)(bg / ngroups);
  const int hl = lane / L, sub = lane % L;
  const int h = hg * HW + hl;
  const bool hv = h < p.H;
  const int hc = hv ? h : 0;

  const int32_t* ip = p.idx + (int64_t)b * p.isb + (int64_t)t * p.ist;
  bool bad = false;
  for (int s = lane; s < K; s += 32) sI[s] = decode_slot(ip[(int64_t)s * p.iss], p, bad);
  if (__any_sync(kFullB, bad) && lane == 0 && p.status) atomicOr(p.status, 1);

  float qf[E], gf[E];
  {
    const TI* qp = static_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)hc * p.qsh + (int64_t)t * p.qst;
    const TI* gp = static_cast<const TI*>(p.dout) + (int64_t)b * p.osb + (int64_t)hc * p.osh + (int64_t)t * p.ost;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      V16::unpack(ldg16(qp + (v * L + sub) * VEC), qf + v * VEC);
      V16::unpack(ldg16(gp + (v * L + sub) * VEC), gf + v * VEC);
    }
  }
  __syncwarp();
  const TI* kb = static_cast<const TI*>(p.k) + (int64_t)b * p.ksb + (int64_t)hc * p.ksh + sub * VEC;
  const TI* vb = static_cast<const TI*>(p.v) + (int64_t)b * p.vsb + (int64_t)hc * p.vsh + sub * VEC;
  float* myP = sP + hl * KP;
  float* myD = sD + hl * KP;

  // dot of the lane's E elements of `x` with gathered rows, reduced over the head's L lanes
  auto gather_dot = [&](const TI* base, int64_t st, const float* x, float* dst, bool scale_it) {
#pragma unroll 1
    for (int k0 = 0; k0 < K; k0 += kUB) {
      uint4 raw[kUB][NV];
      int jj[kUB];
      if (vec) {
        const int4 j4 = *reinterpret_cast<const int4*>(sI + k0);
        jj[0] = j4.x; jj[1] = j4.y; jj[2] = j4.z; jj[3] = j4.w;
      } else {
#pragma unroll
        for (int u = 0; u < kUB; ++u) jj[u] = (k0 + u < K) ? sI[k0 + u] : kMaskedB;
      }
#pragma unroll
      for (int u = 0; u < kUB; ++u) {
        const int j = jj[u];
#pragma unroll
        for (int v = 0; v < NV; ++v)
          raw[u][v] = (j >= 0 && hv) ? ldg16(base + (int64_t)j * st + v * L * VEC) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kUB; ++u) {
        float d = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          float f[VEC];
          V16::unpack(raw[u][v], f);
#pragma unroll
          for (int e = 0; e < VEC; ++e) d = fmaf(x[v * VEC + e], f[e], d);
        }
#pragma unroll
        for (int o = L / 2; o > 0; o >>= 1) d += __shfl_xor_sync(kFullB, d, o);
        if (sub == 0 && k0 + u < K) {
          const int j = jj[u];
          dst[k0 + u] = j >= 0 ? (scale_it ? d * p.scale : d) : (scale_it ? -INFINITY : 0.f);
        }
      }
    }
    __syncwarp();
  };

  // 1. scores and softmax (the forward's arithmetic)
  gather_dot(kb, p.kst, qf, myP, true);
  float m = -INFINITY;
  for (int s = sub; s < K; s += L) m = fmaxf(m, myP[s]);
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullB, m, o));
  float sum = 0.f;
  for (int s = sub; s < K; s += L) {
    const float x = myP[s];
    const float e = (x == -INFINITY) ? 0.f : expf(x - m);
    myP[s] = e;
    sum += e;
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(kFullB, sum, o);
  const float inv = sum > 0.f ? 1.0f / sum : 0.f;
  __syncwarp();
  // 2. dp_k = <dO, v_k>
  gather_dot(vb, p.vst, gf, myD, false);
  // With dropout the forward weighted v_k by p_k z_k, z_k = keep / (1 - rate): the
  // gradient with respect to p_k is dp_k z_k, and dv uses p_k z_k.
  const bool drop = p.drop_rate > 0.f;
  const uint64_t drow = (((uint64_t)b * p.H + (uint64_t)hc) * p.Tq + (uint64_t)t) * (uint64_t)K;
  const float inv_keep = drop ? 1.0f / (1.0f - p.drop_rate) : 1.0f;
  float dsum = 0.f;
  for (int s = sub; s < K; s += L) {
    const float pk = myP[s] * inv;
    myP[s] = pk;
    if (drop) myD[s] *= dropout_scale(p.drop_seed, drow + (uint64_t)s, p.drop_rate, inv_keep);
    dsum = fmaf(pk, myD[s], dsum);
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) dsum += __shfl_xor_sync(kFullB, dsum, o);
  // 3. scale * ds_k, and both coefficients for the key-side kernel ([b][t][k][h])
  float* Pg = p.P + ((int64_t)b * p.Tq + t) * K * p.H;
  float* Dg = p.DS + ((int64_t)b * p.Tq + t) * K * p.H;
  for (int s = sub; s < K; s += L) {
    const float pk = myP[s];
    const float dsk = p.scale * pk * (myD[s] - dsum);
    myD[s] = dsk;
    if (hv) {
      Pg[(int64_t)s * p.H + h] = drop ? pk * dropout_scale(p.drop_seed, drow + (uint64_t)s, p.drop_rate, inv_keep) : pk;
      Dg[(int64_t)s * p.H + h] = dsk;
    }
  }
  __syncwarp();
  // 4. dq = sum_k (scale * ds_k) k_k
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
#pragma unroll 1
  for (int k0 = 0; k0 < K; k0 += kUB) {
    uint4 raw[kUB][NV];
    float cw[kUB];
    int jj[kUB];
    if (vec) {
      const int4 j4 = *reinterpret_cast<const int4*>(sI + k0);
      const float4 c4 = *reinterpret_cast<const float4*>(myD + k0);
      jj[0] = j4.x; jj[1] = j4.y; jj[2] = j4.z; jj[3] = j4.w;
      cw[0] = c4.x; cw[1] = c4.y; cw[2] = c4.z; cw[3] = c4.w;
    } else {
#pragma unroll
      for (int u = 0; u < kUB; ++u) {
        const bool in = k0 + u < K;
        jj[u] = in ? sI[k0 + u] : kMaskedB;
        cw[u] = in ? myD[k0 + u] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUB; ++u) {
      const int j = jj[u];
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[u][v] = (j >= 0 && hv) ? ldg16(kb + (int64_t)j * p.kst + v * L * VEC) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUB; ++u)
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float f[VEC];
        V16::unpack(raw[u][v], f);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[v * VEC + e] = fmaf(cw[u], f[e], acc[v * VEC + e]);
      }
  }
  if (hv) {
    TG* o = static_cast<TG*>(p.dq) + (int64_t)b * p.dqsb + (int64_t)h * p.dqsh + (int64_t)t * p.dqst;
#pragma unroll
    for (int v = 0; v < NV; ++v) store_row<TG>(o + (v * L + sub) * VEC, acc + v * VEC, VEC, p.dq_vec_ok);
  }
}

// --- inverse index -----------------------------------------------------------
__global__ void csr_count_kernel(const AttnBwdParams p) {
  const int64_t n = (int64_t)p.B * p.Tq * p.K;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e % p.K);
    const int64_t bt = e / p.K;
    const int t = (int)(bt % p.Tq), b = (int)(bt / p.Tq);
    bool bad = false;
    const int j = decode_slot(p.idx[(int64_t)b * p.isb + (int64_t)t * p.ist + (int64_t)k * p.iss], p, bad);
    if (j >= 0) atomicAdd(&p.cnt[(int64_t)b * p.Tk + j], 1);
  }
}

// One block per batch element: exclusive scan of the counts into off[b][0..Tk],
// then the counts are zeroed to serve as fill cursors.
__global__ void __launch_bounds__(1024) csr_scan_kernel(const AttnBwdParams p) {
  __shared__ int wsum[32];
  const int b = blockIdx.x;
  int32_t* c = p.cnt + (int64_t)b * p.Tk;
  int32_t* off = p.off + (int64_t)b * (p.Tk + 1);
  const int per = (p.Tk + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(lo + per, p.Tk);
  int local = 0;
  for (int j = lo; j < hi; ++j) local += c[j];
  // block exclusive scan of `local`
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullB, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int x = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullB, x, o);
      if (lane >= o) x += y;
    }
    wsum[lane] = x;  // inclusive over warps
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? wsum[warp - 1] : 0);
  for (int j = lo; j < hi; ++j) {
    off[j] = run;
    run += c[j];
    c[j] = 0;
  }
  if (threadIdx.x == blockDim.x - 1) off[p.Tk] = run;
}

__global__ void csr_fill_kernel(const AttnBwdParams p) {
  const int64_t n = (int64_t)p.B * p.Tq * p.K;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e % p.K);
    const int64_t bt = e / p.K;
    const int t = (int)(bt % p.Tq), b = (int)(bt / p.Tq);
    bool bad = false;
    const int j = decode_slot(p.idx[(int64_t)b * p.isb + (int64_t)t * p.ist + (int64_t)k * p.iss], p, bad);
    if (j < 0) continue;
    const int64_t kj = (int64_t)b * p.Tk + j;
    const int pos = p.off[(int64_t)b * (p.Tk + 1) + j] + atomicAdd(&p.cnt[kj], 1);
    p.list[(int64_t)b * p.Tq * p.K + pos] = (t << 9) | k;  // K <= 512
  }
}

// --- key side ----------------------------------------------------------------
template <typename TI, typename TG, int D, int E>
__global__ void __launch_bounds__(128, 4) attn_bwd_key_kernel(const AttnBwdParams p) {
  using V16 = Vec16<TI>;
  constexpr int VEC = V16::N;
  constexpr int NV = E / VEC;
  constexpr int L = D / E;
  constexpr int HW = 32 / L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = (p.H + HW - 1) / HW;
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (w >= (int64_t)p.B * p.Tk * ngroups) return;
  const int hg = (int)(w % ngroups);
  const int64_t bj = w / ngroups;
  const int j = (int)(bj % p.Tk);
  const int b = (int)(bj / p.Tk);
  const int hl = lane / L, sub = lane % L;
  const int h = hg * HW + hl;
  const bool hv = h < p.H;
  const int hc = hv ? h : 0;
  const int32_t* off = p.off + (int64_t)b * (p.Tk + 1);
  const int e0 = off[j], e1 = off[j + 1];
  const int32_t* lst = p.list + (int64_t)b * p.Tq * p.K;
  const TI* qb = static_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)hc * p.qsh + sub * VEC;
  const TI* gb = static_cast<const TI*>(p.dout) + (int64_t)b * p.osb + (int64_t)hc * p.osh + sub * VEC;
  const float* Pb = p.P + (int64_t)b * p.Tq * p.K * p.H;
  const float* Db = p.DS + (int64_t)b * p.Tq * p.K * p.H;
  float dk[E], dv[E];
#pragma unroll
  for (int e = 0; e < E; ++e) dk[e] = dv[e] = 0.f;
  constexpr int KU = sizeof(TI) == 4 ? 2 : kUB;  // fp32 rows are twice as many registers
  // list entries (t << 9 | slot) of the next batch are loaded one batch ahead
  int nxt[KU];
#pragma unroll
  for (int u = 0; u < KU; ++u) nxt[u] = e0 + u < e1 ? lst[e0 + u] : -1;
#pragma unroll 1
  for (int e = e0; e < e1; e += KU) {
    int cur[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      cur[u] = nxt[u];
      nxt[u] = e + KU + u < e1 ? lst[e + KU + u] : -1;
    }
    uint4 rq[KU][NV], rg[KU][NV];
    float cp[KU], cd[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const bool in = cur[u] >= 0 && hv;
      const int t = cur[u] >> 9;
      const int64_t ci = ((int64_t)t * p.K + (cur[u] & 511)) * p.H + h;
      cp[u] = in ? Pb[ci] : 0.f;
      cd[u] = in ? Db[ci] : 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        rq[u][v] = in ? ldg16(qb + (int64_t)t * p.qst + v * L * VEC) : make_uint4(0, 0, 0, 0);
        rg[u][v] = in ? ldg16(gb + (int64_t)t * p.ost + v * L * VEC) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u)
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float fq[VEC], fg[VEC];
        V16::unpack(rq[u][v], fq);
        V16::unpack(rg[u][v], fg);
#pragma unroll
        for (int x = 0; x < VEC; ++x) {
          dk[v * VEC + x] = fmaf(cd[u], fq[x], dk[v * VEC + x]);
          dv[v * VEC + x] = fmaf(cp[u], fg[x], dv[v * VEC + x]);
        }
      }
  }
  if (hv) {
    TG* odk = static_cast<TG*>(p.dk) + (int64_t)b * p.dksb + (int64_t)h * p.dksh + (int64_t)j * p.dkst;
    TG* ov = static_cast<TG*>(p.dv) + (int64_t)b * p.dvsb + (int64_t)h * p.dvsh + (int64_t)j * p.dvst;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      store_row<TG>(odk + (v * L + sub) * VEC, dk + v * VEC, VEC, p.dk_vec_ok);
      store_row<TG>(ov + (v * L + sub) * VEC, dv + v * VEC, VEC, p.dv_vec_ok);
    }
  }
}

constexpr size_t kBwdSmemBudget = 96 * 1024;

template <typename TI, typename TG, int D, int E>
int launch_bwd_t(const AttnBwdParams& p, cudaStream_t stream) {
  constexpr int L = D / E;
  constexpr int HW = 32 / L;
  const int ngroups = (p.H + HW - 1) / HW;
  const bool vec = L >= 4 && (p.K & 31) == 0;  // the kernel's row-stride rule
  const size_t per_warp = ((size_t)p.K + 2 * (size_t)HW * (vec ? p.K + L : (p.K | 1))) * sizeof(int);
  int wpb = (int)(kBwdSmemBudget / per_warp);
  wpb = wpb < 1 ? 1 : (wpb > 8 ? 8 : wpb);
  const size_t smem = per_warp * wpb;
  auto qk = attn_bwd_query_kernel<TI, TG, D, E>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(qk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
  }
  const int64_t qwork = (int64_t)p.B * p.Tq * ngroups;
  qk<<<(unsigned)((qwork + wpb - 1) / wpb), wpb * 32, smem, stream>>>(p, wpb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  // inverse index
  e = cudaMemsetAsync(p.cnt, 0, sizeof(int32_t) * (size_t)p.B * p.Tk, stream);
  if (e != cudaSuccess) return (int)e;
  const int64_t n = (int64_t)p.B * p.Tq * p.K;
  const unsigned eg = (unsigned)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  csr_count_kernel<<<eg, 256, 0, stream>>>(p);
  csr_scan_kernel<<<p.B, 1024, 0, stream>>>(p);
  csr_fill_kernel<<<eg, 256, 0, stream>>>(p);
  const int64_t kwork = (int64_t)p.B * p.Tk * ngroups;
  attn_bwd_key_kernel<TI, TG, D, E><<<(unsigned)((kwork + 3) / 4), 128, 0, stream>>>(p);
  return (int)cudaGetLastError();
}

template <typename TI, typename TG, int D>
int launch_bwd_e(const AttnBwdParams& p, cudaStream_t s) {
  constexpr int EMIN = 16 / sizeof(TI);
  constexpr int EA = 16 < EMIN ? EMIN : 16;
  constexpr int EB = 8 < EMIN ? EMIN : 8;
  if ((int64_t)p.H * D >= 32 * EA) return launch_bwd_t<TI, TG, D, EA>(p, s);
  return launch_bwd_t<TI, TG, D, EB>(p, s);
}

template <typename TI, typename TG>
int launch_bwd_d(const AttnBwdParams& p, cudaStream_t s) {
  switch (p.D) {
    case 32: return launch_bwd_e<TI, TG, 32>(p, s);
    case 64: return launch_bwd_e<TI, TG, 64>(p, s);
    case 128: return launch_bwd_e<TI, TG, 128>(p, s);
    default: return -1;
  }
}

template <typename TI>
int launch_bwd_ti(const AttnBwdParams& p, int grad_dtype, cudaStream_t s) {
  if (grad_dtype == kF32) return launch_bwd_d<TI, float>(p, s);
  if (grad_dtype == kBF16 && std::is_same<TI, __nv_bfloat16>::value) return launch_bwd_d<TI, TI>(p, s);
  if (grad_dtype == kF16 && std::is_same<TI, __half>::value) return launch_bwd_d<TI, TI>(p, s);
  return -1;
}

}  // namespace

size_t attn_bwd_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t Tk, int K) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t coef = al((size_t)B * Tq * K * H * sizeof(float));
  return 2 * coef + al((size_t)B * Tk * 4) + al((size_t)B * (Tk + 1) * 4) + al((size_t)B * Tq * K * 4);
}

int launch_sparse_attention_backward(AttnBwdParams p, void* ws, size_t ws_bytes, int dtype, int grad_dtype,
                                     cudaStream_t stream) {
  if (p.D != 32 && p.D != 64 && p.D != 128) return -1;
  if (p.K < 1 || p.K > 512) return -1;
  const size_t need = attn_bwd_workspace_bytes(p.B, p.H, p.Tq, p.Tk, p.K);
  if (!ws || ws_bytes < need || reinterpret_cast<uintptr_t>(ws) % 256) return -3;
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  unsigned char* c = static_cast<unsigned char*>(ws);
  const size_t coef = al((size_t)p.B * p.Tq * p.K * p.H * sizeof(float));
  p.P = reinterpret_cast<float*>(c);
  p.DS = reinterpret_cast<float*>(c + coef);
  p.cnt = reinterpret_cast<int32_t*>(c + 2 * coef);
  p.off = reinterpret_cast<int32_t*>(c + 2 * coef + al((size_t)p.B * p.Tk * 4));
  p.list = reinterpret_cast<int32_t*>(c + 2 * coef + al((size_t)p.B * p.Tk * 4) + al((size_t)p.B * (p.Tk + 1) * 4));
  switch (dtype) {
    case kBF16: return launch_bwd_ti<__nv_bfloat16>(p, grad_dtype, stream);
    case kF16: return launch_bwd_ti<__half>(p, grad_dtype, stream);
    case kF32: return launch_bwd_ti<float>(p, grad_dtype, stream);
    default: return -1;
  }
}

}  // namespace wf
