// Exact causal top-K retrieval with tcgen05 tensor-core scoring (bf16 / fp16 addresses).
//
// Same contract as the CUDA-core kernel in wf_topk.cu (and the reference's
// routing_attention/kernels/causal_topk.py:133-171 + :37-57): for every query
// row g, the K keys j <= g with the largest fp32 score <q_g, k_j>, slots in
// descending score order with ties to the lower index, pad slots for short rows.
//
// Structure of one CTA (128 query rows = the 128 TMEM lanes, 5 warps):
//   warp 4 (producer): TMA-loads the q tile once and streams key chunks of 128
//     rows into a ring of shared-memory stages; one lane issues
//     tcgen05.mma (M=128, N=128, K=16 per instruction, fp32 accumulate) into a
//     ring of TMEM accumulators and commits to the chunk's mbarrier; the warp
//     also records the chunk's max |k| for the error margin below.
//   warps 0-3 (selection): thread t owns query row t and TMEM lane t.  It reads
//     its 128 scores of a chunk with tcgen05.ld and admits a key when the
//     tensor-core score reaches (threshold - margin).  Admitted keys are
//     rescored exactly in fp32 (sequential FMA over d, the same arithmetic as the
//     CUDA-core kernel) from the staged key rows, and only that exact score
//     enters the row's candidate buffer in shared memory.  When a buffer nears
//     capacity, the warp compacts that row to its exact top-K (radix select),
//     which raises the row's threshold.
// The margin, 2^-13 * sum_d |q_d| * max|k|, exceeds any plausible accumulation
// error of a 32-term fp32 dot product with exact products (the error bound is
// ~2^-18 of sum |q_d k_d|), so no key whose exact score beats the threshold is
// ever filtered out: the selection is exact with respect to the fp32 scores.
#include "wf_common.cuh"
#include "wf_kernels.h"
#include "wf_select.cuh"
#include "wf_sm100.cuh"

#include <type_traits>

namespace wf {
namespace {

using namespace sm100;
using select::bitonic_sort_desc;
using select::merge_row;

constexpr int kM = 128;   // query rows per CTA = TMEM lanes
constexpr int kN = 128;   // keys per chunk = MMA N
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kEpiWarps + 1) * 32;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr float kEpsScale = 1.0f / 8192.0f;
constexpr int kMaxDevices = 64;

struct TcParams {
  const void* q;  // for the exact rescoring of admitted keys
  int64_t qsb, qst;
  int B, Tq, Tk, K;
  int pad_mode;
  int rt, rs, r0;
  int32_t* idx;
  int32_t* status;
};

constexpr int stages_for(int R) { return R >= 64 ? 2 : 4; }

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <int R, int EPL>
struct Layout {
  static constexpr int ROWB = R * 2;
  static constexpr int S = stages_for(R);
  static constexpr int CAP = 32 * EPL;
  static constexpr size_t Q_BYTES = (size_t)kM * ROWB;
  static constexpr size_t STAGE_BYTES = (size_t)kN * ROWB;
  static constexpr size_t off_q = 0;
  static constexpr size_t off_k = align_up(Q_BYTES, 1024);
  static constexpr size_t off_kmax = off_k + S * align_up(STAGE_BYTES, 1024);
  static constexpr size_t off_bar = align_up(off_kmax + sizeof(float) * S, 8);
  static constexpr size_t n_bar = 3 * S + 1;
  static constexpr size_t off_misc = off_bar + 8 * n_bar;  // tmem base, abort flag
  static constexpr size_t off_bkey = align_up(off_misc + 16, 16);
  static constexpr size_t KEY_STRIDE = CAP + 1;  // words; odd stride keeps row-private appends conflict-free
  static constexpr size_t IDX_STRIDE = CAP + 2;  // halfwords
  static constexpr size_t off_bidx = off_bkey + sizeof(uint32_t) * kM * KEY_STRIDE;
  static constexpr size_t bytes = off_bidx + sizeof(uint16_t) * kM * IDX_STRIDE;
  static constexpr size_t smem = bytes + 1024;  // slack to align the dynamic base
};

template <typename TI>
__device__ __forceinline__ float rescore(const float* qf, const unsigned char* row, int j, int rowb) {
  // Key row j of a stage stored with the TMA swizzle matching `rowb` (32/64/128 B):
  // 16-byte chunk c lives at chunk c ^ ((j * rowb >> 7) & (rowb / 16 - 1)).
  const int sw = (j * rowb >> 7) & (rowb / 16 - 1);
  float acc = 0.f;
  for (int c = 0; c < rowb / 16; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(row + ((c ^ sw) << 4));
    float f[8];
    Vec16<TI>::unpack(w, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(qf[c * 8 + e], f[e], acc);
  }
  return acc;
}

template <typename TI, int R, int EPL, int SE>
__global__ void __launch_bounds__(kThreads, 1)
    causal_topk_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                          const TcParams p) {
  using L = Layout<R, EPL>;
  constexpr int S = L::S;
  constexpr int ROWB = L::ROWB;
  constexpr int CAP = L::CAP;
  constexpr int KSTEPS = R / 16;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t IDESC = idesc_f16(sizeof(TI) == 2 && !std::is_same<TI, __half>::value, kM, kN);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = base + L::off_q;
  unsigned char* ks = base + L::off_k;
  float* kmax_s = reinterpret_cast<float*>(base + L::off_kmax);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L::off_bar);
  uint64_t* mdone = full + S;
  uint64_t* empty = mdone + S;
  uint64_t* qbar = empty + S;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(base + L::off_misc);
  int* abort_s = reinterpret_cast<int*>(base + L::off_misc + 4);
  uint32_t* bkey = reinterpret_cast<uint32_t*>(base + L::off_bkey);
  uint16_t* bidx = reinterpret_cast<uint16_t*>(base + L::off_bidx);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile = (p.Tq + kM - 1) / kM;
  const int tile = ntile - 1 - (int)blockIdx.x;  // heaviest tiles first
  const int b = blockIdx.y;
  const int l0 = tile * kM;
  const int nrows = min(kM, p.Tq - l0);
  const int g0 = ((l0 / p.rt) * p.rs + p.r0) * p.rt + (l0 % p.rt);
  const int key_end = min(g0 + nrows, p.Tk);
  const int nchunks = (key_end + kN - 1) / kN;

  if (warp == kEpiWarps && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&mdone[s], 2);
      mbar_init(&empty[s], kEpiWarps);
    }
    mbar_init(qbar, 1);
    *abort_s = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_base_s, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == kEpiWarps) {
    // ------------------------------------------------------------ producer
    bool ok = true;
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      mbar_arrive_expect_tx(qbar, (uint32_t)L::Q_BYTES);
      tma_load_3d(qs, &qmap, qbar, 0, l0, b);
      for (int c = 0; c < min(S, nchunks); ++c) {
        mbar_arrive_expect_tx(&full[c], (uint32_t)L::STAGE_BYTES);
        tma_load_3d(ks + c * align_up(L::STAGE_BYTES, 1024), &kmap, &full[c], 0, c * kN, b);
      }
    }
    ok = mbar_wait(qbar, 0, kWaitLimitNs);
    for (int c = 0; c < nchunks && ok; ++c) {
      const int s = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      unsigned char* stage = ks + s * align_up(L::STAGE_BYTES, 1024);
      if (!mbar_wait(&full[s], ph, kWaitLimitNs)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t d = tmem_base + (uint32_t)(s * kN);
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const uint64_t a = smem_desc_kmajor(smem_u32(qs) + kk * 32, ROWB);
          const uint64_t bd = smem_desc_kmajor(smem_u32(stage) + kk * 32, ROWB);
          mma_f16(d, a, bd, IDESC, kk > 0);
        }
        mma_commit(&mdone[s]);
      }
      // max |k| over the staged rows (bit patterns of non-negative floats order like values)
      uint32_t m2 = 0;
      const uint4* v = reinterpret_cast<const uint4*>(stage);
      for (int i = lane; i < (int)(L::STAGE_BYTES / 16); i += 32) {
        const uint4 w = v[i];
        m2 = __vmaxu2(m2, w.x & 0x7fff7fffu);
        m2 = __vmaxu2(m2, w.y & 0x7fff7fffu);
        m2 = __vmaxu2(m2, w.z & 0x7fff7fffu);
        m2 = __vmaxu2(m2, w.w & 0x7fff7fffu);
      }
      uint32_t mb = max(m2 & 0xffffu, m2 >> 16);
      mb = __reduce_max_sync(kFullMask, mb);
      if (lane == 0) {
        float km;
        if (std::is_same<TI, __half>::value) km = __half2float(__ushort_as_half((unsigned short)mb));
        else km = __uint_as_float(mb << 16);
        kmax_s[s] = km;
        mbar_arrive(&mdone[s]);
      }
      // refill the stage that chunk c-1 used once its consumers are done
      const int cn = c - 1 + S;
      if (c >= 1 && cn < nchunks) {
        const int s1 = (c - 1) % S;
        if (!mbar_wait(&empty[s1], (uint32_t)((c - 1) / S) & 1u, kWaitLimitNs)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s1], (uint32_t)L::STAGE_BYTES);
          tma_load_3d(ks + s1 * align_up(L::STAGE_BYTES, 1024), &kmap, &full[s1], 0, cn * kN, b);
        }
      }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      *abort_s = 1;
      if (p.status) atomicOr(p.status, 2);
    }
  } else {
    // ------------------------------------------------------------ selection
    const int r = threadIdx.x;  // row within the tile = TMEM lane
    const bool row_ok = r < nrows;
    const int g = g0 + r;
    float qf[R];
    float qabs = 0.f;
    {
      const TI* qrow = reinterpret_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)(l0 + (row_ok ? r : 0)) * p.qst;
#pragma unroll
      for (int c = 0; c < R / 8; ++c) {
        float f[8];
        Vec16<TI>::unpack(ldg16(qrow + c * 8), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          qf[c * 8 + e] = row_ok ? f[e] : 0.f;
          qabs += fabsf(qf[c * 8 + e]);
        }
      }
    }
    uint32_t* mykey = bkey + r * L::KEY_STRIDE;
    uint16_t* myidx = bidx + r * L::IDX_STRIDE;
    int cnt = 0;
    bool have_thr = false;
    uint32_t thr_key = 0;
    float thr_f = -INFINITY;
    bool ok = true;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

    for (int c = 0; c < nchunks; ++c) {
      const int s = c % S;
      const uint32_t ph = (uint32_t)(c / S) & 1u;
      if (!mbar_wait(&mdone[s], ph, kWaitLimitNs) || !mbar_wait(&full[s], ph, kWaitLimitNs)) { ok = false; break; }
      tc_fence_after();
      const float eps = kEpsScale * qabs * kmax_s[s];
      const float lim = have_thr ? thr_f - eps : -INFINITY;
      const unsigned char* stage = ks + s * align_up(L::STAGE_BYTES, 1024);
#pragma unroll 1
      for (int sl = 0; sl < kN / 32; ++sl) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + lane_base + (uint32_t)(s * kN + sl * 32), v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (__uint_as_float(v[j]) >= lim) {
            const int jj = sl * 32 + j;
            const int key = c * kN + jj;
            if (row_ok && key <= g) {
              const float ex = rescore<TI>(qf, stage + jj * ROWB, jj, ROWB);
              const uint32_t kk = ordered_key(ex);
              if (!have_thr || kk > thr_key) {
                mykey[cnt] = kk;
                myidx[cnt] = (uint16_t)key;
                ++cnt;
              }
            }
          }
        }
        unsigned need = __ballot_sync(kFullMask, cnt > CAP - 32);
        while (need) {
          const int ln = __ffs(need) - 1;
          need &= need - 1;
          const int rr = 32 * warp + ln;
          const int n = __shfl_sync(kFullMask, cnt, ln);
          const uint32_t tau = merge_row<EPL>(bkey + rr * L::KEY_STRIDE, bidx + rr * L::IDX_STRIDE, n, p.K, lane);
          if (lane == ln) {
            cnt = p.K;
            thr_key = tau;
            thr_f = key_to_float(tau);
            have_thr = true;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok && lane == 0) {
      *abort_s = 1;
      if (p.status) atomicOr(p.status, 2);
    }

    // Finalise each row of this warp: exact top-K, sorted, pads.
    for (int ln = 0; ln < 32; ++ln) {
      const int rr = 32 * warp + ln;
      if (rr >= nrows) break;
      int n = __shfl_sync(kFullMask, cnt, ln);
      uint32_t* bk = bkey + rr * L::KEY_STRIDE;
      uint16_t* bi = bidx + rr * L::IDX_STRIDE;
      if (n > p.K) {
        merge_row<EPL>(bk, bi, n, p.K, lane);
        n = p.K;
      }
      uint64_t cc[SE];
#pragma unroll
      for (int i = 0; i < SE; ++i) {
        const int e = i * 32 + lane;
        cc[i] = (e < n) ? (((uint64_t)bk[e] << 32) | (uint32_t)(~(uint32_t)bi[e])) : 0ull;
      }
      bitonic_sort_desc<SE>(cc, lane);
      const int gg = g0 + rr;
      int32_t* out = p.idx + ((int64_t)b * p.Tq + l0 + rr) * p.K;
#pragma unroll
      for (int i = 0; i < SE; ++i) {
        const int s = i * 32 + lane;
        if (s < p.K) {
          int val;
          if (s < n) val = (int)(~(uint32_t)cc[i]);
          else val = p.pad_mode == 0 ? (int)(((int64_t)gg + p.K + s + 1) % p.Tk) : -1;
          out[s] = val;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_map(CUtensorMap* map, const void* ptr, bool bf16, int R, int64_t T, int64_t B, int64_t st, int64_t sb,
              int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)R, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)(st * 2), (cuuint64_t)(sb * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)R, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = R == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : R == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult rc = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return rc == CUDA_SUCCESS;
}

template <typename TI, int R, int EPL, int SE>
int launch_t(const TopkParams& p, cudaStream_t stream) {
  using L = Layout<R, EPL>;
  auto kern = causal_topk_tc_kernel<TI, R, EPL, SE>;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev >= kMaxDevices || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::smem);
    if (e != cudaSuccess) return (int)e;
    if (dev < kMaxDevices) configured[dev] = true;
  }
  const bool bf16 = !std::is_same<TI, __half>::value;
  CUtensorMap qmap, kmap;
  if (!make_map(&qmap, p.q, bf16, R, p.Tq, p.B, p.qst, p.qsb, kM)) return -1;
  if (!make_map(&kmap, p.k, bf16, R, p.Tk, p.B, p.kst, p.ksb, kN)) return -1;
  TcParams t{};
  t.q = p.q;
  t.qsb = p.qsb;
  t.qst = p.qst;
  t.B = p.B; t.Tq = p.Tq; t.Tk = p.Tk; t.K = p.K;
  t.pad_mode = p.pad_mode;
  t.rt = p.rt; t.rs = p.rs; t.r0 = p.r0;
  t.idx = p.idx;
  t.status = p.status;
  dim3 grid((p.Tq + kM - 1) / kM, p.B);
  kern<<<grid, kThreads, L::smem, stream>>>(qmap, kmap, t);
  return (int)cudaGetLastError();
}

template <typename TI, int R>
int launch_r(const TopkParams& p, cudaStream_t s) {
  if (p.K <= 32) return launch_t<TI, R, 4, 1>(p, s);
  if (p.K <= 64) return launch_t<TI, R, 5, 2>(p, s);
  if (p.K <= 128) return launch_t<TI, R, 7, 4>(p, s);
  return -1;
}

template <typename TI>
int launch_ti(const TopkParams& p, cudaStream_t s) {
  switch (p.R) {
    case 16: return launch_r<TI, 16>(p, s);
    case 32: return launch_r<TI, 32>(p, s);
    case 64: return launch_r<TI, 64>(p, s);
    default: return -1;
  }
}

}  // namespace

bool topk_tc_supported(const TopkParams& p, int dtype) {
  if (dtype != kBF16 && dtype != kF16) return false;
  if (p.R != 16 && p.R != 32 && p.R != 64) return false;
  if (p.K > 128 || p.Tk > 65536 || p.B > 65535) return false;
  if (p.qsr != 1 || p.ksr != 1) return false;
  if ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k)) % 16) return false;
  if ((p.qst * 2) % 16 || (p.kst * 2) % 16 || (p.qsb * 2) % 16 || (p.ksb * 2) % 16) return false;
  const bool identity = p.rs == 1 && p.r0 == 0;
  if (!identity && p.rt % kM) return false;
  return encode_fn() != nullptr;
}

int launch_causal_topk_tc(const TopkParams& p, int dtype, cudaStream_t stream) {
  if (dtype == kBF16) return launch_ti<__nv_bfloat16>(p, stream);
  if (dtype == kF16) return launch_ti<__half>(p, stream);
  return -1;
}

}  // namespace wf
