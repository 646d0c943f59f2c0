// Fused learned-address projection: out = normalize_g(x W^T + b).
//
// Replaces LearnedAddressModule.forward_query_key (reference
// routing_attention/models/learned_address.py:39-46): two nn.Linear(d_model, d_A)
// projections followed by F.normalize(dim=-1) on each.  The two weight matrices
// are stacked into one (N = 2*d_A, or d_A for the symmetric module) so a single
// pass over the hidden states produces both addresses; each consecutive group of
// `group` outputs is L2-normalised as F.normalize does: v / max(||v||_2, 1e-12).
//
// bf16 / fp16 inputs: tcgen05.  A CTA owns 128 rows (the TMEM lanes).  Thread 0
// streams 64-column slices of the x tile (128 x 64) and of W (N x 64) with TMA
// (128-byte swizzle) through a 4-stage ring and issues tcgen05.mma kind::f16
// (M=128, N, K=16, fp32 accumulate) into N TMEM columns; after the last slice the
// four warps read their 32 lanes back, add the bias, normalise in fp32 and store
// in the input type.  Bounded waits: a timeout sets status bit 1 (plus 4..16).
// fp32 inputs (and shapes the TMA path does not cover): a CUDA-core kernel with
// the same per-row arithmetic (sequential fp32 FMA over d_model).
//
// The fusion stops at the addresses: the scoring kernel reads every key address
// from about T/256 query tiles, so recomputing addresses inside it from x would
// multiply the projection work by that factor.
#include "wf_common.cuh"
#include "wf_kernels.h"
#include "wf_sm100.cuh"

#include <cuda.h>
#include <type_traits>

namespace wf {
namespace {

using namespace sm100;

constexpr int kPM = 128;      // rows per CTA
constexpr int kPK = 64;       // d_model columns per stage (128 bytes of bf16)
constexpr int kPStages = 4;
constexpr uint64_t kPWaitNs = 1000000000ull;

struct ProjParams {
  const void* bias;  // [N] in the input type, or null
  void* out;         // [M][out_stride]
  int64_t out_stride;
  int M, K, N, group, normalize;
  int32_t* status;
};

template <int N>
struct ProjLayout {
  static constexpr size_t X_BYTES = (size_t)kPM * 128;
  static constexpr size_t W_BYTES = (size_t)N * 128;
  static constexpr size_t STAGE = X_BYTES + W_BYTES;  // multiple of 1024
  static constexpr size_t off_bar = kPStages * STAGE;
  static constexpr size_t off_misc = off_bar + 8 * (2 * kPStages + 1);
  static constexpr size_t off_bias = (off_misc + 16 + 15) / 16 * 16;
  static constexpr size_t bytes = off_bias + 4 * (size_t)N;
  static constexpr size_t smem = bytes + 1024;
  static constexpr uint32_t TMEM_COLS = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32_t(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32_t<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32_t<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f32_t<float>(float v) { return v; }

template <typename T, int N>
__global__ void __launch_bounds__(128, 1)
    addr_proj_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                        const ProjParams p) {
  using L = ProjLayout<N>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L::off_bar);
  uint64_t* empty = full + kPStages;
  uint64_t* done = empty + kPStages;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(base + L::off_misc);
  float* bias_s = reinterpret_cast<float*>(base + L::off_bias);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kPM;
  const int nk = (p.K + kPK - 1) / kPK;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = idesc_f16(kBf16, kPM, N);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbarrier_init();
  }
  for (int i = threadIdx.x; i < N; i += blockDim.x)
    bias_s[i] = p.bias ? to_f32<T>(static_cast<const T*>(p.bias)[i]) : 0.f;
  if (warp == 0) {
    tmem_alloc(tmem_base_s, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  uint32_t why = 0;

  if (threadIdx.x == 0) {
    // TMA producer and MMA issuer in one thread: the ring is refilled as soon as
    // the MMAs that read a stage have completed.
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
    auto load = [&](int kc) {
      const int s = kc % kPStages;
      unsigned char* st = base + s * L::STAGE;
      mbar_arrive_expect_tx(&full[s], (uint32_t)L::STAGE);
      tma_load_3d(st, &xmap, &full[s], kc * kPK, row0, 0);
      tma_load_3d(st + L::X_BYTES, &wmap, &full[s], kc * kPK, 0, 0);
    };
    for (int kc = 0; kc < nk && kc < kPStages; ++kc) load(kc);
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % kPStages;
      if (!mbar_wait(&full[s], (uint32_t)(kc / kPStages) & 1u, kPWaitNs)) { why |= 4; break; }
      tc_fence_after();
      const uint32_t xs = smem_u32(base + s * L::STAGE), ws = xs + (uint32_t)L::X_BYTES;
#pragma unroll
      for (int kk = 0; kk < kPK / 16; ++kk)
        mma_f16(tmem, smem_desc_kmajor(xs + kk * 32, 128), smem_desc_kmajor(ws + kk * 32, 128), IDESC,
                kc > 0 || kk > 0);
      mma_commit(&empty[s]);
      if (kc + kPStages < nk) {
        if (!mbar_wait(&empty[s], (uint32_t)(kc / kPStages) & 1u, kPWaitNs)) { why |= 8; break; }
        load(kc + kPStages);
      }
    }
    mma_commit(done);
  }
  __syncwarp();
  // epilogue: warp w reads TMEM lanes 32w..32w+31 (= rows row0 + 32w + lane)
  bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0, kPWaitNs));
  if (!ok) why |= 16;
  tc_fence_after();
  const int row = row0 + 32 * warp + lane;
  const uint32_t lbase = tmem + ((uint32_t)(32 * warp) << 16);
  // one 32-column slice at a time; every address group lies within a slice (group | 32)
  T* o = static_cast<T*>(p.out) + (int64_t)row * p.out_stride;
#pragma unroll 1
  for (int c = 0; c < N; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(lbase + c, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + bias_s[c + j];
    if (p.normalize) {
      for (int g0 = 0; g0 < 32; g0 += p.group) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j >= g0 && j < g0 + p.group) ss = fmaf(v[j], v[j], ss);
        const float nrm = fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j >= g0 && j < g0 + p.group) v[j] = v[j] / nrm;
      }
    }
    if (ok && row < p.M) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          *reinterpret_cast<__nv_bfloat162*>(o + c + j) = __floats2bfloat162_rn(v[j], v[j + 1]);
        } else {
          *reinterpret_cast<__half2*>(o + c + j) = __floats2half2_rn(v[j], v[j + 1]);
        }
      }
    }
  }
  if (why && p.status && lane == 0) atomicOr(p.status, 2 | (int)why);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// CUDA-core form: block = 256 threads = (256 / N) rows x N outputs; thread (r, o)
// computes the dot product of row r with weight row o (sequential fp32 FMA over
// d_model, weights staged in shared memory 64 columns at a time), and the `group`
// threads of an address normalise together with shuffles.
constexpr int kCcK = 64;
template <typename T>
__global__ void __launch_bounds__(256) addr_proj_cc_kernel(const T* __restrict__ x, int64_t x_stride,
                                                           const T* __restrict__ w, ProjParams p) {
  extern __shared__ float wt[];  // [kCcK][N] transposed weight slice
  const int N = p.N, K = p.K;
  const int rows_per_block = blockDim.x / N;
  const int o = threadIdx.x % N;
  const int row = blockIdx.x * rows_per_block + threadIdx.x / N;
  const bool live = threadIdx.x < rows_per_block * N && row < p.M;
  const T* xr = x + (int64_t)(live ? row : 0) * x_stride;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += kCcK) {
    const int kn = min(kCcK, K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < N * kn; i += blockDim.x) {
      const int oo = i / kn, d = i % kn;
      wt[d * N + oo] = to_f32<T>(w[(size_t)oo * K + k0 + d]);
    }
    __syncthreads();
    if (live)
      for (int d = 0; d < kn; ++d) acc = fmaf(to_f32<T>(xr[k0 + d]), wt[d * N + o], acc);
  }
  if (live && p.bias) acc += to_f32<T>(static_cast<const T*>(p.bias)[o]);
  if (p.normalize) {
    float ss = acc * acc;
    for (int off = p.group / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off, p.group);
    acc = acc / fmaxf(sqrtf(ss), 1e-12f);
  }
  if (live) static_cast<T*>(p.out)[(int64_t)row * p.out_stride + o] = from_f32_t<T>(acc);
}

typedef CUresult (*EncodeTiledFnP)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnP encode_fn_p() {
  static EncodeTiledFnP fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnP>(ptr);
  }
  return fn;
}

// rows x cols matrix (row stride in elements), box of box_rows x 64 columns, 128-byte swizzle
bool make_rows_map(CUtensorMap* map, const void* ptr, bool bf16, int64_t rows, int64_t cols, int64_t stride,
                   int box_rows) {
  EncodeTiledFnP fn = encode_fn_p();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, 1};
  const cuuint64_t strides[2] = {(cuuint64_t)(stride * 2), (cuuint64_t)(stride * 2 * rows)};
  const cuuint32_t box[3] = {(cuuint32_t)kPK, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int N>
int launch_tc(const void* x, int64_t x_stride, const void* w, const ProjParams& p, cudaStream_t stream) {
  using L = ProjLayout<N>;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap xmap, wmap;
  if (!make_rows_map(&xmap, x, bf16, p.M, p.K, x_stride, kPM)) return -1;
  if (!make_rows_map(&wmap, w, bf16, N, p.K, p.K, N)) return -1;
  auto kern = addr_proj_tc_kernel<T, N>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::smem);
  if (e != cudaSuccess) return (int)e;
  kern<<<(unsigned)((p.M + kPM - 1) / kPM), 128, L::smem, stream>>>(xmap, wmap, p);
  return (int)cudaGetLastError();
}

template <typename T>
int launch_cc(const void* x, int64_t x_stride, const void* w, const ProjParams& p, cudaStream_t stream) {
  const size_t smem = (size_t)p.N * kCcK * sizeof(float);  // at most 64 KB (N <= 256)
  auto kern = addr_proj_cc_kernel<T>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
  }
  const int rows_per_block = 256 / p.N;
  kern<<<(unsigned)((p.M + rows_per_block - 1) / rows_per_block), 256, smem, stream>>>(
      static_cast<const T*>(x), x_stride, static_cast<const T*>(w), p);
  return (int)cudaGetLastError();
}

template <typename T>
int launch_tc_n(const void* x, int64_t x_stride, const void* w, const ProjParams& p, cudaStream_t s) {
  switch (p.N) {
    case 32: return launch_tc<T, 32>(x, x_stride, w, p, s);
    case 64: return launch_tc<T, 64>(x, x_stride, w, p, s);
    case 128: return launch_tc<T, 128>(x, x_stride, w, p, s);
    default: return -1;
  }
}

}  // namespace

int launch_address_projection(const void* x, int dtype, int64_t M, int K, int64_t x_stride, const void* w,
                              const void* bias, int N, int group, int normalize, void* out, int64_t out_stride,
                              int32_t* status, cudaStream_t stream) {
  ProjParams p{};
  p.bias = bias;
  p.out = out;
  p.out_stride = out_stride;
  p.M = (int)M;
  p.K = K;
  p.N = N;
  p.group = group;
  p.normalize = normalize;
  p.status = status;
  const bool tc_ok = dtype != kF32 && (N == 32 || N == 64 || N == 128) &&
                     (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) % 16 == 0 &&
                     (x_stride * 2) % 16 == 0 && (K * 2) % 16 == 0 && (out_stride * 2) % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 4 == 0 && encode_fn_p() != nullptr;
  if (tc_ok) {
    if (dtype == kBF16) return launch_tc_n<__nv_bfloat16>(x, x_stride, w, p, stream);
    return launch_tc_n<__half>(x, x_stride, w, p, stream);
  }
  if (dtype == kBF16) return launch_cc<__nv_bfloat16>(x, x_stride, w, p, stream);
  if (dtype == kF16) return launch_cc<__half>(x, x_stride, w, p, stream);
  return launch_cc<float>(x, x_stride, w, p, stream);
}

}  // namespace wf
