// Shared device helpers for the Wayfinder sm_100a kernels.
//
// Element types, the order-preserving float -> uint32 map used by the top-K
// selector, and warp reductions.  Everything here is plain CUDA C++; the
// tensor-core scoring path adds its own PTX wrappers in wf_tc.cuh.
#pragma once
#include <utility>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace wf {

// Programmatic dependent launch: a kernel launched with launch_pdl may start while
// the previous kernel on the stream finishes its last blocks; it calls pdl_wait()
// before touching any memory, which returns once that kernel has completed and its
// writes are visible.  (Without the launch attribute pdl_wait returns at once.)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}


// Matches the WF_DTYPE_* constants of include/wayfinder.h.
enum Dtype : int { kBF16 = 0, kF16 = 1, kF32 = 2 };

__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Unpack a 16-byte vector of T into floats.  N = 16 / sizeof(T).
template <typename T> struct Vec16;
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Vec16<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <> struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    f[0] = __uint_as_float(r.x);
    f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z);
    f[3] = __uint_as_float(r.w);
  }
};

// Read-only 16-byte global load (K/V rows are never written by the kernel).
__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Order-preserving map: a > b (as floats, -0 == +0)  <=>  key(a) > key(b).
// Key 0 is never produced by a finite or infinite value, so it serves as the
// "empty slot" sentinel in the selector.
__device__ __forceinline__ uint32_t ordered_key(float f) {
  uint32_t u = (f == 0.0f) ? 0u : __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Attention-probability dropout: uniform in [0, 1) for element `idx` of the
// (B, H, Tq, K) probability tensor under `seed`, from the SplitMix64 output
// function (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) applied to seed + (idx + 1) * golden-ratio increment;
// 24 high bits.  Counter-based, so the backward recomputes the forward's mask.
__host__ __device__ __forceinline__ float dropout_uniform(uint64_t seed, uint64_t idx) {
  uint64_t z = seed + (idx + 1ull) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}
// Multiplier of a kept (1 / (1 - rate)) or dropped (0) probability.
__device__ __forceinline__ float dropout_scale(uint64_t seed, uint64_t idx, float rate, float inv_keep) {
  return dropout_uniform(seed, idx) >= rate ? inv_keep : 0.f;
}

}  // namespace wf
