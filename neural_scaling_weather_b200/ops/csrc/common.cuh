// Shared device helpers for the sm_100a kernels of neural_scaling_weather_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsw {

// Device-side error word: kernels that give up a bounded wait or see an out-of-range
// index record a code here instead of trapping; the host reads and clears it.
enum ErrorCode : int {
  kErrNone = 0,
  kErrWaitTimeout = 1,
  kErrBounds = 2,
  kErrBadArg = 3,
};

__device__ __forceinline__ void record_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

template <typename T>
struct Vec8;  // 8 x 16-bit values in one 16-byte register group

__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

// unpack/pack 8 16-bit floats from/to a uint4.  The vector is taken by value: a reference to
// a shared- or global-memory uint4 read through a 16-bit pointer can compile to eight 2-byte
// loads (eight times the wavefronts, bank-conflicted) instead of one 16-byte load.
__device__ __forceinline__ void unpack2(uint32_t w, float* f, __nv_bfloat16) {
  f[0] = __uint_as_float(w << 16);
  f[1] = __uint_as_float(w & 0xFFFF0000u);
}
__device__ __forceinline__ void unpack2(uint32_t w, float* f, __half) {
  __half2 h;
  memcpy(&h, &w, 4);
  const float2 v = __half22float2(h);
  f[0] = v.x;
  f[1] = v.y;
}
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 u, float* f) {
  unpack2(u.x, f, T());
  unpack2(u.y, f + 2, T());
  unpack2(u.z, f + 4, T());
  unpack2(u.w, f + 6, T());
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f<T>(f[i]);
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Exact (erf-based) GELU, as torch.nn.GELU() with approximate='none' (CUDA's erff).
__device__ __forceinline__ float gelu_f(float u) {
  return 0.5f * u * (1.0f + erff(u * 0.70710678118654752440f));
}
__device__ __forceinline__ float gelu_grad_f(float u) {
  const float cdf = 0.5f * (1.0f + erff(u * 0.70710678118654752440f));
  const float pdf = expf(-0.5f * u * u) * 0.39894228040143267794f;
  return cdf + u * pdf;
}

// Fast erf-based GELU for GEMM epilogues.  erf(z) for z >= 0 uses Abramowitz & Stegun,
// Handbook of Mathematical Functions, eq. 7.1.26 (Hastings' rational approximation,
// |error| <= 1.5e-7):  erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2),
// t = 1 / (1 + p z); odd symmetry gives z < 0.  With z = u / sqrt(2), exp(-z^2) is also the
// unnormalised normal density, so GELU'(u) = Phi(u) + u phi(u) reuses it.  Costs one
// reciprocal and one exponential (hardware approximations) plus a few FMAs.
struct GeluParts {
  float cdf;  // Phi(u)
  float pdf;  // phi(u)
};
__device__ __forceinline__ GeluParts gelu_parts_fast(float u) {
  const float z = fabsf(u) * 0.70710678118654752440f;
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, z, 1.0f)));
  float e;  // exp(-z^2) = 2^(-z^2 * log2(e))
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-z * z * 1.44269504088896340736f));
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f),
               0.254829592f);
  const float erf_abs = 1.0f - poly * e;
  const float erf_z = u < 0.f ? -erf_abs : erf_abs;
  GeluParts r;
  r.cdf = 0.5f * (1.0f + erf_z);
  r.pdf = e * 0.39894228040143267794f;
  return r;
}
__device__ __forceinline__ float gelu_fast(float u) { return u * gelu_parts_fast(u).cdf; }
__device__ __forceinline__ float gelu_grad_fast(float u) {
  const GeluParts g = gelu_parts_fast(u);
  return g.cdf + u * g.pdf;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace nsw

#define NSW_CUDA_CHECK(expr)                                                          \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess) return _e;                                                 \
  } while (0)
