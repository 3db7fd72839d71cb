// Allocation-free RMSNorm backward (see noalloc.h for the contract).  No counterpart in
// the reference implementation.
//
// Two launches on the caller's stream:
//   1. partial_kernel: NSW_NOALLOC_RMSNORM_PARTS (or fewer) blocks walk the rows, write dx
//      and accumulate dy * xhat per column in registers; each block writes ONE complete
//      partial row of n floats into the file-scope scratch array;
//   2. reduce_kernel: sums the partial rows in block order into dw (deterministic).
// Every partial row that step 2 reads was written by step 1 of the same call, so the
// scratch never needs clearing.
#include <mutex>

#include "common.cuh"
#include "noalloc.h"

namespace {

// The scratch: one partial weight-gradient row per block.
static __device__ __align__(256) float g_rmsnorm_dw_scratch[NSW_NOALLOC_RMSNORM_PARTS * NSW_NOALLOC_RMSNORM_MAX_N];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Device address of the scratch array for the current device (looked up once per device;
// in host code the array's name is only a stand-in, never a device address).
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NSW_NOALLOC_ERR_SYMBOL;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rmsnorm_dw_scratch);
    if (e != cudaSuccess || p == nullptr) return NSW_NOALLOC_ERR_SYMBOL;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return NSW_NOALLOC_OK;
}

template <typename T, int NCH>
__global__ void partial_kernel(const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                               const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ partial,
                               int64_t rows, int n) {
  extern __shared__ float srow[];  // [n]: the block's partial row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int nvec = n >> 3;
  float acc[NCH * 8];
#pragma unroll
  for (int i = 0; i < NCH * 8; ++i) acc[i] = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * nwarps + warp; r < rows; r += (int64_t)gridDim.x * nwarps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * n);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + r * n);
    const float rs = rstd[r];
    float fx[NCH][8], fg[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        nsw::unpack8<T>(xr[c], fx[j]);
        nsw::unpack8<T>(gr[c], fg[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += fg[j][i] * w[8 * c + i] * fx[j][i] * rs;
      }
    }
    dot = nsw::warp_sum(dot) / (float)n;
    uint4* dxr = reinterpret_cast<uint4*>(dx + r * n);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = fx[j][i] * rs;
          o[i] = rs * (fg[j][i] * w[8 * c + i] - xh * dot);
          acc[j * 8 + i] += fg[j][i] * xh;
        }
        dxr[c] = nsw::pack8<T>(o);
      }
    }
  }
  // reduce the warps' column sums through shared memory, one warp at a time
  for (int i = threadIdx.x; i < n; i += blockDim.x) srow[i] = 0.f;
  __syncthreads();
  for (int k = 0; k < nwarps; ++k) {
    if (warp == k) {
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int c = lane + 32 * j;
        if (c < nvec) {
#pragma unroll
          for (int i = 0; i < 8; ++i) srow[8 * c + i] += acc[j * 8 + i];
        }
      }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) partial[(int64_t)blockIdx.x * n + i] = srow[i];
}

__global__ void reduce_kernel(const float* __restrict__ partial, float* __restrict__ dw, int parts, int n) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[(int64_t)p * n + c];
  dw[c] = s;
}

template <typename T>
int launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw, int64_t rows,
           int n, cudaStream_t s, float* scratch) {
  const int threads = 256;
  int parts = NSW_NOALLOC_RMSNORM_PARTS;
  const int64_t need = (rows + (threads / 32) - 1) / (threads / 32);
  if (need < parts) parts = (int)(need > 0 ? need : 1);
  const int nch = (n / 8 + 31) / 32;
  const size_t smem = (size_t)n * sizeof(float);
#define NSW_NA_LAUNCH(NCH)                                                                               \
  partial_kernel<T, NCH><<<parts, threads, smem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx, scratch, \
                                                      rows, n)
  if (nch <= 1) NSW_NA_LAUNCH(1);
  else if (nch <= 2) NSW_NA_LAUNCH(2);
  else if (nch <= 4) NSW_NA_LAUNCH(4);
  else NSW_NA_LAUNCH(8);
#undef NSW_NA_LAUNCH
  if (cudaGetLastError() != cudaSuccess) return NSW_NOALLOC_ERR_LAUNCH;
  reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(scratch, dw, parts, n);
  if (cudaGetLastError() != cudaSuccess) return NSW_NOALLOC_ERR_LAUNCH;
  return NSW_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int nsw_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw, int64_t rows, int n,
    int dtype, void* stream) {
  if (n > NSW_NOALLOC_RMSNORM_MAX_N) return NSW_NOALLOC_ERR_TOO_LARGE;
  if (n <= 0 || n % 8 != 0 || rows < 0 || !dy || !x || !w || !rstd || !dx || !dw) return NSW_NOALLOC_ERR_BAD_ARG;
  if (dtype != 0 && dtype != 1) return NSW_NOALLOC_ERR_BAD_ARG;
  // dy, x and dx are read and written 16 bytes at a time
  if (((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dx)) & 15) != 0)
    return NSW_NOALLOC_ERR_BAD_ARG;
  // An error left pending by an earlier CUDA call of the caller would otherwise be read back
  // (and cleared) below as if one of these launches had failed; report it without clearing.
  if (cudaPeekAtLastError() != cudaSuccess) return NSW_NOALLOC_ERR_PENDING;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {  // no rows: the weight gradient is zero (dw is written, not added)
    return cudaMemsetAsync(dw, 0, (size_t)n * sizeof(float), s) == cudaSuccess ? NSW_NOALLOC_OK
                                                                                : NSW_NOALLOC_ERR_LAUNCH;
  }
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != NSW_NOALLOC_OK) return rc;
  if (dtype == 0) return launch<__nv_bfloat16>(dy, x, w, rstd, dx, dw, rows, n, s, scratch);
  return launch<__half>(dy, x, w, rstd, dx, dw, rows, n, s, scratch);
}

extern "C" __attribute__((visibility("default"))) const char* nsw_noalloc_error_string(int code) {
  switch (code) {
    case NSW_NOALLOC_OK: return "ok";
    case NSW_NOALLOC_ERR_TOO_LARGE: return "n exceeds NSW_NOALLOC_RMSNORM_MAX_N (2048)";
    case NSW_NOALLOC_ERR_BAD_ARG:
      return "invalid argument (null pointer, dy/x/dx not 16-byte aligned, n not a positive multiple of 8, or dtype)";
    case NSW_NOALLOC_ERR_SYMBOL: return "could not obtain the device address of the scratch array";
    case NSW_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    case NSW_NOALLOC_ERR_PENDING: return "a CUDA error from an earlier call was already pending; nothing launched";
    default: return "unknown error";
  }
}
