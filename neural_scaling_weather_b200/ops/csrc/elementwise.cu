// Memory-bound kernels: RMSNorm, GEMM epilogues for the library-GEMM path, GELU backward,
// patch (un)folding, weighted squared-error losses, the fused AdamW update and
// segmented sums of squares.  All use 16-byte vector accesses where rows allow it and
// grids sized to the 148 SMs; reductions are two-pass (per-block partials, then a fixed
// order sum) so results are bit-reproducible.
#include "common.cuh"
#include "kernels.h"

namespace nsw {

static int g_num_sms = 0;
static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

int* device_error_flag() {
  static int* flags[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!flags[dev]) {
    cudaMalloc(&flags[dev], sizeof(int));
    cudaMemset(flags[dev], 0, sizeof(int));
  }
  return flags[dev];
}

// ============================================================================ RMSNorm
// One warp per row; lane owns columns [8*(lane + 32*j), +8) and keeps them in registers
// between the sum of squares and the scaled store (one read, one write per element).
template <typename T, int NCH>
__global__ void rmsnorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                   T* __restrict__ y, float* __restrict__ rstd, int64_t rows, int n,
                                   float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = n >> 3;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps_total) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * n);
    float f[NCH][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        unpack8<T>(xr[c], f[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[j][i] * f[j][i];
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)n + eps);
    if (lane == 0 && rstd) rstd[r] = rs;
    uint4* yr = reinterpret_cast<uint4*>(y + r * n);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c);
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c + 1);
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = f[j][i] * rs * ww[i];
        yr[c] = pack8<T>(o);
      }
    }
  }
}

// dx = rstd * (dy*w - xhat * mean(dy*w*xhat)).  The weight gradient is accumulated in
// registers (a lane always owns the same columns), reduced across the block's warps in
// shared memory and written as one partial row per block.
template <typename T, int NCH>
__global__ void rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   T* __restrict__ dx, float* __restrict__ dw_part, int64_t rows,
                                   int n) {
  extern __shared__ float sdw[];  // [warps, n]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int64_t warps_total = (int64_t)gridDim.x * nwarps;
  const int nvec = n >> 3;
  float acc[NCH * 8];
  float wr[NCH][8];  // this lane's columns of w, constant across rows
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = lane + 32 * j;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[j * 8 + i] = 0.f;
      wr[j][i] = c < nvec ? __ldg(w + 8 * c + i) : 0.f;
    }
  }
  for (int64_t r = (int64_t)blockIdx.x * nwarps + warp; r < rows; r += warps_total) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * n);
    const uint4* dyr = reinterpret_cast<const uint4*>(dy + r * n);
    const float rs = rstd[r];
    float fx[NCH][8], fg[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        unpack8<T>(xr[c], fx[j]);
        unpack8<T>(dyr[c], fg[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += fg[j][i] * wr[j][i] * fx[j][i];
      }
    }
    dot *= rs;
    dot = warp_sum(dot) / (float)n;
    uint4* dxr = reinterpret_cast<uint4*>(dx + r * n);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int c = lane + 32 * j;
      if (c < nvec) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = fx[j][i] * rs;
          o[i] = rs * (fg[j][i] * wr[j][i] - xh * dot);
          acc[j * 8 + i] += fg[j][i] * xh;
        }
        dxr[c] = pack8<T>(o);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = lane + 32 * j;
    if (c < nvec) {
#pragma unroll
      for (int i = 0; i < 8; ++i) sdw[warp * n + 8 * c + i] = acc[j * 8 + i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = 0.f;
    for (int k = 0; k < nwarps; ++k) v += sdw[k * n + i];
    dw_part[(int64_t)blockIdx.x * n + i] = v;
  }
}

cudaError_t rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n,
                        float eps, int dtype, cudaStream_t s) {
  if (rmsnorm_tma_supported(rows, n, dtype))
    return rmsnorm_fwd_tma(x, w, y, rstd, rows, n, eps, dtype, 2 * num_sms(), s);
  return rmsnorm_fwd_rows(x, w, y, rstd, rows, n, eps, dtype, s);
}

// one warp per row, rows held in registers (fallback of the TMA version)
cudaError_t rmsnorm_fwd_rows(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n,
                             float eps, int dtype, cudaStream_t s) {
  if (n % 8 || n > 2048) return cudaErrorInvalidValue;
  const int threads = 256;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  const int nch = (n / 8 + 31) / 32;
#define NSW_RF(T, NCH) \
  rmsnorm_fwd_kernel<T, NCH><<<blocks, threads, 0, s>>>((const T*)x, w, (T*)y, rstd, rows, n, eps)
#define NSW_RF_N(T)                \
  if (nch <= 1) NSW_RF(T, 1);      \
  else if (nch <= 2) NSW_RF(T, 2); \
  else if (nch <= 4) NSW_RF(T, 4); \
  else NSW_RF(T, 8);
  if (dtype == kBF16) { NSW_RF_N(__nv_bfloat16) }
  else if (dtype == kF16) { NSW_RF_N(__half) }
  else return cudaErrorInvalidValue;
#undef NSW_RF_N
#undef NSW_RF
  return cudaGetLastError();
}

cudaError_t rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                        float* dw_partial, int partial_rows, int64_t rows, int n, int dtype,
                        cudaStream_t s, float eps, const void* add) {
  if (rmsnorm_tma_supported(rows, n, dtype))
    return rmsnorm_bwd_tma(dy, x, w, rstd, dx, dw_partial, partial_rows, rows, n, dtype, eps, s, add);
  if (add) return cudaErrorInvalidValue;  // callers add the skip gradient themselves on this path
  return rmsnorm_bwd_rows(dy, x, w, rstd, dx, dw_partial, partial_rows, rows, n, dtype, s);
}

cudaError_t rmsnorm_bwd_rows(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                             float* dw_partial, int partial_rows, int64_t rows, int n, int dtype,
                             cudaStream_t s) {
  if (n % 8 || n > 2048) return cudaErrorInvalidValue;
  const int threads = 256;
  const size_t smem = (size_t)n * sizeof(float) * (threads / 32);
  const int nch = (n / 8 + 31) / 32;
#define NSW_RB(T, NCH)                                                                       \
  do {                                                                                       \
    if (smem > 48 * 1024)                                                                    \
      cudaFuncSetAttribute(rmsnorm_bwd_kernel<T, NCH>,                                        \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);          \
    rmsnorm_bwd_kernel<T, NCH><<<partial_rows, threads, smem, s>>>(                          \
        (const T*)dy, (const T*)x, w, rstd, (T*)dx, dw_partial, rows, n);                    \
  } while (0)
#define NSW_RB_N(T)                          \
  if (nch <= 1) NSW_RB(T, 1);                \
  else if (nch <= 2) NSW_RB(T, 2);           \
  else if (nch <= 4) NSW_RB(T, 4);           \
  else NSW_RB(T, 8);
  if (dtype == kBF16) { NSW_RB_N(__nv_bfloat16) }
  else if (dtype == kF16) { NSW_RB_N(__half) }
  else return cudaErrorInvalidValue;
#undef NSW_RB_N
#undef NSW_RB
  return cudaGetLastError();
}

// ============================================================================ epilogue
template <typename T, typename TA>
__global__ void bias_act_residual_kernel(const TA* __restrict__ acc, const float* __restrict__ bias,
                                         const T* __restrict__ res, int64_t res_period,
                                         T* __restrict__ y, T* __restrict__ preact, int64_t rows,
                                         int n, int act) {
  const int64_t total = rows * (int64_t)n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n;
    const int c = (int)(i - r * n);
    float v = to_f(acc[i]);
    if (bias) v += bias[c];
    if (preact) preact[i] = from_f<T>(v);
    if (act == 1) v = gelu_f(v);
    if (res) v += to_f(res[(r % res_period) * n + c]);
    y[i] = from_f<T>(v);
  }
}

cudaError_t bias_act_residual(const void* acc, int acc_dtype, const float* bias, const void* residual,
                              int64_t res_period, void* y, void* preact, int64_t rows, int n,
                              int act, int dtype, cudaStream_t s) {
  const int threads = 256;
  int64_t blocks = (rows * n + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (res_period <= 0) res_period = rows;
#define NSW_EPI(T, TA)                                                                            \
  bias_act_residual_kernel<T, TA><<<blocks, threads, 0, s>>>((const TA*)acc, bias, (const T*)residual, \
                                                             res_period, (T*)y, (T*)preact, rows, n, act)
  if (dtype == kBF16 && acc_dtype == kBF16) NSW_EPI(__nv_bfloat16, __nv_bfloat16);
  else if (dtype == kBF16 && acc_dtype == kF32) NSW_EPI(__nv_bfloat16, float);
  else if (dtype == kF16 && acc_dtype == kF16) NSW_EPI(__half, __half);
  else if (dtype == kF16 && acc_dtype == kF32) NSW_EPI(__half, float);
  else return cudaErrorInvalidValue;
#undef NSW_EPI
  return cudaGetLastError();
}

template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ u, T* __restrict__ du,
                                int64_t n8) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g[8], x[8], o[8];
    unpack8<T>(reinterpret_cast<const uint4*>(dy)[i], g);
    unpack8<T>(reinterpret_cast<const uint4*>(u)[i], x);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = g[k] * gelu_grad_f(x[k]);
    reinterpret_cast<uint4*>(du)[i] = pack8<T>(o);
  }
}

cudaError_t gelu_bwd(const void* dy, const void* u, void* du, int64_t n, int dtype, cudaStream_t s) {
  if (n % 8) return cudaErrorInvalidValue;
  const int threads = 256;
  int64_t blocks = (n / 8 + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (dtype == kBF16)
    gelu_bwd_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(
        (const __nv_bfloat16*)dy, (const __nv_bfloat16*)u, (__nv_bfloat16*)du, n / 8);
  else if (dtype == kF16)
    gelu_bwd_kernel<__half><<<blocks, threads, 0, s>>>((const __half*)dy, (const __half*)u,
                                                        (__half*)du, n / 8);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// Column sums of [rows, n] (n % 8 == 0 for the vector path): thread owns 8 adjacent
// columns and walks a chunk of rows with 4 independent accumulators (loads in flight);
// block (x = column group, y = row chunk) writes partial[y, :], then one pass sums the
// partial rows in order (deterministic).
template <typename T>
__global__ void col_sum_vec_kernel(const T* __restrict__ x, float* __restrict__ partial, int64_t rows, int n,
                                   int64_t chunk) {
  const int c8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c8 >= n) return;
  const int64_t r0 = (int64_t)blockIdx.y * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  float a[4][8];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int k = 0; k < 8; ++k) a[u][k] = 0.f;
  int64_t r = r0;
  for (; r + 4 <= r1; r += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(x + (r + u) * n + c8), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) a[u][k] += f[k];
    }
  }
  for (; r < r1; ++r) {
    float f[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(x + r * n + c8), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[0][k] += f[k];
  }
  float* out = partial + (int64_t)blockIdx.y * n + c8;
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = (a[0][k] + a[1][k]) + (a[2][k] + a[3][k]);
}

template <typename T>
__global__ void col_sum_partial_kernel(const T* __restrict__ x, float* __restrict__ partial,
                                       int64_t rows, int n, int64_t chunk) {
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(rows, r0 + chunk);
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    float acc = 0.f;
    for (int64_t r = r0; r < r1; ++r) acc += to_f(x[r * n + c]);
    partial[(int64_t)blockIdx.x * n + c] = acc;
  }
}
// Sum of the partial rows: a block owns 32 columns; its 8 warps take interleaved
// partial rows (coalesced 128-byte reads), then combine in shared memory (fixed order).
__global__ void col_sum_final_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                     int parts, int n) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (c < n)
    for (int p = warp; p < parts; p += 8) acc += partial[(int64_t)p * n + c];
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < n) {
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) v += red[k][lane];
    out[c] = v;
  }
}

// out[b, c] = sum_r part[b, r, c] (deterministic: a fixed split of the rows over 8 thread rows, then
// the 8 partial sums in order).  Block (32 columns x 8 row groups) per 32 columns of one batch.
// Used for the per-CTA weight-gradient partial rows of the norm and attention kernels.
__global__ void sum_rows_kernel(const float* __restrict__ part, int64_t rows, int64_t n, float* __restrict__ out,
                                float* __restrict__ out1, int accumulate) {
  __shared__ float red[8][33];
  const int64_t b = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  const int ry = threadIdx.y;
  float acc = 0.f;
  if (c < n) {
    const float* p = part + b * rows * n + c;
    for (int64_t r = ry; r < rows; r += 8) acc += p[r * n];
  }
  red[ry][threadIdx.x] = acc;
  __syncthreads();
  if (ry == 0 && c < n) {
    float t = red[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < 8; ++k) t += red[k][threadIdx.x];
    float* o = (b == 1 && out1) ? out1 + c : out + b * n + c;
    *o = accumulate ? *o + t : t;
  }
}

cudaError_t sum_rows(const float* part, int64_t batches, int64_t rows, int64_t n, float* out, cudaStream_t s,
                     bool accumulate, float* out1) {
  if (batches <= 0 || n <= 0) return cudaSuccess;
  sum_rows_kernel<<<dim3((unsigned)((n + 31) / 32), (unsigned)batches), dim3(32, 8), 0, s>>>(part, rows, n, out, out1,
                                                                                          accumulate ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t col_sum(const void* x, float* out, float* partial, int partial_rows, int64_t rows, int n,
                    int dtype, cudaStream_t s) {
  if (n % 8 == 0 && dtype != kF32) {
    const int threads = n / 8 < 128 ? ((n / 8 + 31) / 32) * 32 : 128;
    const int gx = (n / 8 + threads - 1) / threads;
    int gy = partial_rows / gx;
    if (gy < 1) gy = 1;
    if (gy > rows) gy = (int)rows;
    const int64_t chunk = (rows + gy - 1) / gy;
    gy = (int)((rows + chunk - 1) / chunk);
    dim3 grid(gx, gy);
    if (dtype == kBF16)
      col_sum_vec_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>((const __nv_bfloat16*)x, partial, rows, n, chunk);
    else
      col_sum_vec_kernel<__half><<<grid, threads, 0, s>>>((const __half*)x, partial, rows, n, chunk);
    col_sum_final_kernel<<<(n + 31) / 32, 256, 0, s>>>(partial, out, gy, n);
    return cudaGetLastError();
  }
  const int64_t chunk = (rows + partial_rows - 1) / partial_rows;
  const int threads = n < 256 ? ((n + 31) / 32) * 32 : 256;
  if (dtype == kBF16)
    col_sum_partial_kernel<__nv_bfloat16><<<partial_rows, threads, 0, s>>>(
        (const __nv_bfloat16*)x, partial, rows, n, chunk);
  else if (dtype == kF16)
    col_sum_partial_kernel<__half><<<partial_rows, threads, 0, s>>>((const __half*)x, partial, rows, n,
                                                                     chunk);
  else if (dtype == kF32)
    col_sum_partial_kernel<float><<<partial_rows, threads, 0, s>>>((const float*)x, partial, rows, n,
                                                                    chunk);
  else
    return cudaErrorInvalidValue;
  col_sum_final_kernel<<<(n + 31) / 32, 256, 0, s>>>(partial, out, partial_rows, n);
  return cudaGetLastError();
}

// ============================================================================ patches
// cols[(n*h + i)*w + j, (c*p + py)*p + px] = x[n, c, i*p + py, j*p + px]
template <typename TX, typename T>
__global__ void im2col_kernel(const TX* __restrict__ x, T* __restrict__ cols, int N, int C, int H,
                              int W, int p) {
  const int h = H / p, w = W / p;
  const int K = C * p * p;
  const int64_t total = (int64_t)N * h * w * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / K;
    const int k = (int)(i - row * K);
    const int j = (int)(row % w);
    const int64_t t = row / w;
    const int ii = (int)(t % h);
    const int n = (int)(t / h);
    const int px = k % p;
    const int py = (k / p) % p;
    const int c = k / (p * p);
    cols[i] = from_f<T>(to_f(x[(((int64_t)n * C + c) * H + ii * p + py) * W + j * p + px]));
  }
}

template <typename TX, typename T>
__global__ void col2im_kernel(const T* __restrict__ dcols, TX* __restrict__ dx, int N, int C, int H,
                              int W, int p) {
  const int h = H / p, w = W / p;
  const int K = C * p * p;
  const int64_t total = (int64_t)N * C * H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % W);
    const int yy = (int)((i / W) % H);
    const int c = (int)((i / ((int64_t)W * H)) % C);
    const int n = (int)(i / ((int64_t)W * H * C));
    float v = 0.f;
    const int ii = yy / p, jj = xx / p;
    if (ii < h && jj < w) {
      const int py = yy - ii * p, px = xx - jj * p;
      v = to_f(dcols[(((int64_t)n * h + ii) * w + jj) * K + (c * p + py) * p + px]);
    }
    dx[i] = from_f<TX>(v);
  }
}

// p = 4, fp32 image with W % 4 == 0: one thread per (patch, channel) reads its 4 x 4 pixels as four
// 16-byte rows (consecutive threads take consecutive patches of one image row, so each of the four
// reads is coalesced) and writes the 16 values of its K-slice (c * 16 .. c * 16 + 15) as whole
// 16-byte vectors.
template <typename T>
__global__ void im2col_p4_kernel(const float* __restrict__ x, T* __restrict__ cols, int N, int C, int H, int W) {
  const int h = H / 4, w = W / 4, K = C * 16;
  const int64_t total = (int64_t)N * h * C * w;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int jj = (int)(i % w);
    const int64_t t = i / w;
    const int c = (int)(t % C);
    const int64_t t2 = t / C;
    const int ii = (int)(t2 % h);
    const int64_t n = t2 / h;
    const float* src = x + ((n * C + c) * H + (int64_t)ii * 4) * W + (int64_t)jj * 4;
    alignas(16) T vals[16];
#pragma unroll
    for (int py = 0; py < 4; ++py) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + (int64_t)py * W));
      vals[py * 4 + 0] = from_f<T>(v.x);
      vals[py * 4 + 1] = from_f<T>(v.y);
      vals[py * 4 + 2] = from_f<T>(v.z);
      vals[py * 4 + 3] = from_f<T>(v.w);
    }
    uint4* dst = reinterpret_cast<uint4*>(cols + ((n * h + ii) * w + jj) * K + c * 16);
    dst[0] = reinterpret_cast<const uint4*>(vals)[0];
    dst[1] = reinterpret_cast<const uint4*>(vals)[1];
  }
}

template <typename TX>
static cudaError_t launch_im2col(const TX* x, void* cols, int N, int C, int H, int W, int p,
                                 int dtype, cudaStream_t s) {
  const int64_t total = (int64_t)N * (H / p) * (W / p) * C * p * p;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (dtype == kBF16)
    im2col_kernel<TX, __nv_bfloat16><<<blocks, 256, 0, s>>>(x, (__nv_bfloat16*)cols, N, C, H, W, p);
  else if (dtype == kF16)
    im2col_kernel<TX, __half><<<blocks, 256, 0, s>>>(x, (__half*)cols, N, C, H, W, p);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t im2col_patch(const void* x, int x_dtype, void* cols, int N, int C, int H, int W, int p,
                         int dtype, cudaStream_t s) {
  if (x_dtype == kF32 && p == 4 && W % 4 == 0 && H % 4 == 0 && (dtype == kBF16 || dtype == kF16) &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(cols) & 15) == 0) {
    const int64_t total = (int64_t)N * (H / 4) * C * (W / 4);
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (dtype == kBF16)
      im2col_p4_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>((const float*)x, (__nv_bfloat16*)cols, N, C, H, W);
    else
      im2col_p4_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>((const float*)x, (__half*)cols, N, C, H, W);
    return cudaGetLastError();
  }
  if (x_dtype == kF32) return launch_im2col((const float*)x, cols, N, C, H, W, p, dtype, s);
  if (x_dtype == kBF16) return launch_im2col((const __nv_bfloat16*)x, cols, N, C, H, W, p, dtype, s);
  if (x_dtype == kF16) return launch_im2col((const __half*)x, cols, N, C, H, W, p, dtype, s);
  return cudaErrorInvalidValue;
}

template <typename TX>
static cudaError_t launch_col2im(const void* dcols, TX* dx, int N, int C, int H, int W, int p,
                                 int dtype, cudaStream_t s) {
  const int64_t total = (int64_t)N * C * H * W;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (dtype == kBF16)
    col2im_kernel<TX, __nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)dcols, dx, N, C, H, W, p);
  else if (dtype == kF16)
    col2im_kernel<TX, __half><<<blocks, 256, 0, s>>>((const __half*)dcols, dx, N, C, H, W, p);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t col2im_patch(const void* dcols, void* dx, int x_dtype, int N, int C, int H, int W, int p,
                         int dtype, cudaStream_t s) {
  if (x_dtype == kF32) return launch_col2im(dcols, (float*)dx, N, C, H, W, p, dtype, s);
  if (x_dtype == kBF16) return launch_col2im(dcols, (__nv_bfloat16*)dx, N, C, H, W, p, dtype, s);
  if (x_dtype == kF16) return launch_col2im(dcols, (__half*)dx, N, C, H, W, p, dtype, s);
  return cudaErrorInvalidValue;
}

// out[bt, c, i*p+py, j*p+px] = y2[(bt*h + i)*w + j, (py*p + px)*C + c]
template <typename T>
__global__ void unpatchify_kernel(const T* __restrict__ y2, T* __restrict__ out, int BT, int h, int w,
                                  int p, int C) {
  const int H = h * p, W = w * p;
  const int64_t total = (int64_t)BT * C * H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % W);
    const int yy = (int)((i / W) % H);
    const int c = (int)((i / ((int64_t)W * H)) % C);
    const int64_t bt = i / ((int64_t)W * H * C);
    const int ii = yy / p, py = yy - ii * p, jj = xx / p, px = xx - jj * p;
    out[i] = y2[((bt * h + ii) * w + jj) * ((int64_t)p * p * C) + (py * p + px) * C + c];
  }
}
template <typename T>
__global__ void patchify_kernel(const T* __restrict__ dout, T* __restrict__ dy2, int BT, int h, int w,
                                int p, int C) {
  const int H = h * p, W = w * p;
  const int K = p * p * C;
  const int64_t total = (int64_t)BT * h * w * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / K;
    const int k = (int)(i - row * K);
    const int c = k % C;
    const int px = (k / C) % p;
    const int py = k / (C * p);
    const int jj = (int)(row % w);
    const int ii = (int)((row / w) % h);
    const int64_t bt = row / ((int64_t)w * h);
    dy2[i] = dout[((bt * C + c) * H + ii * p + py) * (int64_t)W + jj * p + px];
  }
}

// Tiled forms for 16-bit data: one block per (bt, patch row ii, JB consecutive patches).  The JB rows
// of y2 (JB * K contiguous elements, K = p * p * C) move through shared memory, so both global sides
// are whole 16-byte vectors: y2 rows are read (unpatchify) or written (patchify) contiguously, and
// each output image row segment (c, y = ii * p + py, x in [j0 * p, (j0 + nj) * p)) is written (or
// read) as consecutive vectors.  Shared rows are padded by 8 elements to spread the column reads
// over the banks.
constexpr int kPatchJB = 16;

template <typename T>
__global__ void unpatchify_tiled_kernel(const T* __restrict__ y2, T* __restrict__ out, int h, int w, int p, int C) {
  extern __shared__ uint4 patch_smem[];
  T* sm = reinterpret_cast<T*>(patch_smem);
  const int K = p * p * C, Kp = K + 8;
  const int nbw = (w + kPatchJB - 1) / kPatchJB;
  const int jb = (int)(blockIdx.x % nbw);
  const int64_t r = blockIdx.x / nbw;
  const int ii = (int)(r % h);
  const int64_t bt = r / h;
  const int j0 = jb * kPatchJB, nj = min(kPatchJB, w - j0);
  const int64_t row0 = (bt * h + ii) * w + j0;
  const int kv = K / 8;  // 16-byte vectors per row
  const uint4* src = reinterpret_cast<const uint4*>(y2 + row0 * K);
  for (int v = threadIdx.x; v < nj * kv; v += blockDim.x) {
    const int jj = v / kv, k = v - jj * kv;
    *reinterpret_cast<uint4*>(sm + jj * Kp + k * 8) = src[v];
  }
  __syncthreads();
  const int64_t H = (int64_t)h * p, W = (int64_t)w * p;
  const int vper = nj * p / 8;  // 16-byte vectors per output row segment
  for (int t = threadIdx.x; t < C * p * vper; t += blockDim.x) {
    const int v = t % vper, cp = t / vper, py = cp % p, c = cp / p;
    alignas(16) T vals[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int x = v * 8 + e, jj = x / p, px = x - jj * p;
      vals[e] = sm[jj * Kp + (py * p + px) * C + c];
    }
    *reinterpret_cast<uint4*>(out + ((bt * C + c) * H + ii * p + py) * W + (int64_t)j0 * p + v * 8) =
        *reinterpret_cast<const uint4*>(vals);
  }
}

template <typename T>
__global__ void patchify_tiled_kernel(const T* __restrict__ dout, T* __restrict__ dy2, int h, int w, int p, int C) {
  extern __shared__ uint4 patch_smem[];
  T* sm = reinterpret_cast<T*>(patch_smem);
  const int K = p * p * C, Kp = K + 8;
  const int nbw = (w + kPatchJB - 1) / kPatchJB;
  const int jb = (int)(blockIdx.x % nbw);
  const int64_t r = blockIdx.x / nbw;
  const int ii = (int)(r % h);
  const int64_t bt = r / h;
  const int j0 = jb * kPatchJB, nj = min(kPatchJB, w - j0);
  const int64_t H = (int64_t)h * p, W = (int64_t)w * p;
  const int vper = nj * p / 8;
  for (int t = threadIdx.x; t < C * p * vper; t += blockDim.x) {
    const int v = t % vper, cp = t / vper, py = cp % p, c = cp / p;
    alignas(16) T vals[8];
    *reinterpret_cast<uint4*>(vals) = *reinterpret_cast<const uint4*>(
        dout + ((bt * C + c) * H + ii * p + py) * W + (int64_t)j0 * p + v * 8);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int x = v * 8 + e, jj = x / p, px = x - jj * p;
      sm[jj * Kp + (py * p + px) * C + c] = vals[e];
    }
  }
  __syncthreads();
  const int kv = K / 8;
  uint4* dst = reinterpret_cast<uint4*>(dy2 + ((bt * h + ii) * w + j0) * K);
  for (int v = threadIdx.x; v < nj * kv; v += blockDim.x) {
    const int jj = v / kv, k = v - jj * kv;
    dst[v] = *reinterpret_cast<const uint4*>(sm + jj * Kp + k * 8);
  }
}

// the tiled forms apply: 16-bit data, whole vectors on both sides
static bool patch_tiled_ok(int w, int p, int C, int dtype) {
  if (dtype != kBF16 && dtype != kF16) return false;
  const int K = p * p * C;
  if (K % 8 || ((int64_t)w * p) % 8) return false;
  // every segment of nj * p elements, the last (ragged) one included, is whole vectors
  if ((kPatchJB * p) % 8 || ((w % kPatchJB) * p) % 8) return false;
  return (size_t)kPatchJB * (K + 8) * 2 <= 100 * 1024;
}

template <typename T>
static cudaError_t launch_patch_tiled(bool unpatch, const void* a, void* b, int BT, int h, int w, int p, int C,
                                      cudaStream_t s) {
  const int nbw = (w + kPatchJB - 1) / kPatchJB;
  const int64_t blocks = (int64_t)BT * h * nbw;
  const size_t smem = (size_t)kPatchJB * (p * p * C + 8) * sizeof(T);
  auto kern = unpatch ? unpatchify_tiled_kernel<T> : patchify_tiled_kernel<T>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<(unsigned)blocks, 256, smem, s>>>((const T*)a, (T*)b, h, w, p, C);
  return cudaGetLastError();
}

cudaError_t unpatchify(const void* y2, void* out, int BT, int h, int w, int p, int C, int dtype,
                       cudaStream_t s) {
  if (patch_tiled_ok(w, p, C, dtype))
    return dtype == kBF16 ? launch_patch_tiled<__nv_bfloat16>(true, y2, out, BT, h, w, p, C, s)
                          : launch_patch_tiled<__half>(true, y2, out, BT, h, w, p, C, s);
  const int64_t total = (int64_t)BT * C * h * p * w * p;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (dtype == kBF16)
    unpatchify_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)y2, (__nv_bfloat16*)out, BT, h, w, p, C);
  else if (dtype == kF16)
    unpatchify_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)y2, (__half*)out, BT, h, w, p, C);
  else if (dtype == kF32)
    unpatchify_kernel<float><<<blocks, 256, 0, s>>>((const float*)y2, (float*)out, BT, h, w, p, C);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t patchify(const void* dout, void* dy2, int BT, int h, int w, int p, int C, int dtype,
                     cudaStream_t s) {
  if (patch_tiled_ok(w, p, C, dtype))
    return dtype == kBF16 ? launch_patch_tiled<__nv_bfloat16>(false, dout, dy2, BT, h, w, p, C, s)
                          : launch_patch_tiled<__half>(false, dout, dy2, BT, h, w, p, C, s);
  const int64_t total = (int64_t)BT * C * h * p * w * p;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  if (dtype == kBF16)
    patchify_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)dout, (__nv_bfloat16*)dy2, BT, h, w, p, C);
  else if (dtype == kF16)
    patchify_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)dout, (__half*)dy2, BT, h, w, p, C);
  else if (dtype == kF32)
    patchify_kernel<float><<<blocks, 256, 0, s>>>((const float*)dout, (float*)dy2, BT, h, w, p, C);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// ============================================================================ losses
// x, y: [lead, C, H, W]; weight = area_w[h] * ch_w[c]
template <typename TX, typename TY>
__global__ void sse_partial_kernel(const TX* __restrict__ x, const TY* __restrict__ y,
                                   const float* __restrict__ aw, const float* __restrict__ cw,
                                   float* __restrict__ partial, int64_t total, int C, int H, int W) {
  float acc = 0.f;
  const int64_t HW = (int64_t)H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float d = to_f(x[i]) - to_f(y[i]);
    float wgt = 1.f;
    if (aw) wgt *= aw[(i / W) % H];
    if (cw) wgt *= cw[(i / HW) % C];
    acc += wgt * d * d;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}
__global__ void sum_partials_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[0] = v;
  }
}

template <typename TX, typename TY>
__global__ void sse_bwd_kernel(const TX* __restrict__ x, const TY* __restrict__ y,
                               const float* __restrict__ aw, const float* __restrict__ cw,
                               const float* __restrict__ gscale, TX* __restrict__ dx, int64_t total,
                               int C, int H, int W) {
  const float g = 2.f * gscale[0];
  const int64_t HW = (int64_t)H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float wgt = g;
    if (aw) wgt *= aw[(i / W) % H];
    if (cw) wgt *= cw[(i / HW) % C];
    dx[i] = from_f<TX>(wgt * (to_f(x[i]) - to_f(y[i])));
  }
}

template <typename TX, typename TY>
__global__ void se_plane_kernel(const TX* __restrict__ x, const TY* __restrict__ y,
                                const float* __restrict__ aw, float* __restrict__ out, int H, int W) {
  const int64_t plane = blockIdx.x;
  const int64_t HW = (int64_t)H * W;
  const TX* xp = x + plane * HW;
  const TY* yp = y + plane * HW;
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) {
    const float d = to_f(xp[i]) - to_f(yp[i]);
    acc += aw[i / W] * d * d;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[plane] = v;
  }
}

// Plane-structured variants (W % 8 == 0): block (x = row chunk, y = plane); the channel
// weight is constant per block and rows are walked with 8-element vector accesses.
template <typename T>
__device__ __forceinline__ void load8f(const T* p, float* f);
template <>
__device__ __forceinline__ void load8f<float>(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <>
__device__ __forceinline__ void load8f<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(p), f);
}
template <>
__device__ __forceinline__ void load8f<__half>(const __half* p, float* f) {
  unpack8<__half>(*reinterpret_cast<const uint4*>(p), f);
}
template <typename T>
__device__ __forceinline__ void store8f(T* p, const float* f);
template <>
__device__ __forceinline__ void store8f<float>(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
template <>
__device__ __forceinline__ void store8f<__nv_bfloat16>(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = pack8<__nv_bfloat16>(f);
}
template <>
__device__ __forceinline__ void store8f<__half>(__half* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = pack8<__half>(f);
}

template <typename TX, typename TY, bool BWD>
__global__ void sse_plane_kernel(const TX* __restrict__ x, const TY* __restrict__ y,
                                 const float* __restrict__ aw, const float* __restrict__ cw,
                                 const float* __restrict__ gscale, TX* __restrict__ dx,
                                 float* __restrict__ partial, int C, int H, int W, int rows_per_block) {
  const int plane = blockIdx.y;
  const int c = plane % C;
  const float wc = cw ? cw[c] : 1.f;
  const int64_t base = (int64_t)plane * H * W;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(H, r0 + rows_per_block);
  const int wv = W >> 3;
  const float g2 = BWD ? 2.f * gscale[0] * wc : 0.f;
  float acc = 0.f;
  for (int idx = threadIdx.x; idx < (r1 - r0) * wv; idx += blockDim.x) {
    const int rr = r0 + idx / wv;
    const int64_t off = base + (int64_t)rr * W + (int64_t)(idx % wv) * 8;
    float fx[8], fy[8];
    load8f<TX>(x + off, fx);
    load8f<TY>(y + off, fy);
    const float wr = aw ? aw[rr] : 1.f;
    if (BWD) {
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = g2 * wr * (fx[k] - fy[k]);
      store8f<TX>(dx + off, o);
    } else {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float d = fx[k] - fy[k];
        t += d * d;
      }
      acc += wr * t;
    }
  }
  if (BWD) return;
  acc *= wc;
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[(int64_t)blockIdx.y * gridDim.x + blockIdx.x] = v;
  }
}

#define NSW_DISPATCH_XY(XD, YD, MACRO)                                                 \
  if ((XD) == kBF16 && (YD) == kF32) { MACRO(__nv_bfloat16, float); }                  \
  else if ((XD) == kBF16 && (YD) == kBF16) { MACRO(__nv_bfloat16, __nv_bfloat16); }    \
  else if ((XD) == kF16 && (YD) == kF32) { MACRO(__half, float); }                     \
  else if ((XD) == kF16 && (YD) == kF16) { MACRO(__half, __half); }                    \
  else if ((XD) == kF32 && (YD) == kF32) { MACRO(float, float); }                      \
  else return cudaErrorInvalidValue;

static int sse_rows_per_block(int H, int64_t planes, int partial_n) {
  // enough blocks to fill the GPU while keeping planes * blocks_per_plane <= partial_n
  int64_t per_plane = partial_n / (planes > 0 ? planes : 1);
  if (per_plane < 1) per_plane = 1;
  int rpb = (int)((H + per_plane - 1) / per_plane);
  return rpb < 1 ? 1 : rpb;
}

cudaError_t weighted_sse(const void* x, int x_dtype, const void* y, int y_dtype, const float* area_w,
                         const float* ch_w, float* partial, int partial_n, float* out, int64_t lead,
                         int C, int H, int W, cudaStream_t s) {
  const int64_t total = lead * C * (int64_t)H * W;
  const int64_t planes = lead * C;
  if (W % 8 == 0 && planes <= 65535 && planes <= partial_n) {
    const int rpb = sse_rows_per_block(H, planes, partial_n);
    dim3 grid((H + rpb - 1) / rpb, (unsigned)planes);
#define NSW_SSEP(TX, TY)                                                                               \
  sse_plane_kernel<TX, TY, false><<<grid, 256, 0, s>>>((const TX*)x, (const TY*)y, area_w, ch_w, nullptr, \
                                                       nullptr, partial, C, H, W, rpb)
    NSW_DISPATCH_XY(x_dtype, y_dtype, NSW_SSEP)
#undef NSW_SSEP
    sum_partials_kernel<<<1, 1024, 0, s>>>(partial, (int)(grid.x * grid.y), out);
    return cudaGetLastError();
  }
#define NSW_SSE(TX, TY)                                                                         \
  sse_partial_kernel<TX, TY><<<partial_n, 256, 0, s>>>((const TX*)x, (const TY*)y, area_w, ch_w, \
                                                       partial, total, C, H, W)
  NSW_DISPATCH_XY(x_dtype, y_dtype, NSW_SSE)
#undef NSW_SSE
  sum_partials_kernel<<<1, 1024, 0, s>>>(partial, partial_n, out);
  return cudaGetLastError();
}

cudaError_t weighted_sse_bwd(const void* x, int x_dtype, const void* y, int y_dtype,
                             const float* area_w, const float* ch_w, const float* gscale, void* dx,
                             int64_t lead, int C, int H, int W, cudaStream_t s) {
  const int64_t total = lead * C * (int64_t)H * W;
  const int64_t planes = lead * C;
  if (W % 8 == 0 && planes <= 65535) {
    const int rpb = sse_rows_per_block(H, planes, 4 * num_sms());
    dim3 grid((H + rpb - 1) / rpb, (unsigned)planes);
#define NSW_SSEPB(TX, TY)                                                                              \
  sse_plane_kernel<TX, TY, true><<<grid, 256, 0, s>>>((const TX*)x, (const TY*)y, area_w, ch_w, gscale, \
                                                      (TX*)dx, nullptr, C, H, W, rpb)
    NSW_DISPATCH_XY(x_dtype, y_dtype, NSW_SSEPB)
#undef NSW_SSEPB
    return cudaGetLastError();
  }
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
#define NSW_SSEB(TX, TY)                                                                     \
  sse_bwd_kernel<TX, TY><<<blocks, 256, 0, s>>>((const TX*)x, (const TY*)y, area_w, ch_w, gscale, \
                                                (TX*)dx, total, C, H, W)
  NSW_DISPATCH_XY(x_dtype, y_dtype, NSW_SSEB)
#undef NSW_SSEB
  return cudaGetLastError();
}

cudaError_t weighted_se_per_plane(const void* x, int x_dtype, const void* y, int y_dtype,
                                  const float* area_w, float* out, int64_t planes, int H, int W,
                                  cudaStream_t s) {
#define NSW_SEP(TX, TY) \
  se_plane_kernel<TX, TY><<<planes, 512, 0, s>>>((const TX*)x, (const TY*)y, area_w, out, H, W)
  NSW_DISPATCH_XY(x_dtype, y_dtype, NSW_SEP)
#undef NSW_SEP
  return cudaGetLastError();
}

// ============================================================================ optimizer
// One pass over the flat fp32 buffers: g' = g * gscale; (Adam: g' += wd * p);
// AdamW: p *= 1 - lr*wd; m, v update; p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps);
// shadow = low-precision copy of p.  Skipped entirely when *skip != 0 (inf/nan grads).
template <typename TS>
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, TS* __restrict__ shadow,
                             const float* __restrict__ gscale, const int* __restrict__ skip, int64_t n4,
                             float lr, float b1, float b2, float eps, float wd, float bc1,
                             float inv_sqrt_bc2, bool decoupled) {
  if (skip && skip[0] != 0) return;
  const float gs = gscale ? gscale[0] : 1.f;
  const float step = lr / bc1;
  const float decay = decoupled ? (1.f - lr * wd) : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* P = &pp.x;
    const float* G = &gg.x;
    float* M = &mm.x;
    float* V = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float gk = G[k] * gs;
      if (!decoupled) gk += wd * P[k];
      P[k] *= decay;
      M[k] = b1 * M[k] + (1.f - b1) * gk;
      V[k] = b2 * V[k] + (1.f - b2) * gk * gk;
      const float denom = sqrtf(V[k]) * inv_sqrt_bc2 + eps;
      P[k] -= step * M[k] / denom;
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (shadow) {
#pragma unroll
      for (int k = 0; k < 4; ++k) shadow[4 * i + k] = from_f<TS>(P[k]);
    }
  }
}

cudaError_t adamw_step(float* p, const float* g, float* m, float* v, void* shadow, int shadow_dtype,
                       const float* gscale, const int* skip, int64_t n, float lr, float b1, float b2,
                       float eps, float wd, float bc1, float bc2, bool decoupled, cudaStream_t s) {
  if (n % 4) return cudaErrorInvalidValue;
  const int threads = 256;
  int64_t blocks = (n / 4 + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  const float isb = 1.f / sqrtf(bc2);
  if (shadow == nullptr || shadow_dtype == kF32)
    adamw_kernel<float><<<blocks, threads, 0, s>>>(p, g, m, v, (float*)shadow, gscale, skip, n / 4, lr,
                                                   b1, b2, eps, wd, bc1, isb, decoupled);
  else if (shadow_dtype == kBF16)
    adamw_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(p, g, m, v, (__nv_bfloat16*)shadow, gscale,
                                                           skip, n / 4, lr, b1, b2, eps, wd, bc1, isb,
                                                           decoupled);
  else if (shadow_dtype == kF16)
    adamw_kernel<__half><<<blocks, threads, 0, s>>>(p, g, m, v, (__half*)shadow, gscale, skip, n / 4,
                                                    lr, b1, b2, eps, wd, bc1, isb, decoupled);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// Sum of squares per class.  Block b covers [block_lo[b], block_hi[b]) of one segment;
// partial[b] is reduced per class in block order by a single block (deterministic).
__global__ void sumsq_blocks_kernel(const float* __restrict__ x, const int64_t* __restrict__ blo,
                                    const int64_t* __restrict__ bhi, float* __restrict__ partial) {
  const int64_t lo = blo[blockIdx.x], hi = bhi[blockIdx.x];
  float acc = 0.f;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = x[i];
    acc += v * v;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}
__global__ void sumsq_classes_kernel(const float* __restrict__ partial, const int* __restrict__ bcls,
                                     int nblocks, int ncls, float* __restrict__ out) {
  for (int c = threadIdx.x; c < ncls; c += blockDim.x) {
    float acc = 0.f;
    for (int b = 0; b < nblocks; ++b)
      if (bcls[b] == c) acc += partial[b];
    out[c] = acc;
  }
}

cudaError_t segment_sumsq(const float* x, const int64_t* block_lo, const int64_t* block_hi,
                          const int* block_cls, int nblocks, int ncls, float* partial, float* out,
                          cudaStream_t s) {
  sumsq_blocks_kernel<<<nblocks, 256, 0, s>>>(x, block_lo, block_hi, partial);
  sumsq_classes_kernel<<<1, 32, 0, s>>>(partial, block_cls, nblocks, ncls, out);
  return cudaGetLastError();
}

}  // namespace nsw
