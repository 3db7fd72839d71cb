// Legendre part of the real spherical harmonic transform on an equiangular grid (the transform of
// torch_harmonics.RealSHT(grid="equiangular") that the reference's AMSE loss and power spectra use:
// utils/losses.py:143-228, utils/misc_utils.py:103-123).
//
// After the longitude DFT, the field of one batch row r at colatitude node k and order m is
// F[m, k, n] (n = 2 r + {re, im}); its coefficients are
//   C[m, l, n] = sum_k P[m, l, k] F[m, k, n],   P[m, l, k] = w_k * Pbar_l^m(x_k),  l >= m
// and the adjoint (gradient) is dF[m, k, n] = sum_{l >= m} P[m, l, k] dC[m, l, n].
// P is packed by m: the rows l = m .. L-1 of order m start at row row_off[m]; it is generated on
// the device from the standard recurrences (orthonormal Pbar with the Condon-Shortley phase:
// sectoral seed, then the three-term recurrence in l; Holmes & Featherstone 2002), in double
// precision, stored as float.  The contractions are batched fp32 GEMMs on the CUDA cores (64 x 64
// output tiles, 4 x 4 per thread).
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace nsw {
namespace {

constexpr int TL = 64, TN = 64, TK = 16;

// one thread per (m, k): Pbar_l^m(x_k) * w_k for l = m .. L-1
__global__ void legendre_table_kernel(const double* __restrict__ x, const double* __restrict__ w, int m0, int m_count,
                                      int L, int K, const int64_t* __restrict__ row_off, float* __restrict__ P,
                                      int csphase) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)m_count * K) return;
  const int mi = (int)(idx / K), k = (int)(idx - (int64_t)mi * K);
  const int m = m0 + mi;
  if (m >= L) return;
  const double xk = x[k], wk = w[k];
  const double sint = sqrt(fmax(0.0, 1.0 - xk * xk));
  double pmm = 1.0 / sqrt(4.0 * 3.14159265358979323846);
  for (int j = 1; j <= m; ++j) {
    pmm = sqrt((2.0 * j + 1.0) / (2.0 * j)) * sint * pmm;
    if (csphase) pmm = -pmm;
  }
  float* Pm = P + row_off[mi] * (int64_t)K + k;
  Pm[0] = (float)(pmm * wk);
  if (m + 1 >= L) return;
  double p_lm1 = pmm;
  double p_l = sqrt(2.0 * m + 3.0) * xk * pmm;
  Pm[(int64_t)K] = (float)(p_l * wk);
  for (int l = m + 2; l < L; ++l) {
    const double a = sqrt((4.0 * l * l - 1.0) / ((double)l * l - (double)m * m));
    const double b = sqrt(((l - 1.0) * (l - 1.0) - (double)m * m) / (4.0 * (l - 1.0) * (l - 1.0) - 1.0));
    const double p_new = a * (xk * p_l - b * p_lm1);
    p_lm1 = p_l;
    p_l = p_new;
    Pm[(int64_t)(l - m) * K] = (float)(p_l * wk);
  }
}

// C[mi, l, n] = sum_k P[mi, l, k] F[mi, k, n]  (l < m: zero)
__global__ void __launch_bounds__(256) legendre_fwd_kernel(const float* __restrict__ P,
                                                           const int64_t* __restrict__ row_off,
                                                           const float* __restrict__ F, float* __restrict__ C,
                                                           int m0, int L, int K, int N) {
  __shared__ float As[TK][TL + 4];
  __shared__ float Bs[TK][TN + 4];
  const int mi = blockIdx.z, m = m0 + mi;
  const int l0 = blockIdx.y * TL, n0 = blockIdx.x * TN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const float* Pm = P + row_off[mi] * (int64_t)K;
  const float* Fm = F + (int64_t)mi * K * N;
  if (l0 + TL > m) {
    for (int k0 = 0; k0 < K; k0 += TK) {
      for (int i = threadIdx.x; i < TL * TK; i += 256) {
        const int r = i / TK, c = i - r * TK;
        const int l = l0 + r, k = k0 + c;
        As[c][r] = (l >= m && l < L && k < K) ? Pm[(int64_t)(l - m) * K + k] : 0.f;
      }
      for (int i = threadIdx.x; i < TK * TN; i += 256) {
        const int r = i / TN, c = i - r * TN;
        const int k = k0 + r, n = n0 + c;
        Bs[r][c] = (k < K && n < N) ? Fm[(int64_t)k * N + n] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int t = 0; t < TK; ++t) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[t][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[t][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
  }
  float* Cm = C + (int64_t)mi * L * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + ty * 4 + i;
    if (l >= L) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) Cm[(int64_t)l * N + n] = acc[i][j];
    }
  }
}

// dF[mi, k, n] = sum_{l >= m} P[mi, l, k] dC[mi, l, n]
__global__ void __launch_bounds__(256) legendre_bwd_kernel(const float* __restrict__ P,
                                                           const int64_t* __restrict__ row_off,
                                                           const float* __restrict__ dC, float* __restrict__ dF,
                                                           int m0, int L, int K, int N) {
  __shared__ float As[TK][TL + 4];  // [l][k]
  __shared__ float Bs[TK][TN + 4];  // [l][n]
  const int mi = blockIdx.z, m = m0 + mi;
  const int k0 = blockIdx.y * TL, n0 = blockIdx.x * TN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const float* Pm = P + row_off[mi] * (int64_t)K;
  const float* dCm = dC + (int64_t)mi * L * N;
  for (int ls = (m / TK) * TK; ls < L; ls += TK) {
    for (int i = threadIdx.x; i < TK * TL; i += 256) {
      const int r = i / TL, c = i - r * TL;
      const int l = ls + r, k = k0 + c;
      As[r][c] = (l >= m && l < L && k < K) ? Pm[(int64_t)(l - m) * K + k] : 0.f;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      const int r = i / TN, c = i - r * TN;
      const int l = ls + r, n = n0 + c;
      Bs[r][c] = (l < L && n < N) ? dCm[(int64_t)l * N + n] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < TK; ++t) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[t][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[t][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* dFm = dF + (int64_t)mi * K * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = k0 + ty * 4 + i;
    if (k >= K) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) dFm[(int64_t)k * N + n] = acc[i][j];
    }
  }
}

}  // namespace

cudaError_t legendre_table(const double* x, const double* w, int m0, int m_count, int L, int K,
                           const int64_t* row_off, float* P, int csphase, cudaStream_t s) {
  const int64_t n = (int64_t)m_count * K;
  if (n <= 0) return cudaSuccess;
  legendre_table_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, w, m0, m_count, L, K, row_off, P, csphase);
  return cudaGetLastError();
}

cudaError_t legendre_fwd(const float* P, const int64_t* row_off, const float* F, float* C, int m0, int m_count, int L,
                         int K, int N, cudaStream_t s) {
  if (m_count <= 0) return cudaSuccess;
  dim3 grid((N + TN - 1) / TN, (L + TL - 1) / TL, m_count);
  legendre_fwd_kernel<<<grid, 256, 0, s>>>(P, row_off, F, C, m0, L, K, N);
  return cudaGetLastError();
}

cudaError_t legendre_bwd(const float* P, const int64_t* row_off, const float* dC, float* dF, int m0, int m_count, int L,
                         int K, int N, cudaStream_t s) {
  if (m_count <= 0) return cudaSuccess;
  dim3 grid((N + TN - 1) / TN, (K + TL - 1) / TL, m_count);
  legendre_bwd_kernel<<<grid, 256, 0, s>>>(P, row_off, dC, dF, m0, L, K, N);
  return cudaGetLastError();
}

}  // namespace nsw
