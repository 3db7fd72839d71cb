// RMSNorm forward / backward over rows of n <= 4096 16-bit values, streamed through shared
// memory by TMA bulk copies.
//
// Reference semantics: the block norms of models/swin_helpers.py (`RMSNorm(E)` before attention
// and MLP; transformer-engine `te.RMSNorm` in models/swin_helpers_te.py): y = x * rsqrt(mean(x^2)
// + eps) * w, weight-only.
//
// Design: one persistent CTA per SM walks tiles of R consecutive rows (R * n * 2 bytes, at most
// 32 KB per tensor).  Thread 0 keeps a ring of three tiles in flight with cp.async.bulk (the
// rows of a tile are one contiguous range of global memory), so ~192 KB of loads per SM hide
// HBM latency without holding rows in registers.  Eight warps take a tile's rows round-robin;
// a lane owns the 16-byte chunks lane + 32 j of a row and reads them from shared memory twice
// (reduction, then output), which keeps the register count low.  The output row is written
// straight to global memory (each warp store covers 512 contiguous bytes).  The backward
// accumulates the weight gradient in registers (a lane always owns the same columns), then
// writes one partial row per CTA.
#include <algorithm>
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace nsw {
namespace rms_tma {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 3;
constexpr int kTileBytes = 32 * 1024;  // per tensor per stage
constexpr int kMaxN = 4096;  // 16 chunks of 16 bytes per lane
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ bool wait_parity(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (uint32_t spin = 0;; ++spin) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (spin == 0) t0 = t;
    else if (t - t0 > kWaitNs) {
      record_error(err, kErrWaitTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void expect_bytes(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

struct Geometry {
  int64_t rows;
  int n;
  int R;          // rows per tile
  int64_t tiles;  // ceil(rows / R)
  uint32_t copy_bytes;  // bytes per bulk copy (multiple of 16)
};

// Issue the loads of `tile` (one or two tensors) into `stage`.
template <typename T>
__device__ __forceinline__ void issue_tile(const Geometry& gm, int64_t tile, int stage, const T* a, const T* b,
                                           unsigned char* sa, unsigned char* sb, uint64_t* bar) {
  const int64_t r0 = tile * gm.R;
  const int64_t nr = min((int64_t)gm.R, gm.rows - r0);
  const uint32_t bytes = (uint32_t)(nr * gm.n * (int64_t)sizeof(T));
  expect_bytes(bar, b ? 2 * bytes : bytes);
  // several smaller bulk copies per tile keep more requests in flight per SM
  const unsigned char* ga = reinterpret_cast<const unsigned char*>(a + r0 * gm.n);
  const unsigned char* gb = b ? reinterpret_cast<const unsigned char*>(b + r0 * gm.n) : nullptr;
  for (uint32_t off = 0; off < bytes; off += gm.copy_bytes) {
    const uint32_t len = min(gm.copy_bytes, bytes - off);
    bulk_load(sa + (size_t)stage * kTileBytes + off, ga + off, len, bar);
    if (b) bulk_load(sb + (size_t)stage * kTileBytes + off, gb + off, len, bar);
  }
}

// Wait for the loads still in flight after an error (k = index of the iteration that failed).
__device__ __forceinline__ void drain(uint64_t* bar, int k, int64_t first, int64_t step, int64_t tiles) {
  for (int s = 0; s < kStages; ++s) {
    const int j = k + ((s - k % kStages) + kStages) % kStages;  // first iteration >= k on stage s
    if (first + (int64_t)j * step < tiles) wait_parity(&bar[s], (uint32_t)((j / kStages) & 1), nullptr);
  }
}

template <typename T, int NCH>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ y, float* __restrict__ rstd,
               Geometry gm, float eps, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* sx = smem;                                  // [kStages][kTileBytes]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kStages * kTileBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvec = gm.n >> 3;
  float wr[NCH][8];  // this lane's columns of w (a lane always owns the same columns)
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) wr[j][i] = lane + 32 * j < nvec ? __ldg(w + 8 * (lane + 32 * j) + i) : 0.f;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int64_t first = blockIdx.x, step = gridDim.x;
  if (tid == 0)
    for (int s = 0; s < kStages; ++s)
      if (first + s * step < gm.tiles) issue_tile<T>(gm, first + s * step, s, x, nullptr, sx, nullptr, &bar[s]);
  bool ok = true;
  int k = 0;
  for (int64_t tile = first; tile < gm.tiles && ok; tile += step, ++k) {
    const int stage = k % kStages;
    // one thread polls the stage barrier; the others wait in the block barrier (no smem spinning)
    ok = __syncthreads_and(tid == 0 ? wait_parity(&bar[stage], (uint32_t)((k / kStages) & 1), err) : true);
    if (!ok) break;
    const unsigned char* tx = sx + (size_t)stage * kTileBytes;
    const int64_t r0 = tile * gm.R;
    const int nr = (int)min((int64_t)gm.R, gm.rows - r0);
    for (int rr = warp; rr < nr; rr += kWarps) {
      const uint4* xr = reinterpret_cast<const uint4*>(tx + (size_t)rr * gm.n * sizeof(T));
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int c = lane + 32 * j;
        if (c < nvec) {
          float f[8];
          unpack8<T>(xr[c], f);
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
        }
      }
      ss = warp_sum(ss);
      const float rs = rsqrtf(ss / (float)gm.n + eps);
      const int64_t r = r0 + rr;
      if (lane == 0 && rstd) rstd[r] = rs;
      uint4* yr = reinterpret_cast<uint4*>(y + r * gm.n);
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int c = lane + 32 * j;
        if (c < nvec) {
          float f[8], o[8];
          unpack8<T>(xr[c], f);
          const float* ww = wr[j];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = f[i] * rs * ww[i];
          yr[c] = pack8<T>(o);
        }
      }
    }
    __syncthreads();  // the stage is free
    if (tid == 0 && tile + kStages * step < gm.tiles)
      issue_tile<T>(gm, tile + kStages * step, stage, x, nullptr, sx, nullptr, &bar[stage]);
  }
  // an error leaves loads in flight: let them land before the CTA's shared memory is released
  if (!ok && tid == 0) drain(bar, k, first, step, gm.tiles);
  __syncthreads();
}

template <typename T, int NCH>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
               const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ dw_part, Geometry gm, float eps,
               const T* __restrict__ add, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* sx = smem;                          // [kStages][kTileBytes]
  unsigned char* sg = smem + kStages * kTileBytes;   // [kStages][kTileBytes]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kTileBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvec = gm.n >> 3;
  float wr[NCH][8];  // this lane's columns of w (a lane always owns the same columns)
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) wr[j][i] = lane + 32 * j < nvec ? __ldg(w + 8 * (lane + 32 * j) + i) : 0.f;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int64_t first = blockIdx.x, step = gridDim.x;
  if (tid == 0)
    for (int s = 0; s < kStages; ++s)
      if (first + s * step < gm.tiles) issue_tile<T>(gm, first + s * step, s, x, dy, sx, sg, &bar[s]);
  float acc[NCH][8];
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;
  bool ok = true;
  int k = 0;
  for (int64_t tile = first; tile < gm.tiles && ok; tile += step, ++k) {
    const int stage = k % kStages;
    // one thread polls the stage barrier; the others wait in the block barrier (no smem spinning)
    ok = __syncthreads_and(tid == 0 ? wait_parity(&bar[stage], (uint32_t)((k / kStages) & 1), err) : true);
    if (!ok) break;
    const unsigned char* tx = sx + (size_t)stage * kTileBytes;
    const unsigned char* tg = sg + (size_t)stage * kTileBytes;
    const int64_t r0 = tile * gm.R;
    const int nr = (int)min((int64_t)gm.R, gm.rows - r0);
    for (int rr = warp; rr < nr; rr += kWarps) {
      const uint4* xr = reinterpret_cast<const uint4*>(tx + (size_t)rr * gm.n * sizeof(T));
      const uint4* gr = reinterpret_cast<const uint4*>(tg + (size_t)rr * gm.n * sizeof(T));
      const int64_t r = r0 + rr;
      // the skip-connection gradient added to dx (when given) is fetched first, so its global
      // latency overlaps the reduction pass
      uint4 addv[NCH];
      if (add) {
#pragma unroll
        for (int j = 0; j < NCH; ++j)
          if (lane + 32 * j < nvec) addv[j] = __ldg(reinterpret_cast<const uint4*>(add + r * gm.n) + lane + 32 * j);
      }
      // dx = rs * (g*w - xhat * mean(g*w*xhat)),  xhat = x * rs;  dw += g * xhat.  With eps >= 0,
      // rs is recomputed from the x row in smem (the forward's arithmetic, so the same value) in
      // the pass that forms the dot product, instead of a dependent global load per row.
      float dot = 0.f, ss = 0.f;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int c = lane + 32 * j;
        if (c < nvec) {
          float fx[8], fg[8];
          unpack8<T>(xr[c], fx);
          unpack8<T>(gr[c], fg);
          const float* ww = wr[j];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            dot = fmaf(fg[i] * ww[i], fx[i], dot);
            ss = fmaf(fx[i], fx[i], ss);
          }
        }
      }
      const float rs = eps >= 0.f ? rsqrtf(warp_sum(ss) / (float)gm.n + eps) : __ldg(rstd + r);
      dot = warp_sum(dot) * rs / (float)gm.n;
      uint4* dxr = reinterpret_cast<uint4*>(dx + r * gm.n);
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int c = lane + 32 * j;
        if (c < nvec) {
          float fx[8], fg[8], o[8];
          unpack8<T>(xr[c], fx);
          unpack8<T>(gr[c], fg);
          const float* ww = wr[j];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float xh = fx[i] * rs;
            o[i] = rs * (fg[i] * ww[i] - xh * dot);
            acc[j][i] = fmaf(fg[i], xh, acc[j][i]);
          }
          if (add) {
            float fa[8];
            unpack8<T>(addv[j], fa);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] += fa[i];
          }
          dxr[c] = pack8<T>(o);
        }
      }
    }
    __syncthreads();  // the stage is free
    if (tid == 0 && tile + kStages * step < gm.tiles)
      issue_tile<T>(gm, tile + kStages * step, stage, x, dy, sx, sg, &bar[stage]);
  }
  if (!ok && tid == 0) drain(bar, k, first, step, gm.tiles);
  __syncthreads();
  // weight-gradient partial of this CTA: warps' registers -> smem (the stage area) -> one row
  float* sdw = reinterpret_cast<float*>(smem);  // [kWarps][n] floats <= 128 KB
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c = lane + 32 * j;
    if (c < nvec) {
#pragma unroll
      for (int i = 0; i < 8; ++i) sdw[warp * gm.n + 8 * c + i] = acc[j][i];
    }
  }
  __syncthreads();
  for (int i = tid; i < gm.n; i += kThreads) {
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) v += sdw[q * gm.n + i];
    dw_part[(int64_t)blockIdx.x * gm.n + i] = v;
  }
}

Geometry make_geometry(int64_t rows, int n, int elem) {
  Geometry gm;
  gm.rows = rows;
  gm.n = n;
  gm.R = (int)std::max<int64_t>(1, std::min<int64_t>(64, kTileBytes / ((int64_t)n * elem)));
  gm.tiles = (rows + gm.R - 1) / gm.R;
  static const char* env = getenv("NSW_RMS_COPY_BYTES");  // tuning knob
  const int cb = env ? atoi(env) : 32768;
  gm.copy_bytes = (uint32_t)std::max(16, (cb / 16) * 16);
  return gm;
}

}  // namespace rms_tma

bool rmsnorm_tma_supported(int64_t rows, int n, int dtype) {
  return (dtype == kBF16 || dtype == kF16) && n % 8 == 0 && n >= 8 && n <= rms_tma::kMaxN && rows > 0;
}

cudaError_t rmsnorm_fwd_tma(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n, float eps,
                            int dtype, int grid, cudaStream_t s) {
  using namespace rms_tma;
  if (!rmsnorm_tma_supported(rows, n, dtype)) return cudaErrorInvalidValue;
  const Geometry gm = make_geometry(rows, n, 2);
  const size_t smem = (size_t)kStages * kTileBytes + 64;
  const int g = (int)std::min<int64_t>(grid, gm.tiles);
  const int nch = (n / 8 + 31) / 32;
#define NSW_RF(T, NC)                                                                                        \
  do {                                                                                                       \
    NSW_CUDA_CHECK(cudaFuncSetAttribute(fwd_kernel<T, NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    fwd_kernel<T, NC><<<g, kThreads, smem, s>>>((const T*)x, w, (T*)y, rstd, gm, eps, device_error_flag());   \
  } while (0)
#define NSW_RF_N(T)                    \
  if (nch <= 1) NSW_RF(T, 1);          \
  else if (nch <= 2) NSW_RF(T, 2);     \
  else if (nch <= 4) NSW_RF(T, 4);     \
  else if (nch <= 8) NSW_RF(T, 8);     \
  else NSW_RF(T, 16);
  if (dtype == kBF16) { NSW_RF_N(__nv_bfloat16) }
  else { NSW_RF_N(__half) }
#undef NSW_RF_N
#undef NSW_RF
  return cudaGetLastError();
}

cudaError_t rmsnorm_bwd_tma(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dw_partial, int partial_rows, int64_t rows, int n, int dtype, float eps,
                            cudaStream_t s, const void* add) {
  using namespace rms_tma;
  if (!rmsnorm_tma_supported(rows, n, dtype)) return cudaErrorInvalidValue;
  const Geometry gm = make_geometry(rows, n, 2);
  const size_t smem = (size_t)2 * kStages * kTileBytes + 64;
  const int nch = (n / 8 + 31) / 32;
  // every one of the partial_rows CTAs writes its partial row (CTAs without tiles write zeros)
#define NSW_RB(T, NC)                                                                                        \
  do {                                                                                                       \
    NSW_CUDA_CHECK(cudaFuncSetAttribute(bwd_kernel<T, NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    bwd_kernel<T, NC><<<partial_rows, kThreads, smem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx,       \
                                                           dw_partial, gm, eps, (const T*)add,              \
                                                           device_error_flag());                            \
  } while (0)
#define NSW_RB_N(T)                    \
  if (nch <= 1) NSW_RB(T, 1);          \
  else if (nch <= 2) NSW_RB(T, 2);     \
  else if (nch <= 4) NSW_RB(T, 4);     \
  else if (nch <= 8) NSW_RB(T, 8);     \
  else NSW_RB(T, 16);
  if (dtype == kBF16) { NSW_RB_N(__nv_bfloat16) }
  else { NSW_RB_N(__half) }
#undef NSW_RB_N
#undef NSW_RB
  return cudaGetLastError();
}

}  // namespace nsw
