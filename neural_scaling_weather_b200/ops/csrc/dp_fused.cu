// Data-parallel gradient reduction and sharded AdamW over NVLink peer memory (one node).
//
// The flat fp32 gradient buffer, the fp32 parameters and their 16-bit shadow of every rank live in
// symmetric memory, so each kernel gets every rank's pointer.  Each rank owns one slice of every
// gradient bucket (the bucket split W ways).  Reference behaviour: the DDP all-reduce with the
// comm hook dividing by dp (distributed/mappings.py:217-341), the clip (utils/trainer.py:416-448)
// and the fused Adam/AdamW step (utils/optimizer_utils.py:56-72).
//   dp_reduce_kernel  (per bucket, on a side stream while backward continues): announces that this
//     rank's gradients of the bucket are final (epoch-tagged flag in every peer's flag array), waits
//     (bounded) until every rank has announced, then pulls the owned slice from every rank with
//     plain peer loads, sums in rank order (deterministic, the same on every rank) and writes
//     sum / W into its own buffer.
//   dp_adamw_kernel   (after the clip coefficient is known): AdamW on the owned slices; the new fp32
//     parameter and its 16-bit shadow are stored into EVERY rank's buffers (peer stores): the
//     all-gather of the parameters rides on the update.
//   dp_barrier_kernel: announces this rank's stores complete and waits (bounded) for every rank's,
//     so no rank's next forward reads a parameter before all owners have written it.
// No TMA and no multicast touches peer memory.  Every wait records kErrWaitTimeout in the device
// error word when it runs out (4 s) and the kernel returns.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace nsw {
namespace {

// announce (slot, epoch) to every rank, then wait for every rank's announcement of the same slot
__device__ bool dp_exchange(const DpPeers& pr, int slot, uint32_t epoch, int* err) {
  __threadfence_system();
  for (int r = 0; r < pr.world; ++r)
    peer::st_release(pr.flags[r] + kDpFlagBase + (int64_t)pr.rank * pr.slots + slot, epoch);
  bool ok = true;
  for (int r = 0; r < pr.world && ok; ++r)
    ok = peer::wait_geq(pr.flags[pr.rank] + kDpFlagBase + (int64_t)r * pr.slots + slot, epoch, err);
  return ok;
}

__global__ void dp_reduce_kernel(const __grid_constant__ DpPeers pr, int slot, uint32_t epoch, int64_t lo,
                                 int64_t hi, float scale, int* err) {
  __shared__ int go;
  if (threadIdx.x == 0) {
    // every block announces (idempotent) and waits, so no block reads a peer before it is ready
    go = dp_exchange(pr, slot, epoch, err) ? 1 : 0;
  }
  __syncthreads();
  if (!go) return;
  float* mine = pr.grad[pr.rank];
  const int64_t n4 = (hi - lo) / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = lo + 4 * i;
    float4 s = *reinterpret_cast<const float4*>(pr.grad[0] + e);
    for (int r = 1; r < pr.world; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(pr.grad[r] + e);
      s.x += x.x;
      s.y += x.y;
      s.z += x.z;
      s.w += x.w;
    }
    s.x *= scale;
    s.y *= scale;
    s.z *= scale;
    s.w *= scale;
    *reinterpret_cast<float4*>(mine + e) = s;
  }
}

template <typename TS>
__global__ void dp_adamw_kernel(const __grid_constant__ DpPeers pr, const int64_t* __restrict__ rlo,
                                const int64_t* __restrict__ rhi, const int64_t* __restrict__ rstart, int nranges,
                                int64_t total4, float* __restrict__ m, float* __restrict__ v,
                                const float* __restrict__ gscale, const int* __restrict__ skip, float lr, float b1,
                                float b2, float eps, float wd, float bc1, float inv_sqrt_bc2, int decoupled) {
  if (skip && skip[0] != 0) return;
  const float gs = gscale ? gscale[0] : 1.f;
  const float step = lr / bc1;
  const float decay = decoupled ? (1.f - lr * wd) : 1.f;
  float* p = pr.data[pr.rank];
  const float* g = pr.grad[pr.rank];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    // range holding the i-th owned float4 (ranges are few: binary search over their starts)
    int a = 0, b = nranges - 1;
    while (a < b) {
      const int mid = (a + b + 1) >> 1;
      if (rstart[mid] <= i) a = mid;
      else b = mid - 1;
    }
    const int64_t e = rlo[a] + 4 * (i - rstart[a]);
    float4 pp = *reinterpret_cast<const float4*>(p + e);
    const float4 gg = *reinterpret_cast<const float4*>(g + e);
    float4 mm = *reinterpret_cast<const float4*>(m + e);
    float4 vv = *reinterpret_cast<const float4*>(v + e);
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
    *reinterpret_cast<float4*>(m + e) = mm;
    *reinterpret_cast<float4*>(v + e) = vv;
    uint2 sh;
    {
      TS h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) h[k] = from_f<TS>(P[k]);
      sh = *reinterpret_cast<const uint2*>(h);
    }
    for (int r = 0; r < pr.world; ++r) {
      *reinterpret_cast<float4*>(pr.data[r] + e) = pp;
      if (pr.shadow[r]) *reinterpret_cast<uint2*>(reinterpret_cast<TS*>(pr.shadow[r]) + e) = sh;
    }
  }
  (void)rhi;
}

__global__ void dp_barrier_kernel(const __grid_constant__ DpPeers pr, int slot, uint32_t epoch, int* err) {
  if (threadIdx.x == 0 && blockIdx.x == 0) dp_exchange(pr, slot, epoch, err);
}

}  // namespace

cudaError_t dp_reduce(const DpPeers& pr, int slot, uint32_t epoch, int64_t lo, int64_t hi, float scale,
                      cudaStream_t s) {
  if (pr.world < 1 || pr.world > 8 || (lo & 3) || ((hi - lo) & 3) || slot < 0 || slot >= pr.slots)
    return cudaErrorInvalidValue;
  const int64_t n4 = (hi - lo) / 4;
  int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 32);
  if (blocks < 1) blocks = 1;
  dp_reduce_kernel<<<blocks, 256, 0, s>>>(pr, slot, epoch, lo, hi, scale, device_error_flag());
  return cudaGetLastError();
}

cudaError_t dp_adamw(const DpPeers& pr, const int64_t* rlo, const int64_t* rhi, const int64_t* rstart, int nranges,
                     int64_t total4, float* m, float* v, int shadow_dtype, const float* gscale, const int* skip,
                     float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, bool decoupled,
                     cudaStream_t s) {
  if (pr.world < 1 || pr.world > 8 || nranges < 1) return cudaErrorInvalidValue;
  int64_t blocks = (total4 + 255) / 256;
  const int64_t cap = 148 * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const float isb = 1.f / sqrtf(bc2);
  if (shadow_dtype == kF16)
    dp_adamw_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(pr, rlo, rhi, rstart, nranges, total4, m, v, gscale,
                                                             skip, lr, b1, b2, eps, wd, bc1, isb, decoupled ? 1 : 0);
  else
    dp_adamw_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(pr, rlo, rhi, rstart, nranges, total4, m, v,
                                                                     gscale, skip, lr, b1, b2, eps, wd, bc1, isb,
                                                                     decoupled ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t dp_barrier(const DpPeers& pr, int slot, uint32_t epoch, cudaStream_t s) {
  if (pr.world < 1 || pr.world > 8 || slot < 0 || slot >= pr.slots) return cudaErrorInvalidValue;
  dp_barrier_kernel<<<1, 32, 0, s>>>(pr, slot, epoch, device_error_flag());
  return cudaGetLastError();
}

}  // namespace nsw
