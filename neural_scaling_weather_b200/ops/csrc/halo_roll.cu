// Cyclic roll of a spatially sharded (B, T, H, W, C) activation over NVLink peer memory.
//
// Shifted-window attention on a globe split into sp1 (latitude) x sp2 (longitude) shards needs
// out[h, w] = x[(h - sh) mod H, (w - sw) mod W] in global coordinates (reference:
// distributed/helpers.py:192-277 `_distributed_roll`, used by models/swin_helpers.py:399-433
// around the window attention; there each dimension is one NCCL send/recv plus copies).  With
// shifts smaller than every shard, an output position draws from its own shard or from a band of
// |sh| rows / |sw| columns at the edge of a neighbouring shard (the diagonal one included).  Two
// kernels, one launch each per roll:
//   halo_pack_kernel   waits (bounded) until every peer has finished reading this rank's bands from
//                      the previous roll, copies this rank's edge bands (rows [H_l - sh, H_l) or
//                      [0, -sh), columns likewise) into its symmetric band buffer, and the last
//                      block publishes "ready = epoch" into every peer's flag words.
//   halo_gather_kernel copies every output row whose source is local (the bulk, no waiting), then
//                      waits (bounded) for the peers' ready flags and copies the remaining rows
//                      from their band buffers with plain peer loads; the last block publishes
//                      "ack = epoch" to every peer and advances this rank's epoch word.
// A row is C contiguous elements (16-byte vectors); each warp moves one row.  The epoch lives in
// device memory and the block counters are reset by the last block, so CUDA-graph replays need no
// host state.  No TMA and no multicast touches peer memory.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace nsw {
namespace {

__device__ __forceinline__ int shard_of(const int* off, int n, int g) {
  int i = 0;
  while (i + 1 < n && off[i + 1] <= g) ++i;
  return i;
}

// one row of v 16-byte vectors by one warp, four loads in flight per lane before the stores
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int v, int lane) {
  int k = lane;
  for (; k + 96 < v; k += 128) {
    const uint4 a = src[k], b = src[k + 32], c = src[k + 64], d = src[k + 96];
    dst[k] = a;
    dst[k + 32] = b;
    dst[k + 64] = c;
    dst[k + 96] = d;
  }
  for (; k < v; k += 32) dst[k] = src[k];
}

struct BandGeom {  // where one shard's edge bands sit inside its band buffer (units: rows)
  int64_t nrow_r;  // rows in the latitude band (BT * |sh| * W_l), 0 if latitude is not split
  int r0, c0;      // first local row / column of the bands
};

__device__ __forceinline__ BandGeom band_geom(const HaloArgs& a, int hl, int wl) {
  BandGeom g;
  const int ash = a.sh < 0 ? -a.sh : a.sh, asw = a.sw < 0 ? -a.sw : a.sw;
  g.nrow_r = (a.n1 > 1 && ash) ? (int64_t)a.bt * ash * wl : 0;
  g.r0 = a.sh > 0 ? hl - ash : 0;
  g.c0 = a.sw > 0 ? wl - asw : 0;
  return g;
}

__global__ void halo_pack_kernel(const __grid_constant__ HaloArgs a, int* err) {
  __shared__ int go;
  uint32_t* mine = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(mine + kHaloEpoch) + 1u;
  if (threadIdx.x == 0) {
    bool ok = true;
    // every peer has finished reading the bands of the previous roll
    for (int r = 0; r < a.world && ok; ++r)
      if (r != a.rank) ok = peer::wait_geq(mine + kHaloAck + r, epoch - 1u, err);
    go = ok ? 1 : 0;
  }
  __syncthreads();
  const int i1 = a.coord1[a.rank], i2 = a.coord2[a.rank];
  const int hl = a.h_off[i1 + 1] - a.h_off[i1], wl = a.w_off[i2 + 1] - a.w_off[i2];
  const BandGeom g = band_geom(a, hl, wl);
  const int ash = a.sh < 0 ? -a.sh : a.sh, asw = a.sw < 0 ? -a.sw : a.sw;
  const int64_t nrow_c = (a.n2 > 1 && asw) ? (int64_t)a.bt * hl * asw : 0;
  const int64_t rows = g.nrow_r + nrow_c;
  const int v = a.row_vec;
  if (go) {
    const uint4* x = reinterpret_cast<const uint4*>(a.x);
    uint4* band = reinterpret_cast<uint4*>(a.band[a.rank]);
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = warp; row < rows; row += nwarps) {
      int64_t bt, h, w;
      if (row < g.nrow_r) {
        const int64_t per = (int64_t)ash * wl;
        bt = row / per;
        const int64_t rem = row - bt * per;
        h = g.r0 + rem / wl;
        w = rem % wl;
      } else {
        const int64_t rr = row - g.nrow_r, per = (int64_t)hl * asw;
        bt = rr / per;
        const int64_t rem = rr - bt * per;
        h = rem / asw;
        w = g.c0 + rem % asw;
      }
      const uint4* src = x + ((bt * hl + h) * wl + w) * v;
      copy_row(band + row * v, src, v, lane);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(mine + kHaloPackCount, 1u) == gridDim.x - 1) {
      mine[kHaloPackCount] = 0;
      __threadfence_system();
      for (int r = 0; r < a.world; ++r)
        if (r != a.rank) peer::st_release(a.flags[r] + kHaloReady + a.rank, epoch);
    }
  }
}

__global__ void halo_gather_kernel(const __grid_constant__ HaloArgs a, int* err) {
  __shared__ int go;
  uint32_t* mine = a.flags[a.rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(mine + kHaloEpoch) + 1u;
  const int i1 = a.coord1[a.rank], i2 = a.coord2[a.rank];
  const int hl = a.h_off[i1 + 1] - a.h_off[i1], wl = a.w_off[i2 + 1] - a.w_off[i2];
  const int h0 = a.h_off[i1], w0 = a.w_off[i2];
  const int H = a.h_off[a.n1], W = a.w_off[a.n2];
  const int v = a.row_vec;
  const int ash = a.sh < 0 ? -a.sh : a.sh, asw = a.sw < 0 ? -a.sw : a.sw;
  const uint4* x = reinterpret_cast<const uint4*>(a.x);
  uint4* out = reinterpret_cast<uint4*>(a.out);
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t rows = (int64_t)a.bt * hl * wl;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      __syncthreads();
      if (threadIdx.x == 0) {
        bool ok = true;
        for (int r = 0; r < a.world && ok; ++r)
          if (r != a.rank) ok = peer::wait_geq(mine + kHaloReady + r, epoch, err);
        go = ok ? 1 : 0;
      }
      __syncthreads();
      if (!go) break;
    }
    for (int64_t row = warp; row < rows; row += nwarps) {
      const int64_t bt = row / ((int64_t)hl * wl);
      const int64_t rem = row - bt * hl * wl;
      const int h = (int)(rem / wl), w = (int)(rem % wl);
      int gh = (h0 + h - a.sh) % H;
      if (gh < 0) gh += H;
      int gw = (w0 + w - a.sw) % W;
      if (gw < 0) gw += W;
      const int o1 = shard_of(a.h_off, a.n1, gh), o2 = shard_of(a.w_off, a.n2, gw);
      const int lh = gh - a.h_off[o1], lw = gw - a.w_off[o2];
      const bool local = (o1 == i1 && o2 == i2);
      if (local != (pass == 0)) continue;
      const uint4* src;
      if (local) {
        src = x + ((bt * hl + lh) * wl + lw) * v;
      } else {
        const int o = a.grid_rank[o1 * a.n2 + o2];
        const int hlo = a.h_off[o1 + 1] - a.h_off[o1], wlo = a.w_off[o2 + 1] - a.w_off[o2];
        const BandGeom g = band_geom(a, hlo, wlo);
        int64_t idx;
        if (g.nrow_r > 0 && lh >= g.r0 && lh < g.r0 + ash) {
          idx = (bt * ash + (lh - g.r0)) * wlo + lw;
        } else if (a.n2 > 1 && asw && lw >= g.c0 && lw < g.c0 + asw) {
          idx = g.nrow_r + (bt * hlo + lh) * asw + (lw - g.c0);
        } else {  // not in a band: the host checks the shifts against the shards, so never taken
          if (lane == 0) record_error(err, kErrBounds);
          continue;
        }
        src = reinterpret_cast<const uint4*>(a.band[o]) + idx * v;
      }
      copy_row(out + row * v, src, v, lane);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(mine + kHaloDoneCount, 1u) == gridDim.x - 1) {
      mine[kHaloDoneCount] = 0;
      __threadfence_system();
      for (int r = 0; r < a.world; ++r)
        if (r != a.rank) peer::st_release(a.flags[r] + kHaloAck + a.rank, epoch);
      mine[kHaloEpoch] = epoch;
    }
  }
}

}  // namespace

int64_t halo_band_bytes(const HaloArgs& a, int shard) {
  const int i1 = a.coord1[shard], i2 = a.coord2[shard];
  const int hl = a.h_off[i1 + 1] - a.h_off[i1], wl = a.w_off[i2 + 1] - a.w_off[i2];
  const int ash = std::abs(a.sh), asw = std::abs(a.sw);
  const int64_t nr = (a.n1 > 1 && ash) ? (int64_t)a.bt * ash * wl : 0;
  const int64_t nc = (a.n2 > 1 && asw) ? (int64_t)a.bt * hl * asw : 0;
  return (nr + nc) * a.row_vec * 16;
}

cudaError_t halo_roll(const HaloArgs& a, cudaStream_t s) {
  if (a.world < 2 || a.world > 8 || a.rank < 0 || a.rank >= a.world || a.n1 < 1 || a.n2 < 1 ||
      a.n1 * a.n2 != a.world || a.row_vec < 1 || a.bt < 1)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.out)) & 15) return cudaErrorInvalidValue;
  for (int r = 0; r < a.world; ++r)
    if (!a.band[r] || !a.flags[r] || (reinterpret_cast<uintptr_t>(a.band[r]) & 15)) return cudaErrorInvalidValue;
  // every source outside the own shard must lie in a neighbour's band: shifts below every split shard
  for (int i = 0; i < a.n1; ++i)
    if (a.n1 > 1 && std::abs(a.sh) >= a.h_off[i + 1] - a.h_off[i]) return cudaErrorInvalidValue;
  for (int j = 0; j < a.n2; ++j)
    if (a.n2 > 1 && std::abs(a.sw) >= a.w_off[j + 1] - a.w_off[j]) return cudaErrorInvalidValue;
  int* err = device_error_flag();
  const int i1 = a.coord1[a.rank], i2 = a.coord2[a.rank];
  const int64_t rows = (int64_t)a.bt * (a.h_off[i1 + 1] - a.h_off[i1]) * (a.w_off[i2 + 1] - a.w_off[i2]);
  const int64_t band_rows = halo_band_bytes(a, a.rank) / (16 * (int64_t)a.row_vec);
  // 8 warps per block, one row per warp per iteration
  const int pack_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((band_rows + 7) / 8, 148));
  const int gather_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 148 * 6));
  halo_pack_kernel<<<pack_blocks, 256, 0, s>>>(a, err);
  halo_gather_kernel<<<gather_blocks, 256, 0, s>>>(a, err);
  return cudaGetLastError();
}

}  // namespace nsw
