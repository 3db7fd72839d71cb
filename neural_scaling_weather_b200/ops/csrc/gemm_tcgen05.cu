// Persistent, warp-specialised tcgen05 GEMM with fused epilogues for sm_100a.
//
//   D[m, n] = epilogue( alpha * sum_k A[m, k] * B[n, k] )
//   epilogue: (+ bias[n]) -> (store pre-activation) -> (GELU) -> (+ residual[m % P, n])
//             or, with act == 2, (* GELU'(aux[m, n])) for the MLP backward (aux in `residual`);
//             act == 3: GELU with GELU'(u) (not u) written as the pre-activation output, and
//             act == 4: (* aux[m, n]) -- the MLP forward / backward pair that keeps the erf and
//             exponential out of the backward GEMM
//             -> bf16/fp16 store, or fp32 store / fp32 accumulate (D += ...)
//
// A [M, K] and B [N, K] are K-major (row-major with K contiguous), bf16 or fp16.
// Tiles are 128 x BN x 64.  Roles inside a CTA of 6 warps:
//   warp 0: TMA producer (one elected lane) filling a STAGES-deep ring of A/B tiles
//           (128-byte swizzle) tracked by full/empty mbarriers;
//   warp 1: allocates 2*BN TMEM columns and issues tcgen05.mma (one elected lane),
//           committing each stage back to its empty barrier and each finished tile to
//           a tmem_full barrier; two accumulators let the epilogue of tile i overlap
//           the MMAs of tile i+1;
//   warps 2-9: epilogue, two warps per TMEM lane quadrant (32 rows) splitting the
//           columns; tcgen05.ld 32 columns at a time, fused bias/GELU/residual, and
//           row-major 32x32 tiles staged in shared memory so that global loads/stores
//           are coalesced (4 lanes per 64-byte row segment).
// The CTA grid is the SM count; tiles are walked with N fastest so concurrently
// running CTAs share the A tile through L2.  Every mbarrier wait is bounded by a
// %globaltimer budget: on expiry the kernel records kErrWaitTimeout in the device error
// word, stops issuing work, and still frees its TMEM before returning.
#include <cuda.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace nsw {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16: 128 bytes = one swizzle row
constexpr int kEpiWarps = 8;                   // 2 warps per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer + MMA + epilogue
constexpr int kStageRow = 32;                   // staging row: 32 elements (64 bytes)

// element offset of 16-byte chunk c (0..3) of staging row r: chunk c ^ ((r >> 1) & 3), the TMA
// SWIZZLE_64B pattern for 64-byte rows (buffers are 512-byte aligned); a warp writing one row per
// lane, or reading 4 chunks of 8 rows, hits distinct banks
__device__ __forceinline__ int stg_off(int r, int c) { return r * kStageRow + ((c ^ ((r >> 1) & 3)) << 3); }
constexpr unsigned long long kWaitBudgetNs = 4000000000ull;  // 4 s

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; returns false (and raises the abort flag) on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitBudgetNs) {
        *abort_flag = 1;
        record_error(err, kErrWaitTimeout);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// named barrier of the epilogue warps only (the producer / MMA warps keep running)
__device__ __forceinline__ void epi_sync(int warps = kEpiWarps) {
  asm volatile("bar.sync 1, %0;" ::"r"(warps * 32) : "memory");
}

__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO), LBO unused (1),
  // descriptor version 1, layout type 2 (SWIZZLE_128B).
  const uint32_t a = smem_u32(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// tcgen05.ld without the wait, and the wait with the loaded registers as in-out operands so no
// use of them can be scheduled before it (double-buffered TMEM reads in the epilogue)
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// synchronous form: the wait names the loaded registers, so no use of them precedes it
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  tmem_wait_ld(r);
}

// system-scope flag publication / observation (peer GPUs over NVLink)
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// wait (bounded) until *p >= v (wrap-safe); false on timeout (error recorded)
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* p, uint32_t v, int* err) {
  if ((int)(ld_acquire_sys(p) - v) >= 0) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t spin = 0;; ++spin) {
    if ((int)(ld_acquire_sys(p) - v) >= 0) return true;
    if ((spin & 63u) == 63u) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 4000000000ull) {
        record_error(err, kErrWaitTimeout);
        return false;
      }
    }
  }
}

// TMA store of a 32 x 32 tile (SWIZZLE_64B staging in smem) and its bulk-group bookkeeping
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

struct EpiParams {
  CUtensorMap map_d;    // TMA store maps (32 x 32 box, SWIZZLE_64B) of D and the pre-activation;
  CUtensorMap map_pre;  // used when tma_out is set (16-bit D, N % 8 == 0)
  CUtensorMap map_res;  // TMA load map of the residual / aux tensor (same box and swizzle)
  int tma_out;
  void* D;
  int64_t M, N, ldd;
  const float* bias;
  const void* residual;
  int64_t ldr, res_period;
  void* preact;
  int act;
  int out_f32;
  int accumulate;
  float alpha;
  // Tensor-parallel all-reduce fused into the epilogue (ar_world > 1; 16-bit D, no
  // pre-activation / GELU).  Every rank's symmetric buffer ar_part[r] has one [M, N] slot per rank
  // (slot s at s * M * N).  Each rank's CTA drains its tile as a 16-bit partial into slot `rank` of
  // its own buffer, releases the accumulator, pushes the tile with plain stores into slot `rank`
  // of every peer's buffer (posted NVLink writes: no warp waits on a remote round trip), publishes
  // a per-tile ready flag to every peer, and, once every peer's flag for the tile is seen, sums the
  // W slots of its own buffer (local reads only) before bias / residual / store.  Flags (uint32 words): [0] the epoch of
  // the last finished launch, [1] CTAs of this rank that finished (all launches), [2 + r] CTAs
  // of rank r that finished reading this rank's partials (all launches), [kArFlagBase + r * tiles
  // + t] the epoch in which rank r published its partial of tile t.  Epochs increase by one per
  // launch and counters by the grid size, so nothing is ever reset (and a captured CUDA graph
  // replays correctly); every rank launches the same grid.
  int ar_world, ar_rank;
  int64_t ar_tiles;
  void* ar_part[8];
  uint32_t* ar_flags[8];
  long long* ar_stamps;  // phase timestamps (nullptr: off)
};
constexpr int kArFlagBase = 16;

// Epilogue of one warp for one accumulator tile: rows [row_base, row_base + 32) (the warp's
// TMEM lane quadrant) and columns [n0 + half * BN/2, n0 + (half + 1) * BN/2).
// The 32-column chunks of a tile one epilogue warp drains: begin, begin + step, ... (n of them).
// Eight warps: two per TMEM lane quadrant, each a contiguous half of the columns.  Twelve warps:
// three per quadrant, warp j taking chunks j, j + 3, j + 6.
struct ChunkSet {
  int begin, step, n;
};

template <typename T, int BN>
struct EpiWarp {
  static constexpr int kChunks = BN / 64;  // most chunks one warp drains

  // TMEM -> registers -> fused bias / GELU / residual -> stores.  Full 32-column chunks of a
  // 16-bit D leave through TMA stores: the warp writes the chunk into one of its two 2 KB staging
  // buffers (32 rows x 64 bytes, SWIZZLE_64B) and lane 0 issues one bulk tensor store, so no
  // lane loads the tile back or issues global stores; the TMEM read of the next chunk is in
  // flight meanwhile.  `ring` counts this warp's staging uses across tiles.
  // DB: double-buffered TMEM reads (the next chunk's load in flight while this one is
  // processed); without it (twelve epilogue warps, 128 registers) each chunk is loaded and waited
  // for in turn and the other warps of the quadrant cover the latency.
  template <bool DB = true>
  __device__ __forceinline__ void drain(const EpiParams& ep, T* stg, uint32_t t_row, int64_t row_base, int64_t n0,
                                        ChunkSet cs, int lane, uint32_t& ring) {
    const int sub_r = lane >> 2, sub_c = (lane & 3) * 8;
    const int64_t row = row_base + lane;
    const bool row_ok = row < ep.M;
    uint32_t r[DB ? 2 : 1][32];
    if (DB) {
      tmem_ld32_async(t_row + (uint32_t)(cs.begin * 32), r[0]);
      tmem_wait_ld(r[0]);
    }
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      if (cc >= cs.n) break;
      const int c = cs.begin + cc * cs.step;
      uint32_t* rc = r[DB ? (cc & 1) : 0];
      if (!DB) {
        tmem_ld32_async(t_row + (uint32_t)(c * 32), rc);
        tmem_wait_ld(rc);
      } else if (cc + 1 < cs.n) {
        tmem_ld32_async(t_row + (uint32_t)((c + cs.step) * 32), r[(cc + 1) & 1]);
      }
      const int64_t nb = n0 + c * 32;
      if (nb < ep.N) {  // warp-uniform
        const bool full = nb + 32 <= ep.N;
        float f[32];
        if (ep.alpha != 1.f) {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(rc[j]) * ep.alpha;
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(rc[j]);
        }
        if (ep.bias) {
          if (full) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 b4 = __ldg(reinterpret_cast<const float4*>(ep.bias + nb) + v);
              f[4 * v] += b4.x;
              f[4 * v + 1] += b4.y;
              f[4 * v + 2] += b4.z;
              f[4 * v + 3] += b4.w;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (nb + j < ep.N) f[j] += ep.bias[nb + j];
          }
        }
        if (!full || ep.out_f32 || !ep.tma_out) {
          direct_stores(ep, f, row, row_ok, nb, full);
        } else {
          const int m_tile = (int)row_base, n_tile = (int)nb;
          if (ep.act == 3) {  // GELU, and GELU'(u) kept for the backward (one erf / exp per element)
            float g[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const GeluParts gp = gelu_parts_fast(f[j]);
              g[j] = gp.cdf + f[j] * gp.pdf;
              f[j] *= gp.cdf;
            }
            if (ep.preact) stage_store(&ep.map_pre, g, stg, lane, n_tile, m_tile, ring);
          } else if (ep.preact) {
            stage_store(&ep.map_pre, f, stg, lane, n_tile, m_tile, ring);
          }
          if (ep.act == 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = gelu_fast(f[j]);
          }
          if (ep.residual) {
            // (the kernel's RT form brings residual tiles in by TMA; this is the fallback)
            // coalesced loads (lane -> row sub_r + 8 i, 8-column group sub_c) -> this lane's row,
            // through a staging buffer
            uint4 rv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int64_t rr = row_base + sub_r + 8 * i;
              rv[i] = make_uint4(0, 0, 0, 0);
              if (rr < ep.M)
                rv[i] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(ep.residual) +
                                                       (rr % ep.res_period) * ep.ldr + nb + sub_c);
            }
            T* buf = stg + (ring & 1) * (32 * kStageRow);
            if (lane == 0) bulk_wait_read_1();
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i)
              *reinterpret_cast<uint4*>(buf + stg_off(sub_r + 8 * i, sub_c >> 3)) = rv[i];
            __syncwarp();
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float rr8[8];
              unpack8<T>(*reinterpret_cast<const uint4*>(buf + stg_off(lane, v)), rr8);
              if (ep.act == 2) {
#pragma unroll
                for (int j = 0; j < 8; ++j) f[8 * v + j] *= gelu_grad_fast(rr8[j]);
              } else if (ep.act == 4) {
#pragma unroll
                for (int j = 0; j < 8; ++j) f[8 * v + j] *= rr8[j];
              } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) f[8 * v + j] += rr8[j];
              }
            }
            __syncwarp();
          }
          stage_store(&ep.map_d, f, stg, lane, n_tile, m_tile, ring);
        }
      }
      if (DB && cc + 1 < cs.n) tmem_wait_ld(r[(cc + 1) & 1]);
    }
  }

  // Residual / aux by TMA (the kernel's RT form): lane 0 loads the warp's kChunks 32 x 32 tiles of
  // the residual into the warp's kChunks buffers (same SWIZZLE_64B layout as the output staging)
  // before the accumulator wait; the drain reads each lane's row there, combines it with the
  // accumulator row, writes the result back in place and stores it by TMA from the same buffer.
  // Earlier stores from these buffers must have read them first.  Returns the bytes expected.
  __device__ __forceinline__ static void issue_res(const EpiParams& ep, T* bufs, uint64_t* bar, int64_t row_base,
                                                   int64_t n0, ChunkSet cs, int lane) {
    if (lane != 0) return;
    bulk_wait_read_0();
    uint32_t bytes = 0;
    for (int cc = 0; cc < cs.n; ++cc)
      if (n0 + (cs.begin + cc * cs.step) * 32 < ep.N) bytes += 32 * kStageRow * sizeof(T);
    mbar_expect_tx(bar, bytes);
    const int rrow = (int)(row_base % ep.res_period);
    for (int cc = 0; cc < cs.n; ++cc) {
      const int64_t nb = n0 + (cs.begin + cc * cs.step) * 32;
      if (nb < ep.N) tma_load_2d(bufs + cc * 32 * kStageRow, &ep.map_res, bar, (int)nb, rrow);
    }
  }

  template <bool DB = true>
  __device__ __forceinline__ void drain_res(const EpiParams& ep, T* bufs, uint32_t t_row, int64_t row_base,
                                            int64_t n0, ChunkSet cs, int lane) {
    uint32_t r[DB ? 2 : 1][32];
    if (DB) {
      tmem_ld32_async(t_row + (uint32_t)(cs.begin * 32), r[0]);
      tmem_wait_ld(r[0]);
    }
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      if (cc >= cs.n) break;
      const int c = cs.begin + cc * cs.step;
      uint32_t* rc = r[DB ? (cc & 1) : 0];
      if (!DB) {
        tmem_ld32_async(t_row + (uint32_t)(c * 32), rc);
        tmem_wait_ld(rc);
      } else if (cc + 1 < cs.n) {
        tmem_ld32_async(t_row + (uint32_t)((c + cs.step) * 32), r[(cc + 1) & 1]);
      }
      const int64_t nb = n0 + c * 32;
      if (nb < ep.N) {  // warp-uniform
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(rc[j]) * ep.alpha;
        if (ep.bias) {
          if (nb + 32 <= ep.N) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 b4 = __ldg(reinterpret_cast<const float4*>(ep.bias + nb) + v);
              f[4 * v] += b4.x;
              f[4 * v + 1] += b4.y;
              f[4 * v + 2] += b4.z;
              f[4 * v + 3] += b4.w;
            }
          } else {
            for (int j = 0; j < 32 && nb + j < ep.N; ++j) f[j] += ep.bias[nb + j];
          }
        }
        if (ep.act == 1) {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = gelu_fast(f[j]);
        }
        T* buf = bufs + cc * 32 * kStageRow;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float rr8[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(buf + stg_off(lane, v)), rr8);
          if (ep.act == 2) {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[8 * v + j] *= gelu_grad_fast(rr8[j]);
          } else if (ep.act == 4) {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[8 * v + j] *= rr8[j];
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[8 * v + j] += rr8[j];
          }
          *reinterpret_cast<uint4*>(buf + stg_off(lane, v)) = pack8<T>(&f[8 * v]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) tma_store_2d(&ep.map_d, buf, (int)nb, (int)row_base);
      }
      if (DB && cc + 1 < cs.n) tmem_wait_ld(r[(cc + 1) & 1]);
    }
  }

  // This lane's row of a 32-column chunk into the next staging buffer, then one TMA store.
  __device__ __forceinline__ static void stage_store(const CUtensorMap* map, const float* f, T* stg, int lane,
                                                     int n_tile, int m_tile, uint32_t& ring) {
    T* buf = stg + (ring & 1) * (32 * kStageRow);
    if (lane == 0) bulk_wait_read_1();  // the store that last used this buffer has read it
    __syncwarp();
#pragma unroll
    for (int v = 0; v < 4; ++v) *reinterpret_cast<uint4*>(buf + stg_off(lane, v)) = pack8<T>(&f[8 * v]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) tma_store_2d(map, buf, n_tile, m_tile);
    ++ring;
  }

  // All-reduce mode, step 1: this warp's part of the accumulator as a 16-bit partial in slot `rank`
  // of the rank's own symmetric buffer (this lane's row, 64 contiguous bytes per 32-column chunk).
  __device__ __forceinline__ void drain_partial(const EpiParams& ep, uint32_t t_row, int64_t row_base, int64_t n0,
                                                int half, int lane) {
    const int64_t row = row_base + lane;
    T* part = reinterpret_cast<T*>(ep.ar_part[ep.ar_rank]) + (int64_t)ep.ar_rank * ep.M * ep.N;
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int c = half * kChunks + cc;
      uint32_t r[32];
      tmem_ld32(t_row + (uint32_t)(c * 32), r);
      const int64_t nb = n0 + c * 32;
      if (nb >= ep.N || row >= ep.M) continue;
      float f[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]) * ep.alpha;
      uint4* dst = reinterpret_cast<uint4*>(part + row * ep.N + nb);
#pragma unroll
      for (int v = 0; v < 4; ++v) dst[v] = pack8<T>(&f[8 * v]);
    }
  }

  // All-reduce mode, step 2: copy this warp's block of the partial (rows [row_base, row_base + 32) x
  // columns [n0 + half * BN/2, n0 + (half + 1) * BN/2), just written to the own slot and still in L2)
  // into slot `rank` of every peer's buffer.  Lanes walk the block row-contiguously (16 bytes each, a
  // 128-column row half is 16 lanes), so each warp store is two whole 256-byte row segments over
  // NVLink; eight rows' loads are in flight per lane before their stores.  The stores are posted
  // (nothing waits for them here); the caller fences them system-wide before the tile's flag is
  // published, after other work has given them time to land.
  __device__ __forceinline__ void push_partial(const EpiParams& ep, int64_t row_base, int64_t n0, int half,
                                               int lane) {
    constexpr int kLanesPerRow = (BN / 2) * (int)sizeof(T) / 16;
    constexpr int kRowsPerStep = 32 / kLanesPerRow;
    constexpr int kUnroll = 4;
    const int64_t col = n0 + half * (BN / 2) + (lane % kLanesPerRow) * 8;
    const int64_t slot = (int64_t)ep.ar_rank * ep.M * ep.N;
    const T* own = reinterpret_cast<const T*>(ep.ar_part[ep.ar_rank]) + slot;
#pragma unroll 1
    for (int r0 = 0; r0 < 32; r0 += kRowsPerStep * kUnroll) {
      uint4 v[kUnroll];
      int64_t off[kUnroll];
      bool ok[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t row = row_base + r0 + u * kRowsPerStep + lane / kLanesPerRow;
        ok[u] = col < ep.N && row < ep.M;
        off[u] = row * ep.N + col;
        if (ok[u]) v[u] = *reinterpret_cast<const uint4*>(own + off[u]);
      }
#pragma unroll
      for (int q = 1; q < 8; ++q) {
        if (q >= ep.ar_world) break;
        const int r = (ep.ar_rank + q) % ep.ar_world;
        T* dst = reinterpret_cast<T*>(ep.ar_part[r]) + slot;
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (ok[u]) *reinterpret_cast<uint4*>(dst + off[u]) = v[u];
      }
    }
  }

  // All-reduce mode, step 3 (every rank's partial of the tile is in this rank's slots): sum the W
  // slots of the own buffer (local reads, past L1), add bias and residual, store D.  Same block and
  // lane walk as push_partial; two rows per lane are in flight at once, each with every slot, and the
  // sum runs in rank order 0 .. W-1 on every rank, so all ranks store identical results.
  __device__ __forceinline__ void reduce_store(const EpiParams& ep, int64_t row_base, int64_t n0, int half,
                                               int lane) {
    constexpr int kLanesPerRow = (BN / 2) * (int)sizeof(T) / 16;  // 16-byte pieces in a row half
    constexpr int kRowsPerStep = 32 / kLanesPerRow;
    constexpr int kUnroll = 4;  // row steps per round: 8 rows of this warp's block per lane group
    const int64_t col = n0 + half * (BN / 2) + (lane % kLanesPerRow) * 8;
    const bool col_ok = col < ep.N;
    const int64_t slot = ep.M * ep.N;
    const T* mine = reinterpret_cast<const T*>(ep.ar_part[ep.ar_rank]);
    float b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = 0.f;
    if (ep.bias && col_ok) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(ep.bias + col) + 1);
      b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w, b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
    }
#pragma unroll 1
    for (int r0 = 0; r0 < 32; r0 += kRowsPerStep * kUnroll) {
      int64_t off[kUnroll], rows[kUnroll];
      bool ok[kUnroll];
      uint4 res[kUnroll], s0[kUnroll], s1[kUnroll];
      float f[kUnroll][8];
      // slots 0 and 1 and the residual of kUnroll row steps in flight at once (one round trip for
      // two ranks); further slots follow one by one.  The sum runs in rank order 0 .. W-1, the same
      // on every rank.
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t row = row_base + r0 + u * kRowsPerStep + lane / kLanesPerRow;
        rows[u] = row;
        ok[u] = col_ok && row < ep.M;
        off[u] = row * ep.N + col;
        if (ok[u]) {
          s0[u] = __ldcg(reinterpret_cast<const uint4*>(mine + off[u]));
          s1[u] = __ldcg(reinterpret_cast<const uint4*>(mine + slot + off[u]));
          if (ep.residual)
            res[u] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(ep.residual) +
                                                         (row % ep.res_period) * ep.ldr + col));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float x[8], y[8];
        unpack8<T>(s0[u], x);
        unpack8<T>(s1[u], y);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[u][i] = x[i] + y[i];
      }
      for (int r = 2; r < ep.ar_world; ++r) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (ok[u]) s0[u] = __ldcg(reinterpret_cast<const uint4*>(mine + (int64_t)r * slot + off[u]));
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          float x[8];
          unpack8<T>(s0[u], x);
#pragma unroll
          for (int i = 0; i < 8; ++i) f[u][i] += x[i];
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (!ok[u]) continue;
#pragma unroll
        for (int i = 0; i < 8; ++i) f[u][i] += b[i];
        if (ep.residual) {
          float x[8];
          unpack8<T>(res[u], x);
#pragma unroll
          for (int i = 0; i < 8; ++i) f[u][i] += x[i];
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(ep.D) + rows[u] * ep.ldd + col) = pack8<T>(f[u]);
      }
    }
  }

  // Ragged column edge, fp32 output, or no TMA maps: per-row stores of this lane's row.
  __device__ __forceinline__ void direct_stores(const EpiParams& ep, float* f, int64_t row, bool row_ok, int64_t nb,
                                                bool full) {
    if (!row_ok) return;
    if (ep.preact) {
      T* pp = reinterpret_cast<T*>(ep.preact) + row * ep.ldd + nb;
      for (int j = 0; j < 32 && nb + j < ep.N; ++j) pp[j] = from_f<T>(ep.act == 3 ? gelu_grad_fast(f[j]) : f[j]);
    }
    if (ep.act == 1 || ep.act == 3) {
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = gelu_fast(f[j]);
    }
    if (ep.residual) {
      const T* rp = reinterpret_cast<const T*>(ep.residual) + (row % ep.res_period) * ep.ldr + nb;
      if (ep.act == 2) {
        for (int j = 0; j < 32 && nb + j < ep.N; ++j) f[j] *= gelu_grad_fast(to_f(rp[j]));
      } else if (ep.act == 4) {
        for (int j = 0; j < 32 && nb + j < ep.N; ++j) f[j] *= to_f(rp[j]);
      } else {
        for (int j = 0; j < 32 && nb + j < ep.N; ++j) f[j] += to_f(rp[j]);
      }
    }
    if (ep.out_f32) {
      float* dp = reinterpret_cast<float*>(ep.D) + row * ep.ldd + nb;
      if (full) {
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float4 o = make_float4(f[4 * v], f[4 * v + 1], f[4 * v + 2], f[4 * v + 3]);
          if (ep.accumulate) {
            const float4 old = reinterpret_cast<float4*>(dp)[v];
            o.x += old.x;
            o.y += old.y;
            o.z += old.z;
            o.w += old.w;
          }
          reinterpret_cast<float4*>(dp)[v] = o;
        }
      } else {
        for (int j = 0; j < 32 && nb + j < ep.N; ++j) dp[j] = ep.accumulate ? dp[j] + f[j] : f[j];
      }
    } else {
      T* dp = reinterpret_cast<T*>(ep.D) + row * ep.ldd + nb;
      if (full) {
#pragma unroll
        for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dp)[v] = pack8<T>(&f[8 * v]);
      } else {
        for (int j = 0; j < 32 && nb + j < ep.N; ++j) dp[j] = from_f<T>(f[j]);
      }
    }
  }
};

// RT (residual by TMA): one 2 KB buffer per 32-column chunk of a warp's half tile (the residual
// tile lands there and the result leaves from there); otherwise two 2 KB staging buffers per warp.
template <typename T, int BN, int STAGES, bool RT, int EW>
struct Smem {
  static constexpr int kBufs = RT ? (EW == 8 ? BN / 64 : (BN / 32 + EW / 4 - 1) / (EW / 4)) : 2;
  alignas(1024) T a[STAGES][BM * BK];
  alignas(1024) T b[STAGES][BN * BK];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t res_full[EW];  // RT: a warp's residual tiles landed
  uint64_t pushed[2];     // all-reduce: every epilogue warp has pushed the tile (alternate tiles)
  uint64_t published[2];  // all-reduce: the publisher warp has published that tile's flag
  alignas(1024) T stage[EW][kBufs * 32 * kStageRow];
  uint32_t tmem_base;
  int abort_flag;
  int epi_stop;  // all-reduce epilogue: written by its leader only, read after a named barrier
};

// PUB: the fused tensor-parallel all-reduce form, with one more warp (the publisher, after the
// epilogue warps) that fences each tile's pushed partials system-wide and publishes its flag, so the
// epilogue warps never wait for a system-scope fence.
template <typename T, int BN, int STAGES, bool RT, int EW, bool PUB = false>
__global__ void __launch_bounds__(64 + 32 * EW + (PUB ? 32 : 0), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                int64_t M, int64_t N, int64_t K, const __grid_constant__ EpiParams ep, uint32_t idesc,
                int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // align the working area to 1024 B (the swizzle atom)
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto& S = *reinterpret_cast<Smem<T, BN, STAGES, RT, EW>*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m_tiles = (M + BM - 1) / BM;
  const int64_t n_tiles = (N + BN - 1) / BN;
  const int64_t num_tiles = m_tiles * n_tiles;
  const int k_blocks = (int)((K + BK - 1) / BK);
  volatile int* abort_flag = &S.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S.tmem_full[a], 1);
      mbar_init(&S.tmem_empty[a], EW);
    }
    for (int w = 0; w < EW; ++w) mbar_init(&S.res_full[w], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.pushed[b], EW);
      mbar_init(&S.published[b], 1);
    }
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S.tmem_base)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (int)((tile / n_tiles) * BM);
        const int n0 = (int)((tile % n_tiles) * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1, abort_flag, err)) break;
          mbar_expect_tx(&S.full[stage], (uint32_t)((BM + BN) * BK * sizeof(T)));
          tma_load_2d(S.a[stage], &map_a, &S.full[stage], kb * BK, m0);
          tma_load_2d(S.b[stage], &map_b, &S.full[stage], kb * BK, n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int64_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&S.tmem_empty[acc], acc_phase ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&S.full[stage], phase, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = smem_desc_sw128(&S.a[stage][k * 16]);
            const uint64_t db = smem_desc_sw128(&S.b[stage][k * 16]);
            umma_f16(d_tmem, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&S.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&S.tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else if (PUB && warp == 2 + EW) {
    // ------------------------------------------------------------------ publisher (all-reduce)
    // tile i of this CTA: once every epilogue warp has pushed it (pushed[i & 1], its (i >> 1)-th
    // phase), one system fence orders those stores (cumulatively, through the mbarrier's release /
    // acquire) before the tile's ready flag in every peer's flag words
    if (lane == 0) {
      uint32_t* my_flags = ep.ar_flags[ep.ar_rank];
      const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags) + 1u;
      int64_t i = 0;
      for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
        if (!mbar_wait(&S.pushed[i & 1], (uint32_t)((i >> 1) & 1), abort_flag, err)) break;
        fence_acq_rel_sys();  // with the relaxed flag store below: a release at system scope
        for (int r = 0; r < ep.ar_world; ++r)
          if (r != ep.ar_rank) st_relaxed_sys(ep.ar_flags[r] + kArFlagBase + ep.ar_rank * ep.ar_tiles + tile, epoch);
        mbar_arrive(&S.published[i & 1]);
      }
    }
  } else if (PUB) {
    // ------------------------------------------------------------------ epilogue + all-reduce
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    const bool leader = ew == 0 && lane == 0;  // publishes and observes flags for the CTA
    T* stg = S.stage[ew];
    uint32_t ring = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t* my_flags = ep.ar_flags[ep.ar_rank];
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags) + 1u;
    bool ok = true;
    if (leader) S.epi_stop = 0;
    epi_sync();
    // Per tile t: drain the accumulator into the own slot, push it into every peer's slot (posted
    // stores), reduce the previous tile of this CTA (the peers have had a whole tile's time to
    // deliver it, so the flag wait rarely stalls, and this tile's stores drain over NVLink
    // meanwhile), fence, publish tile t's flag.  Every iteration takes exactly two epilogue
    // barriers and all warps leave on the leader's decision (S.epi_stop), so no warp is left
    // waiting at a barrier.
    int64_t prev = -1;
    int it = 0;
    // phase stamps (diagnostics): the leader of CTAs 0..3 records eight times per tile
    long long* stamp = (ep.ar_stamps && blockIdx.x < 4 && leader) ? ep.ar_stamps + (int64_t)blockIdx.x * 32 * 8
                                                                   : nullptr;
    auto mark = [&](int phase) {
      if (stamp && it < 32) stamp[it * 8 + phase] = (long long)globaltimer();
    };
    for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int64_t m0 = (tile / n_tiles) * BM;
      const int64_t n0 = (tile % n_tiles) * BN;
      const int64_t row_base = m0 + q * 32;
      EpiWarp<T, BN> epi;
      mark(0);
      const bool have = mbar_wait(&S.tmem_full[acc], acc_phase, abort_flag, err);
      mark(1);
      if (have) {
        tc_fence_after();
        epi.drain_partial(ep, tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN), row_base, n0, half,
                          lane);
      } else {
        *abort_flag = 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && have) mbar_arrive(&S.tmem_empty[acc]);  // the MMAs of the next tile may start
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
      mark(2);
      if (have) epi.push_partial(ep, row_base, n0, half, lane);  // posted stores, not yet fenced
      mark(3);
      // the previous tile: once every peer's partial of it has arrived, reduce it (while this
      // tile's pushed stores drain over NVLink)
      if (leader) {
        bool go = !*abort_flag;
        if (go && prev >= 0)
          for (int r = 0; r < ep.ar_world && go; ++r)
            if (r != ep.ar_rank) go = wait_flag_geq(my_flags + kArFlagBase + r * ep.ar_tiles + prev, epoch, err);
        if (!go) *abort_flag = 1;
        S.epi_stop = go ? 0 : 1;
      }
      epi_sync();
      mark(4);
      if (*reinterpret_cast<volatile int*>(&S.epi_stop)) {
        ok = false;
        break;
      }
      if (prev >= 0) epi.reduce_store(ep, (prev / n_tiles) * BM + q * 32, (prev % n_tiles) * BN, half, lane);
      mark(5);
      // hand this tile's pushes to the publisher warp (its fence and flag); the barrier it reuses two
      // tiles later must have been consumed first (never waits in practice)
      __syncwarp();
      if (lane == 0 && have) {
        bool fine = it < 2 || mbar_wait(&S.published[it & 1], (uint32_t)(((it >> 1) - 1) & 1), abort_flag, err);
        if (fine) mbar_arrive(&S.pushed[it & 1]);
      }
      mark(6);
      mark(7);
      prev = tile;
    }
    if (ok && prev >= 0) {  // the last tile of this CTA
      if (leader) {
        bool go = true;
        for (int r = 0; r < ep.ar_world && go; ++r)
          if (r != ep.ar_rank) go = wait_flag_geq(my_flags + kArFlagBase + r * ep.ar_tiles + prev, epoch, err);
        if (!go) *abort_flag = 1;
        S.epi_stop = go ? 0 : 1;
      }
      epi_sync();
      if (!*reinterpret_cast<volatile int*>(&S.epi_stop)) {
        EpiWarp<T, BN> epi;
        epi.reduce_store(ep, (prev / n_tiles) * BM + q * 32, (prev % n_tiles) * BN, half, lane);
      }
    }
    (void)stg;
    (void)ring;
    // this CTA has read its peers' partials; before the launch ends, every CTA of every peer has
    // read this rank's partials (the next launch overwrites them)
    epi_sync();
    if (leader) {
      __threadfence_system();
      for (int r = 0; r < ep.ar_world; ++r)
        if (r != ep.ar_rank) red_release_sys_add(ep.ar_flags[r] + 2 + ep.ar_rank, 1u);
      const uint32_t target = epoch * gridDim.x;
      for (int r = 0; r < ep.ar_world; ++r)
        if (r != ep.ar_rank) wait_flag_geq(my_flags + 2 + r, target, err);
      // the last CTA of this launch on this rank advances the epoch (all CTAs have read it)
      if (atomicAdd(my_flags + 1, 1u) == target - 1u) atomicExch(my_flags, epoch);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;   // TMEM lane quadrant this warp may access
    const int j = ew >> 2;    // this warp's index among the warps of its quadrant
    ChunkSet cs;
    if (EW == 8) {
      cs = {j * (BN / 64), 1, BN / 64};
    } else {
      constexpr int G = EW / 4;
      cs = {j, G, (BN / 32 - j + G - 1) / G};
    }
    T* stg = S.stage[ew];
    uint32_t ring = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t res_phase = 0;
    bool res_pending = false;
    for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int64_t m0 = (tile / n_tiles) * BM;
      const int64_t n0 = (tile % n_tiles) * BN;
      const int64_t row_base = m0 + q * 32;
      EpiWarp<T, BN> epi;
      if constexpr (RT) {
        EpiWarp<T, BN>::issue_res(ep, stg, &S.res_full[ew], row_base, n0, cs, lane);
        res_pending = true;
      }
      if (!mbar_wait(&S.tmem_full[acc], acc_phase, abort_flag, err)) break;
      tc_fence_after();
      if constexpr (RT) {
        if (!mbar_wait(&S.res_full[ew], res_phase, abort_flag, err)) break;
        res_phase ^= 1;
        res_pending = false;
        epi.template drain_res<EW == 8>(ep, stg, tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN),
                                        row_base, n0, cs, lane);
      } else {
        epi.template drain<EW == 8>(ep, stg, tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN),
                                    row_base, n0, cs, lane, ring);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // the warp's TMA stores have completed
    // after an abort, residual loads still in flight land before the shared memory is released
    // (bounded; not recorded again)
    if (RT && res_pending && lane == 0) {
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(&S.res_full[ew], res_phase) && globaltimer() - t0 < kWaitBudgetNs) {
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN));
  }
}


// ============================================================================ 2-SM GEMM
// A CTA pair (cluster of 2 on neighbouring SMs) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2: each CTA loads its own 128 rows of A and its 128-row half of B (plain
// TMA loads into its own shared memory, no multicast) and receives 128 x 256 accumulator rows in
// its own TMEM.  Per SM, an MMA of the pair reads 8 KB of operands per K=16 step instead of 12 KB
// for a 128 x 256 single-CTA tile, which keeps the tensor core's operand reads plus the TMA writes
// within the SM's shared-memory bandwidth.
//   leader (rank 0): warp 1 issues every MMA of the pair and commits, multicast to both CTAs,
//     the stage-free barriers and the accumulator-ready barrier;
//   both CTAs: warp 0 is the TMA producer (its bytes complete the LEADER's stage barrier, which
//     the leader arms with both CTAs' byte count); warps 2-9 drain their CTA's accumulator
//     exactly as the single-CTA kernel does and release it on the leader's barrier.
constexpr int BM2 = 256;  // rows of a pair tile (128 per CTA)
constexpr int BN2 = 256;  // columns of a pair tile (B rows: 128 per CTA)

template <typename T, int STAGES>
struct Smem2 {
  alignas(1024) T a[STAGES][BM * BK];
  alignas(1024) T b[STAGES][(BN2 / 2) * BK];
  uint64_t full[STAGES];    // leader: both CTAs' TMA bytes of a stage have landed
  uint64_t empty[STAGES];   // each CTA: the pair's MMAs are done with this stage
  uint64_t tmem_full[2];    // each CTA: accumulator ready
  uint64_t tmem_empty[2];   // leader: all 2 x kEpiWarps epilogue warps released the accumulator
  uint64_t done;            // each CTA: the peer has finished its last tile
  alignas(1024) T stage[kEpiWarps][2 * 32 * kStageRow];  // two 2 KB staging buffers per epilogue warp
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// TMA load into this CTA's smem whose completion is counted on an mbarrier of either CTA of the pair
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// arrive on the barrier at this offset in both CTAs of the pair once the pair's MMAs are done
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)0x3)
      : "memory");
}

template <typename T, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 int64_t M, int64_t N, int64_t K, const __grid_constant__ EpiParams ep, uint32_t idesc,
                int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto& S = *reinterpret_cast<Smem2<T, STAGES>*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int64_t m_tiles = (M + BM2 - 1) / BM2;
  const int64_t n_tiles = (N + BN2 - 1) / BN2;
  const int64_t num_tiles = m_tiles * n_tiles;
  const int k_blocks = (int)((K + BK - 1) / BK);
  volatile int* abort_flag = &S.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S.tmem_full[a], 1);
      mbar_init(&S.tmem_empty[a], 2 * kEpiWarps);
    }
    mbar_init(&S.done, 1);
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  if (warp == 1) {  // both CTAs take part in the pair's allocation
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(2 * BN2));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync_all();  // barrier initialisation and the TMEM address are visible to both CTAs
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = map_rank(&S.full[0], 0);
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
        const int m0 = (int)((tile / n_tiles) * BM2) + (int)rank * BM;
        const int nb0 = (int)((tile % n_tiles) * BN2) + (int)rank * (BN2 / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1, abort_flag, err)) break;
          if (rank == 0) mbar_expect_tx(&S.full[stage], (uint32_t)(2 * (BM + BN2 / 2) * BK * sizeof(T)));
          tma_load_2d_pair(S.a[stage], &map_a, full_leader + 8u * stage, kb * BK, m0);
          tma_load_2d_pair(S.b[stage], &map_b, full_leader + 8u * stage, kb * BK, nb0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int64_t tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
        if (!mbar_wait(&S.tmem_empty[acc], acc_phase ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN2);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&S.full[stage], phase, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma2_f16(d_tmem, smem_desc_sw128(&S.a[stage][k * 16]), smem_desc_sw128(&S.b[stage][k * 16]), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
          umma2_commit_both(&S.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma2_commit_both(&S.tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    T* stg = S.stage[ew];
    uint32_t ring = 0;
    const uint32_t empty_leader = map_rank(&S.tmem_empty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t tile = pair; tile < num_tiles; tile += npairs) {
      const int64_t m0 = (tile / n_tiles) * BM2 + (int64_t)rank * BM;
      const int64_t n0 = (tile % n_tiles) * BN2;
      const int64_t row_base = m0 + q * 32;
      EpiWarp<T, BN2> epi;
      if (!mbar_wait(&S.tmem_full[acc], acc_phase, abort_flag, err)) break;
      tc_fence_after();
      epi.drain(ep, stg, tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN2), row_base, n0,
                ChunkSet{half * EpiWarp<T, BN2>::kChunks, 1, EpiWarp<T, BN2>::kChunks}, lane, ring);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_leader + 8u * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // the warp's TMA stores have completed
  }

  // teardown: both CTAs are past their last tile before the pair's TMEM is released
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(map_rank(&S.done, rank ^ 1u));
    int never = 0;
    mbar_wait(&S.done, 0, &never, err);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN2));
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D K-major operand [rows, K] with leading dimension ld (elements), box [BK, box_rows].
static bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int64_t ld,
                     int box_rows, int dtype) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// [M, N] 16-bit output with leading dimension ld: box of 32 x 32 elements, 64-byte swizzle
static bool make_store_map(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols, int64_t ld, int dtype) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static EpiParams epi_params(const GemmArgs& a) {
  EpiParams ep;
  memset(&ep, 0, sizeof(ep));
  ep.tma_out = !a.out_f32 && make_store_map(&ep.map_d, a.D, a.M, a.N, a.ldd, a.dtype) &&
               (!a.preact || make_store_map(&ep.map_pre, a.preact, a.M, a.N, a.ldd, a.dtype));
  ep.D = a.D;
  ep.M = a.M;
  ep.N = a.N;
  ep.ldd = a.ldd;
  ep.bias = a.bias;
  ep.residual = a.residual;
  ep.ldr = a.ldr;
  ep.res_period = a.res_period > 0 ? a.res_period : a.M;
  ep.preact = a.preact;
  ep.act = a.act;
  ep.out_f32 = a.out_f32;
  ep.accumulate = a.accumulate;
  ep.alpha = a.alpha;
  ep.ar_world = a.ar_world;
  ep.ar_rank = a.ar_rank;
  for (int r = 0; r < 8; ++r) {
    ep.ar_part[r] = r < a.ar_world ? a.ar_part[r] : nullptr;
    ep.ar_flags[r] = r < a.ar_world ? a.ar_flags[r] : nullptr;
  }
  ep.ar_stamps = a.ar_stamps;
  return ep;
}

// CTA-pair GEMM: cluster launch of 2 x (co-resident pairs, capped at the tile count)
template <typename T, int STAGES>
static cudaError_t launch2(const GemmArgs& a, cudaStream_t s) {
  CUtensorMap ma, mb;
  if (!make_map(&ma, a.A, a.M, a.K, a.lda, BM, a.dtype)) return cudaErrorInvalidValue;
  if (!make_map(&mb, a.B, a.N, a.K, a.ldb, BN2 / 2, a.dtype)) return cudaErrorInvalidValue;
  const EpiParams ep = epi_params(a);
  const uint32_t fmt = a.dtype == kBF16 ? 1u : 0u;
  const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN2 >> 3) << 17) |
                         ((uint32_t)(BM2 >> 4) << 24);
  const size_t smem = sizeof(Smem2<T, STAGES>) + 1024;
  auto k = gemm2_kernel<T, STAGES>;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t tiles = ((a.M + BM2 - 1) / BM2) * ((a.N + BN2 - 1) / BN2);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(sm_count() & ~1, 1, 1);
  static int max_pairs = 0;  // co-resident clusters of this kernel (same for every shape)
  if (!max_pairs) {
    int n = 0;
    NSW_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, k, &cfg));
    max_pairs = n > 0 ? n : 1;
  }
  int pairs = max_pairs;
  if (tiles < pairs) pairs = (int)tiles;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  NSW_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, ma, mb, a.M, a.N, a.K, ep, idesc, device_error_flag()));
  return cudaGetLastError();
}

template <typename T, int BN, int STAGES, bool RT = false, int EW = 8, bool PUB = false>
static cudaError_t launch(const GemmArgs& a, cudaStream_t s) {
  if (PUB != (a.ar_world > 1)) return cudaErrorInvalidValue;  // the all-reduce form and only it
  CUtensorMap ma, mb;
  if (!make_map(&ma, a.A, a.M, a.K, a.lda, BM, a.dtype)) return cudaErrorInvalidValue;
  if (!make_map(&mb, a.B, a.N, a.K, a.ldb, BN, a.dtype)) return cudaErrorInvalidValue;
  EpiParams ep = epi_params(a);
  if (RT && !make_store_map(&ep.map_res, const_cast<void*>(a.residual), ep.res_period, a.N, a.ldr, a.dtype))
    return cudaErrorInvalidValue;
  ep.ar_tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const uint32_t fmt = a.dtype == kBF16 ? 1u : 0u;
  const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
                         ((uint32_t)(BM >> 4) << 24);
  const size_t smem = sizeof(Smem<T, BN, STAGES, RT, EW>) + 1024;
  auto k = gemm_kernel<T, BN, STAGES, RT, EW, PUB>;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int threads = 64 + 32 * EW + (PUB ? 32 : 0);
  static int resident = 0;  // co-resident CTAs of this kernel on the whole device
  if (!resident) {
    int per_sm = 0;
    NSW_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, smem));
    resident = (per_sm > 0 ? per_sm : 1) * sm_count();
  }
  int grid = sm_count() < resident ? sm_count() : resident;
  if (tiles < grid) grid = (int)tiles;
  if (a.ar_world > 1) {
    // The fused all-reduce ends with every CTA waiting for all CTAs of every rank (read-done
    // counters), which completes only if the whole grid is resident at once.  A cooperative
    // launch guarantees that or fails to launch (for example when MPS or another context holds
    // SMs), instead of leaving the ranks to run into the bounded waits.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, ma, mb, a.M, a.N, a.K, ep, idesc, device_error_flag());
  }
  k<<<grid, threads, smem, s>>>(ma, mb, a.M, a.N, a.K, ep, idesc, device_error_flag());
  return cudaGetLastError();
}

// ============================================================================ weight gradient
// dW[m, n] (+)= sum_t dY[t, m] * X[t, n] and db[m] (+)= sum_t dY[t, m]: the weight (and bias)
// gradient of a linear layer, whose operands are token-major ([T, M] and [T, N], features
// contiguous), i.e. MN-major for the MMA.  CTA pair (cta_group::2), 256 x 256 pair tiles, the same
// warp roles as gemm2_kernel:
//   both CTAs, warp 0: TMA producer.  A stage of a CTA holds its 128 features of dY and its 128
//     features of X for 64 tokens, each as two [64 tokens x 64 features] boxes (128-byte swizzle;
//     the 64-feature blocks are 8 KB apart, the leading byte offset of the MN-major descriptor);
//   leader, warp 1: issues the MMAs (A and B MN-major in the instruction descriptor) into one TMEM
//     accumulator of 256 columns; for tiles of the first column block, when db is requested, also
//     an N = 16 MMA of the same dY stage against a tile of ones (columns 256..271: the feature sums);
//   both CTAs, warps 2-9: drain their 128 rows.
// The token range is split S ways (split-K, S chosen on the host so that S x tiles fills the pairs):
// split-major order, so the pairs running at one time read the same token slab of dY and X from L2.
// With S > 1 every (tile, split) writes its fp32 partial to a workspace [S][M_pad][N_pad] (and its
// feature sums to [S][M_pad]) and wgrad_reduce_kernel then sums the S partials in split order
// (deterministic) into D and db.  (A reduction by the last arriving split inside this kernel kept
// that pair's single accumulator from being released for microseconds: 25% slower at S = 8.)
// Bounded mbarrier waits as in the other kernels.
constexpr int WG_STAGES = 6;
constexpr int WG_ACC_COLS = 512;  // TMEM of each CTA: [0, 256) dW, [256, 272) feature sums

struct WgradParams {
  // D (and db) in up to four row segments of seg_rows rows each (the q / k / v weights of one
  // fused projection are separate gradient buffers): row m goes to D[m / seg_rows] at row m % seg_rows
  float* D[4];
  float* db[4];  // all null: no feature sums
  int64_t seg_rows;
  int64_t ldd;
  int accumulate;     // D += result
  int db_accumulate;  // db += sums
  int splits;         // partial slots: S of the uniform split, or the remainder pieces of the balanced one
  int k1;             // 0: uniform split; > 0: balanced (see wg_unit)
  float* ws;          // partials [splits][M_pad][N_pad], then feature sums [splits][M_pad]
  int64_t m_pad;      // M rounded up to the pair tile
  int64_t n_pad;      // N rounded up to the pair tile
};

// The i-th work unit of pair `pair`: a tile, a k-block range, and where its result goes (slot -1:
// straight into D; otherwise partial slot `slot`, added into D by wgrad_reduce_kernel).
//   uniform (k1 == 0): units (split, tile) in split-major order, split s taking k-blocks
//     [s nkb / S, (s + 1) nkb / S); with S == 1 every unit writes D directly;
//   balanced (k1 > 0, tiles < pairs): pair t < tiles takes tile t's k-blocks [0, k1) and writes D;
//     the other pairs share the remainder [k1, nkb) of every tile, cut into `splits` pieces, in
//     piece-major order.  k1 is chosen on the host so that both kinds of pair finish together, so no
//     pair idles when there are fewer tiles than pairs, and most of the work still runs with all
//     pairs at the same k-blocks (reading the same token slab from L2).
struct WUnit {
  int64_t tile;
  int kb0, kb1;
  int slot;
};
__device__ __forceinline__ bool wg_unit(const WgradParams& wp, int64_t tiles, int nkb, int64_t pair, int64_t npairs,
                                        int64_t i, WUnit& u) {
  if (wp.k1 == 0) {
    const int64_t v = pair + i * npairs;
    if (v >= tiles * wp.splits) return false;
    const int split = (int)(v / tiles);
    u.tile = v - (int64_t)split * tiles;
    u.kb0 = (int)((int64_t)split * nkb / wp.splits);
    u.kb1 = (int)((int64_t)(split + 1) * nkb / wp.splits);
    u.slot = wp.splits > 1 ? split : -1;
    return true;
  }
  if (pair < tiles) {
    if (i > 0) return false;
    u.tile = pair;
    u.kb0 = 0;
    u.kb1 = wp.k1;
    u.slot = -1;
    return true;
  }
  const int64_t ps = npairs - tiles;
  const int64_t v = (pair - tiles) + i * ps;
  if (v >= tiles * wp.splits) return false;
  const int piece = (int)(v / tiles);
  const int rem = nkb - wp.k1;
  u.tile = v - (int64_t)piece * tiles;
  u.kb0 = wp.k1 + (int)((int64_t)piece * rem / wp.splits);
  u.kb1 = wp.k1 + (int)((int64_t)(piece + 1) * rem / wp.splits);
  u.slot = piece;
  return true;
}

template <typename T>
struct SmemW {
  alignas(1024) T a[WG_STAGES][BM * BK];
  alignas(1024) T b[WG_STAGES][BM * BK];
  alignas(1024) T ones[8 * BK];  // this CTA's 8 rows of the N = 16 ones operand (K-major)
  uint64_t full[WG_STAGES];
  uint64_t empty[WG_STAGES];
  uint64_t tmem_full;
  uint64_t tmem_empty;
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

// MN-major, 128-byte swizzle: 64-element rows of one K index, 8-row groups 1024 B apart (SBO), and
// 64-wide MN blocks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t smem_desc_mn(const void* p, uint32_t lbo) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// named barrier of the epilogue warps (id 1) that also ANDs a predicate over them, so that a failed
// wait makes every epilogue warp leave together (none is left at a later barrier)
__device__ __forceinline__ bool epi_sync_and(bool v) {
  uint32_t out;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(out)
      : "r"(v ? 1u : 0u), "r"(kEpiWarps * 32)
      : "memory");
  return out != 0;
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    wgrad2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int64_t M,
                  int64_t N, int nkb, const __grid_constant__ WgradParams wp, uint32_t idesc, uint32_t idesc_b,
                  int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto& S = *reinterpret_cast<SmemW<T>*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int64_t m_tiles = (M + BM2 - 1) / BM2;
  const int64_t n_tiles = (N + BN2 - 1) / BN2;
  const int64_t tiles = m_tiles * n_tiles;
  const bool want_db = wp.db[0] != nullptr;
  volatile int* abort_flag = &S.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WG_STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(&S.tmem_full, 1);
    mbar_init(&S.tmem_empty, 2 * kEpiWarps);
    mbar_init(&S.done, 1);
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  // the ones operand (any layout of all ones is the same tile)
  {
    const T one = from_f<T>(1.f);
    for (int i = threadIdx.x; i < 8 * BK; i += blockDim.x) S.ones[i] = one;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(WG_ACC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = map_rank(&S.full[0], 0);
      int stage = 0;
      uint32_t phase = 0;
      WUnit un;
      for (int64_t i = 0; wg_unit(wp, tiles, nkb, pair, npairs, i, un) && !*abort_flag; ++i) {
        const int64_t tile = un.tile;
        const int m0 = (int)((tile / n_tiles) * BM2) + (int)rank * BM;
        const int nb0 = (int)((tile % n_tiles) * BN2) + (int)rank * (BN2 / 2);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1, abort_flag, err)) break;
          if (rank == 0) mbar_expect_tx(&S.full[stage], (uint32_t)(2 * 2 * BM * BK * sizeof(T)));
          const uint32_t fb = full_leader + 8u * stage;
          tma_load_2d_pair(&S.a[stage][0], &map_a, fb, m0, kb * BK);
          tma_load_2d_pair(&S.a[stage][64 * BK], &map_a, fb, m0 + 64, kb * BK);
          tma_load_2d_pair(&S.b[stage][0], &map_b, fb, nb0, kb * BK);
          tma_load_2d_pair(&S.b[stage][64 * BK], &map_b, fb, nb0 + 64, kb * BK);
          if (++stage == WG_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      WUnit un;
      for (int64_t i = 0; wg_unit(wp, tiles, nkb, pair, npairs, i, un) && !*abort_flag; ++i) {
        const bool sums = want_db && (un.tile % n_tiles) == 0;
        const int kb0 = un.kb0, kb1 = un.kb1;
        if (!mbar_wait(&S.tmem_empty, acc_phase ^ 1, abort_flag, err)) break;
        acc_phase ^= 1;
        tc_fence_after();
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&S.full[stage], phase, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // (timed against K-major operands in this kernel: the same 0.46 ms at 64800 x 4096 x 1024)
            const uint64_t da = smem_desc_mn(&S.a[stage][k * 16 * 64], 64 * BK * (uint32_t)sizeof(T));
            const uint64_t db = smem_desc_mn(&S.b[stage][k * 16 * 64], 64 * BK * (uint32_t)sizeof(T));
            const uint32_t accf = (kb > kb0 || k > 0) ? 1u : 0u;
            umma2_f16(tmem_base, da, db, idesc, accf);
            if (sums) umma2_f16(tmem_base + 256u, da, smem_desc_sw128(&S.ones[k * 16]), idesc_b, accf);
          }
          umma2_commit_both(&S.empty[stage]);
          if (++stage == WG_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma2_commit_both(&S.tmem_full);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;  // columns [128 half, 128 half + 128) of the CTA's 256
    const uint32_t empty_leader = map_rank(&S.tmem_empty, 0);
    uint32_t acc_phase = 0;
    WUnit un;
    for (int64_t i = 0; wg_unit(wp, tiles, nkb, pair, npairs, i, un); ++i) {
      const int64_t tile = un.tile;
      const bool sums = want_db && (tile % n_tiles) == 0;
      const int64_t m0 = (tile / n_tiles) * BM2 + (int64_t)rank * BM;
      const int64_t n0 = (tile % n_tiles) * BN2 + 128 * half;
      const int64_t row = m0 + q * 32 + lane;
      const bool row_ok = row < M;
      const int seg = row_ok ? (int)(row / wp.seg_rows) : 0;
      const int64_t lrow = row - (int64_t)seg * wp.seg_rows;
      if (!epi_sync_and(mbar_wait(&S.tmem_full, acc_phase, abort_flag, err))) break;
      acc_phase ^= 1;
      tc_fence_after();
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
      float sum_v = 0.f;
      if (un.slot < 0) {
        // direct: this lane's row, 128 columns, straight to D (and db)
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + (uint32_t)(128 * half + 32 * c), r);
          const int64_t col = n0 + 32 * c;
          if (row_ok && col < N) {
            float* dp = wp.D[seg] + lrow * wp.ldd + col;
            if (col + 32 <= N && (wp.ldd & 3) == 0) {
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                       __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                if (wp.accumulate) {
                  const float4 old = reinterpret_cast<const float4*>(dp)[v];
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                reinterpret_cast<float4*>(dp)[v] = o;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col + j < N) dp[j] = wp.accumulate ? dp[j] + __uint_as_float(r[j]) : __uint_as_float(r[j]);
            }
          }
        }
        if (sums && half == 0) {
          uint32_t r[32];
          tmem_ld32(trow + 256u, r);
          sum_v = __uint_as_float(r[0]);
          if (row_ok) {
            float* bp = wp.db[seg] + lrow;
            *bp = wp.db_accumulate ? *bp + sum_v : sum_v;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(empty_leader);
      } else {
        // split: this CTA's 128 rows of the partial to the workspace (wgrad_reduce_kernel sums them)
        const int64_t prow_i = m0 + q * 32 + lane;  // < m_pad
        float* prow = wp.ws + ((int64_t)un.slot * wp.m_pad + prow_i) * wp.n_pad + n0;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + (uint32_t)(128 * half + 32 * c), r);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            __stcg(reinterpret_cast<float4*>(prow + 32 * c) + v,
                   make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]), __uint_as_float(r[4 * v + 2]),
                               __uint_as_float(r[4 * v + 3])));
        }
        if (sums && half == 0) {
          uint32_t r[32];
          tmem_ld32(trow + 256u, r);
          __stcg(wp.ws + (int64_t)wp.splits * wp.m_pad * wp.n_pad + (int64_t)un.slot * wp.m_pad + prow_i,
                 __uint_as_float(r[0]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(empty_leader);
      }
    }
  }

  // teardown: both CTAs are past their last unit before the pair's TMEM is released
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(map_rank(&S.done, rank ^ 1u));
    int never = 0;
    mbar_wait(&S.done, 0, &never, err);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(WG_ACC_COLS));
}

// D[m, n] (+)= sum_s ws[s][m][n] in split order; db[m] (+)= sum_s sums[s][m].  One thread per four
// consecutive columns of a row (scalar at a ragged edge).
__global__ void wgrad_reduce_kernel(const float* __restrict__ ws, int64_t M, int64_t N,
                                    const __grid_constant__ WgradParams wp, int accumulate, int db_accumulate) {
  const int splits = wp.splits;
  const int64_t m_pad = wp.m_pad, n_pad = wp.n_pad, ldd = wp.ldd;
  const int64_t n4 = (N + 3) / 4;
  const int64_t total = M * n4;
  const int64_t plane = m_pad * n_pad;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n4, c = (i - m * n4) * 4;
    const int seg = (int)(m / wp.seg_rows);
    const float* p = ws + m * n_pad + c;
    float* dp = wp.D[seg] + (m - (int64_t)seg * wp.seg_rows) * ldd + c;
    if (c + 4 <= N && (ldd & 3) == 0) {
      float4 acc = __ldcs(reinterpret_cast<const float4*>(p));
      for (int sp = 1; sp < splits; ++sp) {
        const float4 x = __ldcs(reinterpret_cast<const float4*>(p + sp * plane));
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      if (accumulate) {
        const float4 old = *reinterpret_cast<const float4*>(dp);
        acc.x += old.x;
        acc.y += old.y;
        acc.z += old.z;
        acc.w += old.w;
      }
      *reinterpret_cast<float4*>(dp) = acc;
    } else {
      for (int j = 0; j < 4 && c + j < N; ++j) {
        float acc = p[j];
        for (int sp = 1; sp < splits; ++sp) acc += p[sp * plane + j];
        dp[j] = accumulate ? dp[j] + acc : acc;
      }
    }
  }
  if (wp.db[0]) {
    const float* sums = ws + (int64_t)splits * plane;
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < M; m += (int64_t)gridDim.x * blockDim.x) {
      float acc = sums[m];
      for (int sp = 1; sp < splits; ++sp) acc += sums[sp * m_pad + m];
      const int seg = (int)(m / wp.seg_rows);
      float* bp = wp.db[seg] + (m - (int64_t)seg * wp.seg_rows);
      *bp = db_accumulate ? *bp + acc : acc;
    }
  }
}

static int64_t wgrad_units_cost(int64_t tiles, int splits, int nkb, int pairs) {
  // the busiest pair's k-block steps (about 0.45 us each at the pair's MMA rate), plus, for a split,
  // the partials (a 256 KB partial per unit written, then read by the reduction: about 0.4 steps per
  // unit, fitted to 64800-token measurements at S = 1..9) and the reduction launch (about 4 steps)
  const int64_t units = tiles * splits;
  const int64_t waves = (units + pairs - 1) / pairs;
  const int64_t steps = waves * ((nkb + splits - 1) / splits);
  return steps + (splits > 1 ? (2 * units) / 5 + 4 : 0);
}

// Balanced schedule for tiles < pairs with the remainder in `s2` pieces: k1 such that a pair of the
// remainder (ceil(tiles s2 / (pairs - tiles)) pieces of (nkb - k1) / s2 k-blocks) ends with the first
// part.  Returns k1 (0 if it does not apply) and its cost in k-block steps.
static int wgrad_balanced(int64_t tiles, int s2, int nkb, int pairs, int64_t* cost) {
  if (tiles >= pairs || s2 < 1) return 0;
  const int64_t w2 = (tiles * s2 + (pairs - tiles) - 1) / (pairs - tiles);
  int k1 = (int)((w2 * nkb + (s2 + w2) - 1) / (s2 + w2));
  if (k1 >= nkb || k1 < 1) return 0;
  const int64_t piece = ((int64_t)(nkb - k1) + s2 - 1) / s2;
  *cost = std::max<int64_t>(k1, w2 * piece) + (2 * tiles * s2) / 5 + 4;
  return k1;
}

static int wgrad_pairs(cudaLaunchConfig_t* cfg) {
  static int max_pairs = 0;
  if (!max_pairs) {
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, wgrad2_kernel<__nv_bfloat16>, cfg) != cudaSuccess || n <= 0) n = 1;
    max_pairs = n;
  }
  return max_pairs;
}

// [T, F] token-major operand as an MN-major TMA source: dims {F, T}, box {64 features, 64 tokens}
static bool make_map_mn(CUtensorMap* map, const void* ptr, int64_t T, int64_t F, int64_t ld, int dtype) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)F, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)BK};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
static cudaError_t launch_wgrad(const WgradArgs& a, int pairs_plan, cudaStream_t s) {
  CUtensorMap ma, mb;
  if (!make_map_mn(&ma, a.dy, a.T, a.M, a.ldy, a.dtype) || !make_map_mn(&mb, a.x, a.T, a.N, a.ldx, a.dtype))
    return cudaErrorInvalidValue;
  const uint32_t fmt = a.dtype == kBF16 ? 1u : 0u;
  const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (1u << 16) |
                         ((uint32_t)(BN2 >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
  const uint32_t idesc_b = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | ((uint32_t)(16 >> 3) << 17) |
                           ((uint32_t)(BM2 >> 4) << 24);
  const size_t smem = sizeof(SmemW<T>) + 1024;
  auto k = wgrad2_kernel<T>;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  WgradParams wp;
  for (int i = 0; i < 4; ++i) {
    wp.D[i] = a.D[i];
    wp.db[i] = a.db[i];
  }
  wp.seg_rows = a.seg_rows > 0 ? a.seg_rows : a.M;
  wp.ldd = a.ldd;
  wp.accumulate = a.accumulate;
  wp.db_accumulate = a.db_accumulate;
  wp.splits = a.splits;
  wp.k1 = a.k1;
  wp.ws = a.ws;
  wp.m_pad = (a.M + BM2 - 1) / BM2 * BM2;
  wp.n_pad = (a.N + BN2 - 1) / BN2 * BN2;
  const int64_t tiles = ((a.M + BM2 - 1) / BM2) * ((a.N + BN2 - 1) / BN2);
  const int nkb = (int)((a.T + BK - 1) / BK);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(sm_count() & ~1, 1, 1);
  int pairs = wgrad_pairs(&cfg);
  if (a.k1 > 0) {
    // the balanced schedule was planned for this many pairs
    if (pairs_plan > pairs || pairs_plan <= tiles) return cudaErrorInvalidValue;
    pairs = pairs_plan;
  } else {
    const int64_t units = tiles * a.splits;
    if (units < pairs) pairs = (int)units;
  }
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  NSW_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, ma, mb, a.M, a.N, nkb, wp, idesc, idesc_b, device_error_flag()));
  NSW_CUDA_CHECK(cudaGetLastError());
  if (a.splits > 1 || a.k1 > 0) {
    const int64_t work = a.M * ((a.N + 3) / 4);
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, 8 * sm_count());
    // balanced: the direct part already holds D (with the caller's accumulate), the pieces add to it
    wgrad_reduce_kernel<<<blocks, 256, 0, s>>>(a.ws, a.M, a.N, wp, a.k1 > 0 ? 1 : a.accumulate,
                                               a.k1 > 0 ? 1 : a.db_accumulate);
  }
  return cudaGetLastError();
}

}  // namespace tc

int gemm_tcgen05_supported(const GemmArgs& a) {
  if (a.dtype != kBF16 && a.dtype != kF16) return 0;
  if (a.K % 8 || a.lda % 8 || a.ldb % 8) return 0;                    // 16-byte TMA strides
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) return 0;
  if (a.ldd % 8 || (reinterpret_cast<uintptr_t>(a.D) & 15)) return 0;  // vector stores
  if (a.residual && (a.ldr % 8 || (reinterpret_cast<uintptr_t>(a.residual) & 15))) return 0;
  if (a.preact && (reinterpret_cast<uintptr_t>(a.preact) & 15)) return 0;
  if (a.accumulate && !a.out_f32) return 0;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return 0;
  if (a.ar_world > 1) {  // fused all-reduce: plain (bias / residual) epilogue, whole 32-column chunks
    if (a.ar_world > 8 || a.ar_rank < 0 || a.ar_rank >= a.ar_world) return 0;
    if (a.preact || a.act || a.out_f32 || a.accumulate || a.N % 32) return 0;
    for (int r = 0; r < a.ar_world; ++r)
      if (!a.ar_part[r] || !a.ar_flags[r] || (reinterpret_cast<uintptr_t>(a.ar_part[r]) & 15)) return 0;
  }
  return tc::get_encode() != nullptr;
}

// impl: 0 = default, 1 = single CTA, 2 = CTA pair, 3 = single CTA with the plain-load residual
// path, 4 = single CTA with twelve epilogue warps for GELU epilogues.  The default takes the
// CTA pair for wide GEMMs whose epilogue is light (bias only, or a residual after K >= 2048):
// there the pair's lower shared-memory traffic per MMA wins; with GELU / pre-activation /
// residual epilogues after a short mainloop the single-CTA kernel is faster (measured at
// 64800 x 4096 x 1024), since a pair reuses an accumulator only when both CTAs' epilogues have
// drained it.
cudaError_t gemm_tcgen05(const GemmArgs& a, cudaStream_t s, int impl) {
  if (!gemm_tcgen05_supported(a)) return cudaErrorInvalidValue;
  const bool wide = a.N > 128;
  const bool light = a.act == 0 && !a.residual && !a.preact;
  // the fused all-reduce lives in the single-CTA kernel's epilogue
  // a residual-only epilogue after a long mainloop (fc2 forward, K = 4096) also goes to the pair:
  // its per-SM operand traffic is lower, and the epilogue is a small share of the tile
  // (measured 0.396 against 0.445 ms at 64800 x 1024 x 4096; at K = 1024 the single CTA wins)
  const bool long_res = a.residual && a.act == 0 && !a.preact && a.K >= 2048;
  const bool pair =
      a.ar_world <= 1 && (impl == 2 || (impl == 0 && wide && a.M > tc::BM && (light || long_res)));
  // residual / aux epilogue with the residual tiles brought in by TMA (three pipeline stages
  // leave room for one 2 KB buffer per 32-column chunk and epilogue warp); impl 3 forces the
  // fallback that loads residual chunks with plain loads in the drain
  const int64_t period = a.res_period > 0 ? a.res_period : a.M;
  const bool rt = wide && a.residual && !a.preact && a.act != 3 && !a.out_f32 && a.ar_world <= 1 && !pair &&
                  impl != 3 && a.N % 8 == 0 && period % 32 == 0;
  // impl 4: twelve epilogue warps (three per TMEM lane quadrant, 128 registers, single-buffered
  // TMEM reads) for the GELU / GELU' epilogues; measured within noise of eight at
  // 64800 x 4096 x 1024 (0.538 against 0.548 ms for GELU, 0.614 against 0.581 ms for GELU' with
  // the TMA residual), so eight is the default
  const bool gelu12 = impl == 4 && wide && !pair && a.ar_world <= 1 && (a.act == 1 || a.act == 2);
  if (a.ar_world > 1) {  // the fused all-reduce form (publisher warp)
    if (a.dtype == kBF16)
      return wide ? tc::launch<__nv_bfloat16, 256, 4, false, 8, true>(a, s)
                  : tc::launch<__nv_bfloat16, 128, 6, false, 8, true>(a, s);
    return wide ? tc::launch<__half, 256, 4, false, 8, true>(a, s) : tc::launch<__half, 128, 6, false, 8, true>(a, s);
  }
  if (a.dtype == kBF16) {
    if (pair) return tc::launch2<__nv_bfloat16, 6>(a, s);
    if (rt) return gelu12 ? tc::launch<__nv_bfloat16, 256, 3, true, 12>(a, s) : tc::launch<__nv_bfloat16, 256, 3, true>(a, s);
    if (gelu12) return tc::launch<__nv_bfloat16, 256, 3, false, 12>(a, s);
    return wide ? tc::launch<__nv_bfloat16, 256, 4>(a, s) : tc::launch<__nv_bfloat16, 128, 6>(a, s);
  }
  if (pair) return tc::launch2<__half, 6>(a, s);
  if (rt) return gelu12 ? tc::launch<__half, 256, 3, true, 12>(a, s) : tc::launch<__half, 256, 3, true>(a, s);
  if (gelu12) return tc::launch<__half, 256, 3, false, 12>(a, s);
  return wide ? tc::launch<__half, 256, 4>(a, s) : tc::launch<__half, 128, 6>(a, s);
}

// ---------------------------------------------------------------------------- weight gradient API
int wgrad_tcgen05_supported(const WgradArgs& a) {
  if (a.dtype != kBF16 && a.dtype != kF16) return 0;
  if (a.T <= 0 || a.M <= 0 || a.N <= 0 || !a.D[0] || a.ldd < a.N) return 0;
  const int64_t seg = a.seg_rows > 0 ? a.seg_rows : a.M;
  if ((a.M + seg - 1) / seg > 4) return 0;
  for (int i = 0; i < (int)((a.M + seg - 1) / seg); ++i)
    if (!a.D[i] || ((a.db[0] != nullptr) != (a.db[i] != nullptr))) return 0;
  if (a.ldy % 8 || a.ldx % 8 || a.ldy < a.M || a.ldx < a.N) return 0;  // 16-byte TMA strides
  if ((reinterpret_cast<uintptr_t>(a.dy) | reinterpret_cast<uintptr_t>(a.x)) & 15) return 0;
  return tc::get_encode() != nullptr;
}

WgradPlan wgrad_plan(int64_t M, int64_t N, int64_t T) {
  const int64_t tiles = ((M + tc::BM2 - 1) / tc::BM2) * ((N + tc::BN2 - 1) / tc::BN2);
  const int nkb = (int)((T + tc::BK - 1) / tc::BK);
  int pairs = tc::sm_count() / 2;
  {
    const size_t smem = sizeof(tc::SmemW<__nv_bfloat16>) + 1024;
    if (cudaFuncSetAttribute(tc::wgrad2_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.blockDim = dim3(tc::kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.gridDim = dim3(tc::sm_count() & ~1, 1, 1);
      pairs = tc::wgrad_pairs(&cfg);
    }
  }
  WgradPlan plan;
  plan.splits = 1;
  plan.k1 = 0;
  plan.pairs = pairs;
  // a schedule with partials must beat the plain one by 15%: the power cap lowers the clock when the
  // otherwise idle pairs join (measured at 4096 x 1024: no gain from the balanced schedule's 10%)
  int64_t best_cost = tc::wgrad_units_cost(tiles, 1, nkb, pairs) * 85 / 100;
  for (int sp = 2; sp <= 16; ++sp) {
    if (nkb / sp < 16) break;  // at least 16 k-blocks (1024 tokens) per split
    const int64_t c = tc::wgrad_units_cost(tiles, sp, nkb, pairs);
    if (c < best_cost) {
      best_cost = c;
      plan.splits = sp;
    }
  }
  for (int s2 = 1; s2 <= 8; ++s2) {
    int64_t c = 0;
    const int k1 = tc::wgrad_balanced(tiles, s2, nkb, pairs, &c);
    if (k1 > 0 && (nkb - k1) / s2 >= 8 && c < best_cost) {
      best_cost = c;
      plan.splits = s2;
      plan.k1 = k1;
    }
  }
  return plan;
}

int64_t wgrad_workspace_floats(int64_t M, int64_t N, const WgradPlan& plan) {
  const int splits = plan.splits;
  if (splits <= 1 && plan.k1 == 0) return 0;
  const int64_t m_pad = (M + tc::BM2 - 1) / tc::BM2 * tc::BM2, n_pad = (N + tc::BN2 - 1) / tc::BN2 * tc::BN2;
  return (int64_t)splits * m_pad * (n_pad + 1);
}

cudaError_t wgrad_tcgen05(const WgradArgs& a_in, const WgradPlan& plan, cudaStream_t s) {
  if (!wgrad_tcgen05_supported(a_in)) return cudaErrorInvalidValue;
  WgradArgs a = a_in;
  a.splits = plan.splits < 1 ? 1 : plan.splits;
  a.k1 = plan.k1;
  if ((a.splits > 1 || a.k1 > 0) && !a.ws) return cudaErrorInvalidValue;
  if (a.dtype == kBF16) return tc::launch_wgrad<__nv_bfloat16>(a, plan.pairs, s);
  return tc::launch_wgrad<__half>(a, plan.pairs, s);
}

}  // namespace nsw
