// Shifted-window attention on the 5th-generation tensor cores (tcgen05 + TMEM), forward and
// backward, specialised for head_dim 64 and windows of at most 176 tokens (T*wh*ww <= 176).
//
// Same contract and numerics as the mma.sync kernels in attention.cu (QK-RMSNorm, additive -100
// latitude-wrap mask, exp2-domain softmax, log2-domain LSE in window order for the backward).
// Both kernels are persistent (one CTA of 16 warps per SM walking (window, head) items, heads
// fastest) and bring a window's q/k/v rows in with TMA box loads of a 4-D [B*T, H, W, C] view of
// the token-major activations: one box per time step, split where the shifted window wraps at
// the grid edge, so shift, partition and reverse are never materialised.  S, P, O and the
// gradients live in TMEM; operands are 128-byte-swizzled shared-memory tiles (K-major, or
// MN-major where a transpose is needed).  Every mbarrier wait is bounded by a %globaltimer
// budget and records kErrWaitTimeout in the device error word on expiry.
// Reference behaviour: models/swin_helpers.py:27-70 (window_partition / window_reverse),
// :203-250 (WindowAttention.forward: QK norm, scaled_dot_product_attention with the mask) and
// :380-420 (the shifted block's roll and attn_mask).
#include <float.h>

#include "common.cuh"
#include <algorithm>
#include <cstring>
#include <cstdlib>

#include "kernels.h"

namespace nsw {
namespace attn_tc {

constexpr int HD = 64;
constexpr int ROW_B = HD * 2;        // 128 bytes per row (one swizzle row)
constexpr int MAXL = 176;            // keys padded to a multiple of 16, at most 176
constexpr float kLog2e = 1.4426950408889634f;
constexpr unsigned long long kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * ROW_B + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on the MMA-completion barrier; false on timeout (error recorded).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err) {
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
    if (spin == 0) t0 = gtimer();
    if ((spin & 255u) == 255u && gtimer() - t0 > kWaitBudgetNs) {
      record_error(err, kErrWaitTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint64_t desc_kmajor(const void* p) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major, 128-byte swizzle: K rows of 128 B (64 MN elements), 8-row atoms 1024 B apart
// (SBO); a single 64-wide MN block, so LBO is unused.
__device__ __forceinline__ uint64_t desc_mnmajor(const void* p) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, float* f) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void ld32(uint32_t taddr, float* f) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

struct WinPos {
  int b, wy, wx;
};

__device__ __forceinline__ int64_t token(const AttnGeom& g, const WinPos& p, int i) {
  const int wa = g.wh * g.ww;
  const int t = i / wa;
  const int r = i - t * wa;
  const int iy = r / g.ww, ix = r - iy * g.ww;
  int gy = (p.wy * g.wh + iy + g.sh) % g.H;
  int gx = (p.wx * g.ww + ix + g.sw) % g.W;
  if (gy < 0) gy += g.H;
  if (gx < 0) gx += g.W;
  return ((int64_t)(p.b * g.T + t) * g.H + gy) * g.W + gx;
}
__device__ __forceinline__ int label(const AttnGeom& g, const WinPos& p, int i) {
  if (!g.mask || g.mask_shift <= 0) return 0;
  const int iy = (i % (g.wh * g.ww)) / g.ww;
  return g.row_offset + p.wy * g.wh + iy >= g.h_global - g.mask_shift ? 1 : 0;
}

// ============================================================================ backward
// Persistent: one CTA (16 warps) per SM walks a contiguous range of (window, head) items, heads
// fastest, so the token table is rebuilt only when the window changes and the next item's rows
// are prefetched into L2 while the current item computes.  Warp w reads TMEM lanes 32*(w%4)..
// (its lane quarter) and column group w/4: four warps share every row and split its columns.
// Query tile 0 is rows [0,128); tile 1 is rows [NK-128, NK) with rows < 128 masked, so every
// row buffer holds NK <= 176 rows.  Key tile 1 starts at key 64 (a 64-key block boundary, as
// the MN-major operand needs) and only its keys >= 128 are used.  Per query tile t:
//   S   = Qhat_t Khat^T   -> TMEM R            (A, B K-major)
//   P   = exp2(S*scale*log2e + mask - lse)     bf16 into smem `ps` ([128 rows x 64 keys] SW128
//                                              blocks)
//   dP  = dO_t V^T       -> TMEM R            (A, B K-major)
//   dV += P^T dO_t       -> TMEM dV[kt]       (A = ps read MN-major, B = dO MN-major)
//   dS  = P * (dP - D) * scale                 written over P in `ps`
//   dK += dS^T Qhat_t    -> TMEM dK[kt]       (A = ps MN-major, B = Qhat MN-major)
//   dQ  = dS Khat        -> TMEM dQ           (A = ps K-major, B = Khat MN-major)
//   dQ epilogue: QK-RMSNorm backward from the raw q rows kept in smem; weight-gradient partial.
// After both tiles: dV and dK (with the k-norm backward) per key row.
// The same computation, on CUDA cores, is the mma.sync backward in attention.cu.
constexpr int DQ_COL = 192, DV_COL = 256, DK_COL = 384, BWD_TMEM_COLS = 512;
constexpr int PS_BLOCK = 128 * ROW_B;  // one 64-key block of the P/dS tile (16 KB)
constexpr int BWD_THREADS = 512;
constexpr int KT1 = 64;  // first key of key tile 1
constexpr int ROWBUF = MAXL * ROW_B;
static_assert(BWD_THREADS >= 2 * MAXL, "D is computed by two threads per row");

struct __align__(1024) SmemB {
  // q and k rows in two roles that swap every item: raw (gathered; read by the norm backward)
  // and normalized (MMA operand).  Once an item's last MMA has read its normalized rows, the
  // next item's raw rows are gathered into that buffer.
  unsigned char qbuf[2][ROWBUF];
  unsigned char kbuf[2][ROWBUF];
  unsigned char v[ROWBUF];
  unsigned char dO[ROWBUF];
  unsigned char ps[3 * PS_BLOCK];  // P, then dS, of the current query tile (keys < 192)
  int tok[2][MAXL];                // token rows of the current and the next window
  signed char lab[2][MAXL];
  float lse[MAXL];
  float rq[MAXL];
  float rk[MAXL];
  float red[4][128];  // per-column-group partial dot products of the norm backward
  float wq[16][HD];  // per-warp weight-gradient partials, summed over the CTA's items
  float wk[16][HD];
  float qwv[HD];    // norm weights
  float kwv[HD];
  uint64_t bar;     // MMA completion
  uint64_t bar_ld;  // TMA gather completion
  uint32_t tmem_base;
};

__device__ __forceinline__ uint64_t desc_mn(const void* p, uint32_t lbo_bytes) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// byte offset of (row, key) in the P/dS tile (16-byte chunk granularity)
__device__ __forceinline__ uint32_t ps_off(int row, int key) {
  return (uint32_t)((key >> 6) * PS_BLOCK) + swz(row, (key & 63) >> 3);
}

// TMA tile load of a [1 x wh x ww x 64] box (one time step of a window that does not wrap at
// the grid edge) from a 4-D view [B*T, H, W, cols]; lands in smem in window token order.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Only warp 0 polls an mbarrier; the other warps wait in the block barrier that follows, so
// 500 threads do not spin on shared memory while the tensor core reads its operands there.

// fp32 staging of a 128-row x 64-column tile in ps: 256-byte rows, 16-byte chunk q of row r at
// chunk position q ^ (r & 15), so 32 lanes writing one chunk of 32 rows hit distinct banks.
__device__ __forceinline__ uint32_t f32_off(int r, int q) { return (uint32_t)(r * 256 + ((q ^ (r & 15)) << 4)); }
__device__ __forceinline__ void stage_f32(unsigned char* st, int rt, int cg, const float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<float4*>(st + f32_off(rt, 4 * cg + q)) =
        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// QK-RMSNorm backward of one staged row, eight threads per row (columns [8c, 8c + 8) each):
// y = x * rs * w  =>  dx = rs*w*g - x * rs^3 * sum_j(w_j g_j x_j) / HD;  dw_j += g_j x_j rs.
// The row dot product is combined over the eight lanes by shuffles; dw partials accumulate in
// wacc.  Invalid rows still take part in the shuffles with zeros.
__device__ __forceinline__ void norm_bwd_task(const unsigned char* st, const unsigned char* xbuf, const float* wv,
                                              int row, int r, int c, bool valid, float rs, __nv_bfloat16* dst,
                                              float* wacc) {
  float gg[8], x[8], w[8];
  const float4 g0 = *reinterpret_cast<const float4*>(st + f32_off(row, 2 * c));
  const float4 g1 = *reinterpret_cast<const float4*>(st + f32_off(row, 2 * c + 1));
  gg[0] = g0.x; gg[1] = g0.y; gg[2] = g0.z; gg[3] = g0.w;
  gg[4] = g1.x; gg[5] = g1.y; gg[6] = g1.z; gg[7] = g1.w;
  unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(xbuf + swz(valid ? r : 0, c)), x);
  const float4 w0 = *reinterpret_cast<const float4*>(wv + 8 * c);
  const float4 w1 = *reinterpret_cast<const float4*>(wv + 8 * c + 4);
  w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w;
  w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) dot = fmaf(w[i] * gg[i], x[i], dot);
  if (!valid) dot = 0.f;
  dot += __shfl_xor_sync(0xffffffffu, dot, 1);
  dot += __shfl_xor_sync(0xffffffffu, dot, 2);
  dot += __shfl_xor_sync(0xffffffffu, dot, 4);
  if (!valid) return;
  const float k3 = rs * rs * rs * dot * (1.f / HD);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o[i] = rs * w[i] * gg[i] - x[i] * k3;
    wacc[i] = fmaf(gg[i] * x[i], rs, wacc[i]);
  }
  *reinterpret_cast<uint4*>(dst) = pack8<__nv_bfloat16>(o);
}

// Add the per-thread dw partials of columns [8c, 8c+8) (c = lane & 7) over the warp's four
// row groups, then into the warp's own slot (no atomics; slots are summed once per item).
__device__ __forceinline__ void flush_wacc(float* wacc, float* slot, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = wacc[i];
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    if (lane < 8) slot[8 * lane + i] += v;
  }
}

// Load 16*NCH consecutive TMEM columns of this warp's lane quarter (one wait for all).
template <int NCH>
__device__ __forceinline__ void ld_cols(uint32_t taddr, float* f);
template <>
__device__ __forceinline__ void ld_cols<1>(uint32_t taddr, float* f) {
  ld16(taddr, f);
}
template <>
__device__ __forceinline__ void ld_cols<2>(uint32_t taddr, float* f) {
  ld32(taddr, f);
}
// Two loads and one wait in one statement: the outputs are early-clobber, because the first load
// writes its registers asynchronously while the second still has to read its address operand;
// without it the compiler may give that operand a register the first load overwrites.
template <>
__device__ __forceinline__ void ld_cols<3>(uint32_t taddr, float* f) {
  uint32_t r[48];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%48];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47},"
      " [%49];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=&r"(r[0]), "=&r"(r[1]), "=&r"(r[2]), "=&r"(r[3]), "=&r"(r[4]), "=&r"(r[5]), "=&r"(r[6]), "=&r"(r[7]),
        "=&r"(r[8]), "=&r"(r[9]), "=&r"(r[10]), "=&r"(r[11]), "=&r"(r[12]), "=&r"(r[13]), "=&r"(r[14]), "=&r"(r[15]),
        "=&r"(r[16]), "=&r"(r[17]), "=&r"(r[18]), "=&r"(r[19]), "=&r"(r[20]), "=&r"(r[21]), "=&r"(r[22]), "=&r"(r[23]),
        "=&r"(r[24]), "=&r"(r[25]), "=&r"(r[26]), "=&r"(r[27]), "=&r"(r[28]), "=&r"(r[29]), "=&r"(r[30]), "=&r"(r[31]),
        "=&r"(r[32]), "=&r"(r[33]), "=&r"(r[34]), "=&r"(r[35]), "=&r"(r[36]), "=&r"(r[37]), "=&r"(r[38]), "=&r"(r[39]),
        "=&r"(r[40]), "=&r"(r[41]), "=&r"(r[42]), "=&r"(r[43]), "=&r"(r[44]), "=&r"(r[45]), "=&r"(r[46]), "=&r"(r[47])
      : "r"(taddr), "r"(taddr + 32)
      : "memory");
#pragma unroll
  for (int i = 0; i < 48; ++i) f[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// P = exp2(S * scale * log2e + mask - lse) for keys [16 c0, 16 (c0 + NCH)) of one row, packed
// to bf16 into `ps`.  Chunks fully inside [0, L) of a window with one mask label take the fast
// path (one FMA + one ex2 per element); others add the -100 mask of mismatched labels and
// give padding keys (label -1) P = 0.
template <int NCH>
__device__ __forceinline__ void p_chunks(uint32_t trow, SmemB& S, const signed char* lab, int rt, int c0, float lse_r,
                                         int lr, float sl2, float ml2, int mixed, int L) {
  float v[16 * NCH];
  ld_cols<NCH>(trow + 16 * c0, v);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int j = c0 + c;
    uint32_t pk[8];
    if (!mixed && 16 * j + 16 <= L) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        pk[i] = pack_bf16(ex2(fmaf(v[16 * c + 2 * i], sl2, -lse_r)), ex2(fmaf(v[16 * c + 2 * i + 1], sl2, -lse_r)));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float pr[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int lk = lab[16 * j + 2 * i + e];
          const float s = fmaf(v[16 * c + 2 * i + e], sl2, (lk != lr ? ml2 : 0.f) - lse_r);
          pr[e] = lk >= 0 ? ex2(s) : 0.f;
        }
        pk[i] = pack_bf16(pr[0], pr[1]);
      }
    }
    *reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    *reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j + 8)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

// dS = P * (dP - D) * scale = P * fma(dP, scale, -D*scale), written over P.
template <int NCH>
__device__ __forceinline__ void ds_chunks(uint32_t trow, SmemB& S, int rt, int c0, float scale, float Ds) {
  float v[16 * NCH];
  ld_cols<NCH>(trow + 16 * c0, v);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int j = c0 + c;
    uint4* p0 = reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j));
    uint4* p1 = reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j + 8));
    const uint4 a = *p0, b = *p1;
    const uint32_t pin[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pk[i] = pack_bf16(bf16_lo(pin[i]) * fmaf(v[16 * c + 2 * i], scale, -Ds),
                        bf16_hi(pin[i]) * fmaf(v[16 * c + 2 * i + 1], scale, -Ds));
    *p0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    *p1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

// Partial row sum of P * dP over keys [16 c0, 16 (c0 + NCH)) (D = rowsum(P dP) = rowsum(dO O)).
template <int NCH>
__device__ __forceinline__ float pdp_dot(uint32_t trow, const SmemB& S, int rt, int c0) {
  float v[16 * NCH];
  ld_cols<NCH>(trow + 16 * c0, v);
  float d = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int j = c0 + c;
    const uint4 a = *reinterpret_cast<const uint4*>(S.ps + ps_off(rt, 16 * j));
    const uint4 b = *reinterpret_cast<const uint4*>(S.ps + ps_off(rt, 16 * j + 8));
    const uint32_t pin[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
      d = fmaf(bf16_lo(pin[i]), v[16 * c + 2 * i], fmaf(bf16_hi(pin[i]), v[16 * c + 2 * i + 1], d));
  }
  return d;
}




// How a window's rows are brought in: up to 2 x 2 TMA boxes per time step, split where the
// shifted window wraps at the W (x) or H (y) edge of the token grid.  Boxes are issued y-part
// major, x-part minor, and each lands as [height][width] rows, so smem row j holds the window
// token win_row(j) (attention within a window does not depend on the row order; the token
// table, labels and lse follow the same permutation).
struct WinLoad {
  int x0, y0, bt0;
  int xw[2], yh[2];  // part widths / heights (second is 0 when that edge does not wrap)
};
__device__ __forceinline__ WinLoad win_load(const AttnGeom& g, int64_t w, int nww, int nwh) {
  WinLoad wl;
  const int wx = (int)(w % nww), wy = (int)((w / nww) % nwh), b = (int)(w / ((int64_t)nww * nwh));
  wl.x0 = (wx * g.ww + g.sw) % g.W;
  wl.y0 = (wy * g.wh + g.sh) % g.H;
  if (wl.x0 < 0) wl.x0 += g.W;
  if (wl.y0 < 0) wl.y0 += g.H;
  wl.bt0 = b * g.T;
  wl.xw[0] = min(g.ww, g.W - wl.x0);
  wl.xw[1] = g.ww - wl.xw[0];
  wl.yh[0] = min(g.wh, g.H - wl.y0);
  wl.yh[1] = g.wh - wl.yh[0];
  return wl;
}
// window-order index (t*wh + iy)*ww + ix of smem row j
__device__ __forceinline__ int win_row(const AttnGeom& g, const WinLoad& wl, int j) {
  const int wa = g.wh * g.ww;
  const int t = j / wa;
  int rem = j - t * wa;
  int iy0 = 0;
  for (int yp = 0; yp < 2; ++yp) {
    int ix0 = 0;
    for (int xp = 0; xp < 2; ++xp) {
      const int n = wl.xw[xp] * wl.yh[yp];
      if (rem < n) {
        const int yy = rem / wl.xw[xp], xx = rem - yy * wl.xw[xp];
        return (t * g.wh + iy0 + yy) * g.ww + ix0 + xx;
      }
      rem -= n;
      ix0 += wl.xw[xp];
    }
    iy0 += wl.yh[yp];
  }
  return j;  // not reached
}
// map index of a box: 3 x 3 grid over (width, height) in {full, first part, second part}
__device__ __forceinline__ int box_index(const WinLoad& wl, int xp, int yp) {
  const int xi = wl.xw[1] == 0 ? 0 : 1 + xp;
  const int yi = wl.yh[1] == 0 ? 0 : 1 + yp;
  return yi * 3 + xi;
}

struct BoxMaps {
  CUtensorMap m[9];
};

// One buffer of a window's rows (column `col`, 64 bf16 per token); L * 128 bytes.
__device__ __forceinline__ void load_window(unsigned char* buf, const BoxMaps& maps, uint64_t* bar, int col,
                                            const WinLoad& wl, const AttnGeom& g) {
  const int wa = g.wh * g.ww;
  for (int t = 0; t < g.T; ++t) {
    int row = t * wa;
    for (int yp = 0; yp < 2; ++yp) {
      if (wl.yh[yp] == 0) continue;
      for (int xp = 0; xp < 2; ++xp) {
        if (wl.xw[xp] == 0) continue;
        tma_load_4d(buf + row * ROW_B, &maps.m[box_index(wl, xp, yp)], bar, col, xp == 0 ? wl.x0 : 0,
                    yp == 0 ? wl.y0 : 0, wl.bt0 + t);
        row += wl.xw[xp] * wl.yh[yp];
      }
    }
  }
}

// Token rows and mask labels of window `w`; returns whether the window mixes labels.
__device__ __forceinline__ int build_table(const AttnGeom& g, int64_t w, int nww, int nwh, int L, int* tok,
                                           signed char* lab, int tid, short* wr = nullptr) {
  WinPos p;
  p.wx = (int)(w % nww);
  p.wy = (int)((w / nww) % nwh);
  p.b = (int)(w / ((int64_t)nww * nwh));
  const WinLoad wl = win_load(g, w, nww, nwh);
  const int lab0 = label(g, p, 0);
  int mx = 0;
  for (int j = tid; j < MAXL; j += BWD_THREADS) {
    const int i = j < L ? win_row(g, wl, j) : 0;
    if (wr) wr[j] = (short)i;
    tok[j] = j < L ? (int)token(g, p, i) : 0;
    const int lb = j < L ? label(g, p, i) : -1;
    lab[j] = (signed char)lb;
    mx |= (j < L && lb != lab0);
  }
  return __syncthreads_or(mx);
}

__global__ void __launch_bounds__(BWD_THREADS, 1)
    bwd_kernel(const __grid_constant__ BoxMaps box_qkv, const __grid_constant__ BoxMaps box_dout,
               const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
               const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
               __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqw_part, float* __restrict__ dkw_part,
               AttnGeom g, int* err, long long* __restrict__ stamps) {
  extern __shared__ unsigned char smem_raw[];
  SmemB& S = *reinterpret_cast<SmemB*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lg = warp & 3;   // TMEM lane quarter
  const int cg = warp >> 2;  // column group
  const int L = g.T * g.wh * g.ww;
  const int NK = (L + 15) & ~15;
  const int ntiles = (L + 127) / 128;
  const int nww = g.W / g.ww, nwh = g.H / g.wh;
  const int64_t C = (int64_t)g.nh * HD;
  const int64_t n_items = (int64_t)g.B * nwh * nww * g.nh;
  const int64_t i_begin = n_items * blockIdx.x / gridDim.x;
  const int64_t i_end = n_items * (blockIdx.x + 1) / gridDim.x;
  // optional phase timestamps (SM clock) of the third item of the first CTAs; null in production
  long long* st_base = (stamps && blockIdx.x < 64) ? stamps + 32 * blockIdx.x : nullptr;
  long long* st = nullptr;
  int nst = 0;
#define NSW_STAMP() \
  do {              \
    if (st && threadIdx.x == 0 && nst < 32) st[nst++] = clock64(); \
  } while (0)

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(BWD_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar_ld)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int pad_rows = max(NK, 128);
  // rows [L, max(NK,128)) of the operands and all of ps start as zeros; the window loads write
  // only rows < L, so the padding stays zero
  for (int idx = tid; idx < (pad_rows - L) * 8; idx += BWD_THREADS) {
    const int r = L + (idx >> 3), c = idx & 7;
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      *reinterpret_cast<uint4*>(S.qbuf[b2] + swz(r, c)) = z;
      *reinterpret_cast<uint4*>(S.kbuf[b2] + swz(r, c)) = z;
    }
    *reinterpret_cast<uint4*>(S.v + swz(r, c)) = z;
    *reinterpret_cast<uint4*>(S.dO + swz(r, c)) = z;
  }
  for (int idx = tid; idx < 3 * PS_BLOCK / 16; idx += BWD_THREADS)
    reinterpret_cast<uint4*>(S.ps)[idx] = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < 16 * HD; i += BWD_THREADS) {  // weight-gradient slots, summed over all items
    (&S.wq[0][0])[i] = 0.f;
    (&S.wk[0][0])[i] = 0.f;
  }
  if (tid < HD) {
    S.qwv[tid] = qw[tid];
    S.kwv[tid] = kw[tid];
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  const uint32_t trow = tmem + ((uint32_t)(lg * 32) << 16);
  const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NK >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  const uint32_t id_mn = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                         ((uint32_t)(128 >> 4) << 24);
  const uint32_t id_q = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                        ((uint32_t)(128 >> 4) << 24);
  const float sl2 = g.scale * kLog2e;
  const float ml2 = -100.f * kLog2e;
  const int rt = lg * 32 + lane;  // row within a 128-row tile
  uint32_t parity = 0, ld_parity = 0;
  bool ok = true;
  int raw = 0;   // index of the raw q/k buffers of the current item
  int tcur = 0;  // index of the current window's token table
  int64_t win = i_begin / g.nh;
  int mixed = 0;
  bool ld_pending = false;  // a gather phase was issued and not yet waited for
  float lse_next = 0.f;     // lse of row tid of the next item, loaded a phase ahead
  if (i_begin < i_end) {
    ld_pending = true;
    // first item: its table and all four gathers
    mixed = build_table(g, win, nww, nwh, L, S.tok[0], S.lab[0], tid);
    const WinLoad wl = win_load(g, win, nww, nwh);
    if (tid == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.bar_ld)),
                   "r"(4 * L * ROW_B)
                   : "memory");
    __syncthreads();
    if (lane == 0 && warp < 4) {
      const int h0 = (int)(i_begin - win * g.nh);
      unsigned char* buf = warp == 0 ? S.qbuf[0] : warp == 1 ? S.kbuf[0] : warp == 2 ? S.v : S.dO;
      load_window(buf, warp < 3 ? box_qkv : box_dout, &S.bar_ld, (warp < 3 ? warp * (int)C : 0) + h0 * HD, wl, g);
    }
  }

  for (int64_t item = i_begin; item < i_end && ok; ++item) {
    st = (st_base && item == i_begin + 2) ? st_base : nullptr;
    NSW_STAMP();
    const int h = (int)(item - win * g.nh);
    const bool has_next = item + 1 < i_end;
    const int64_t nwin = (item + 1) / g.nh;
    const int nh_ = (int)(item + 1 - nwin * g.nh);
    const int ntab = nwin == win ? tcur : 1 - tcur;
    int mixed_n = mixed;
    const int* tok = S.tok[tcur];
    const signed char* lab = S.lab[tcur];
    unsigned char* qx = S.qbuf[raw];       // raw q
    unsigned char* qn = S.qbuf[1 - raw];   // normalized q
    unsigned char* kx = S.kbuf[raw];
    unsigned char* kn = S.kbuf[1 - raw];
    // lse rows of this item (items are (window, head) in the forward's lse order; smem row j
    // holds window token win_row(j)); loaded during the previous item except for the first
    if (item == i_begin && tid < L) lse_next = lse[item * L + win_row(g, win_load(g, win, nww, nwh), tid)];
    if (tid < L) S.lse[tid] = lse_next;
    NSW_STAMP();
    ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar_ld, ld_parity, err) : true);
    ld_parity ^= 1;
    ld_pending = false;
    if (!ok) break;
    NSW_STAMP();
    // QK-RMSNorm of the raw rows into the MMA operands (rstd kept for the backward); two
    // threads per row, each with four of its eight 16-byte chunks
    for (int base = 0; base < 4 * L; base += BWD_THREADS) {
      const int idx = base + tid;
      const bool act = idx < 4 * L;
      const int rr = act ? idx >> 1 : 0, half = idx & 1;
      const bool isq = rr < L;
      const int r = isq ? rr : rr - L;
      const unsigned char* src = isq ? qx : kx;
      unsigned char* dst = isq ? qn : kn;
      const float* w = isq ? S.qwv : S.kwv;
      float f[4][8];
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(src + swz(r, 4 * half + c)), f[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[c][i] * f[c][i];
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rs = rsqrtf(ss / (float)HD + FLT_EPSILON);
      if (act) {
        if (half == 0) {
          if (isq) S.rq[r] = rs;
          else S.rk[r] = rs;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 8; ++i) f[c][i] *= rs * w[(4 * half + c) * 8 + i];
          *reinterpret_cast<uint4*>(dst + swz(r, 4 * half + c)) = pack8<__nv_bfloat16>(f[c]);
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    fence_before();
    __syncthreads();
    fence_after();
    NSW_STAMP();

    for (int t = 0; t < ntiles; ++t) {
      const int qb = t == 0 ? 0 : NK - 128;  // first row of the tile
      const int lo = t * 128;                 // rows below lo belong to tile 0
      const int r = qb + rt;
      const bool rvalid = r >= lo && r < L;
      const bool warp_live = qb + lg * 32 + 31 >= lo && qb + lg * 32 < L;  // warp-uniform
      // ---- S (tile 0 here; later tiles are issued before the previous tile's dQ epilogue)
      if (t == 0 && tid == 0) {
        fence_after();
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_ss(tmem, desc_kmajor(qn + ks * 32), desc_kmajor(kn + ks * 32), id_s, ks > 0);
        commit(&S.bar);
      }
      __syncwarp();
      ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar, parity, err) : true);
      parity ^= 1;
      if (!ok) break;
      NSW_STAMP();
      fence_after();
      // ---- P -> ps.  Column group cg owns keys [48 cg, 48 cg + 48) (three 16-key chunks);
      // rows outside the tile's range get lse = +inf and so P = 0 without a branch.
      {
        const int c0 = 3 * cg, nch = max(0, min(3, NK / 16 - c0));
        if (warp_live) {
          const float lse_r = rvalid ? S.lse[r] : INFINITY;
          const int lr = rvalid ? lab[r] : 0;
          if (nch == 3) p_chunks<3>(trow, S, lab, rt, c0, lse_r, lr, sl2, ml2, mixed, L);
          else if (nch == 2) p_chunks<2>(trow, S, lab, rt, c0, lse_r, lr, sl2, ml2, mixed, L);
          else if (nch == 1) p_chunks<1>(trow, S, lab, rt, c0, lse_r, lr, sl2, ml2, mixed, L);
        } else {
          for (int j = c0; j < c0 + nch; ++j) {
            *reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j)) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(S.ps + ps_off(rt, 16 * j + 8)) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncthreads();
      NSW_STAMP();
      // ---- dP = dO V^T; dV += P^T dO
      if (tid == 0) {
        fence_after();
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_ss(tmem, desc_kmajor(S.dO + qb * ROW_B + ks * 32), desc_kmajor(S.v + ks * 32), id_s, ks > 0);
        NSW_STAMP();
        for (int kt = 0; kt < ntiles; ++kt)
          for (int ks = 0; ks < 8; ++ks)
            mma_ss(tmem + DV_COL + 64 * kt, desc_mn(S.ps + kt * PS_BLOCK + ks * 2048, PS_BLOCK),
                   desc_mn(S.dO + qb * ROW_B + ks * 2048, 16), id_mn, (t > 0 || ks > 0));
        commit(&S.bar);
      }
      NSW_STAMP();
      __syncwarp();
      ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar, parity, err) : true);
      parity ^= 1;
      if (!ok) break;
      NSW_STAMP();
      fence_after();
      // v and dO are free once the last tile's dP/dV MMAs are done: gather the next item's
      if (t == ntiles - 1 && has_next) {
        if (nwin != win) mixed_n = build_table(g, nwin, nww, nwh, L, S.tok[ntab], S.lab[ntab], tid);
        if (tid == 0)
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.bar_ld)),
                       "r"(4 * L * ROW_B)
                       : "memory");
        ld_pending = true;
        __syncthreads();
        if (lane == 0 && (warp == 2 || warp == 3))
          load_window(warp == 2 ? S.v : S.dO, warp == 2 ? box_qkv : box_dout, &S.bar_ld,
                      (warp == 2 ? 2 * (int)C : 0) + nh_ * HD, win_load(g, nwin, nww, nwh), g);
        if (tid < L) lse_next = __ldg(lse + (item + 1) * L + win_row(g, win_load(g, nwin, nww, nwh), tid));
      }
      // ---- D = rowsum(P dP) (four column groups combined through smem), then
      // dS = P (dP - D) scale over P (rows of dead warps stay zero)
      {
        const int c0 = 3 * cg, nch = max(0, min(3, NK / 16 - c0));
        float part = 0.f;
        if (warp_live) {
          if (nch == 3) part = pdp_dot<3>(trow, S, rt, c0);
          else if (nch == 2) part = pdp_dot<2>(trow, S, rt, c0);
          else if (nch == 1) part = pdp_dot<1>(trow, S, rt, c0);
        }
        S.red[cg][rt] = part;
        __syncthreads();
        if (warp_live) {
          const float Ds = (S.red[0][rt] + S.red[1][rt] + S.red[2][rt] + S.red[3][rt]) * g.scale;
          if (nch == 3) ds_chunks<3>(trow, S, rt, c0, g.scale, Ds);
          else if (nch == 2) ds_chunks<2>(trow, S, rt, c0, g.scale, Ds);
          else if (nch == 1) ds_chunks<1>(trow, S, rt, c0, g.scale, Ds);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncthreads();
      NSW_STAMP();
      // ---- dK += dS^T Qhat; dQ = dS Khat
      if (tid == 0) {
        fence_after();
        for (int kt = 0; kt < ntiles; ++kt)
          for (int ks = 0; ks < 8; ++ks)
            mma_ss(tmem + DK_COL + 64 * kt, desc_mn(S.ps + kt * PS_BLOCK + ks * 2048, PS_BLOCK),
                   desc_mn(qn + qb * ROW_B + ks * 2048, 16), id_mn, (t > 0 || ks > 0));
        for (int ks = 0; ks < NK / 16; ++ks)
          mma_ss(tmem + DQ_COL, desc_kmajor(S.ps + (ks >> 2) * PS_BLOCK + (ks & 3) * 32),
                 desc_mn(kn + ks * 2048, 16), id_q, ks > 0);
        commit(&S.bar);
      }
      __syncwarp();
      ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar, parity, err) : true);
      parity ^= 1;
      if (!ok) break;
      NSW_STAMP();
      fence_after();
      // S of the next tile overlaps this tile's dQ epilogue (R is free: dP was consumed by dS)
      if (t + 1 < ntiles && tid == 0) {
        fence_after();
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_ss(tmem, desc_kmajor(qn + (NK - 128) * ROW_B + ks * 32), desc_kmajor(kn + ks * 32), id_s, ks > 0);
        commit(&S.bar);
      }
      // the normalized q/k rows are free once the last tile's dK/dQ MMAs are done: gather the
      // next item's raw rows into them
      if (t == ntiles - 1 && has_next && lane == 0 && warp < 2)
        load_window(warp == 0 ? qn : kn, box_qkv, &S.bar_ld, (warp == 0 ? 0 : (int)C) + nh_ * HD,
                    win_load(g, nwin, nww, nwh), g);
      // ---- dQ epilogue: TMEM -> fp32 staging in ps, then the QK-norm backward of q with eight
      // threads per row and coalesced row stores
      {
        if (warp_live) {
          float gq[16];
          ld16(trow + DQ_COL + 16 * cg, gq);
          stage_f32(S.ps, rt, cg, gq);
        }
        __syncthreads();
        NSW_STAMP();
        float wacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int c = tid & 7;
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const int row = (tid >> 3) + 64 * k2;
          const int rr = qb + row;
          const bool valid = rr >= lo && rr < L;
          __nv_bfloat16* dst = dqkv + (valid ? (int64_t)tok[rr] * g.qkv_stride : 0) + (int64_t)h * HD + 8 * c;
          norm_bwd_task(S.ps, qx, S.qwv, row, rr, c, valid, valid ? S.rq[rr] : 0.f, dst, wacc);
        }
        NSW_STAMP();
        flush_wacc(wacc, S.wq[warp], lane);
      }
      fence_before();
      __syncthreads();  // R, dQ, red and ps are reused by the next tile
      NSW_STAMP();
    }
    if (!ok) break;
    if (!ok) break;
    // ---- dV, dK epilogues (key rows): dV through bf16 staging, dK through fp32 staging and the
    // QK-norm backward of k, eight threads per row, coalesced row stores
    for (int kt = 0; kt < ntiles; ++kt) {
      const int kb = kt == 0 ? 0 : KT1;
      const int lo = kt * 128;
      const bool live = kb + lg * 32 + 31 >= lo && kb + lg * 32 < L;  // warp-uniform
      unsigned char* st_v = S.ps + 2 * PS_BLOCK;
      if (live) {
        float gv[16];
        ld16(trow + DV_COL + 64 * kt + 16 * cg, gv);
        *reinterpret_cast<uint4*>(st_v + swz(rt, 2 * cg)) = pack8<__nv_bfloat16>(gv);
        *reinterpret_cast<uint4*>(st_v + swz(rt, 2 * cg + 1)) = pack8<__nv_bfloat16>(gv + 8);
        float gk[16];
        ld16(trow + DK_COL + 64 * kt + 16 * cg, gk);
        stage_f32(S.ps, rt, cg, gk);
      }
      __syncthreads();
      NSW_STAMP();
      float wacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int c = tid & 7;
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int row = (tid >> 3) + 64 * k2;
        const int kr = kb + row;
        const bool valid = kr >= lo && kr < L;
        const int64_t base_off = (valid ? (int64_t)tok[kr] * g.qkv_stride : 0) + (int64_t)h * HD + 8 * c;
        if (valid)
          *reinterpret_cast<uint4*>(dqkv + base_off + 2 * C) = *reinterpret_cast<const uint4*>(st_v + swz(row, c));
        norm_bwd_task(S.ps, kx, S.kwv, row, kr, c, valid, valid ? S.rk[kr] : 0.f, dqkv + base_off + C, wacc);
      }
      NSW_STAMP();
      flush_wacc(wacc, S.wk[warp], lane);
      __syncthreads();  // the staging area is rewritten by the next key tile
      NSW_STAMP();
    }
    fence_before();
    __syncthreads();  // TMEM and staging are reused by the next item
    raw = 1 - raw;
    tcur = ntab;
    win = nwin;
    mixed = mixed_n;
  }
#undef NSW_STAMP
  // after an error, let gathers still in flight land before the shared memory is released
  // (bounded; a second timeout is not recorded again)
  if (!ok && ld_pending && tid == 0) wait_bar(&S.bar_ld, ld_parity, nullptr);
  fence_before();
  __syncthreads();
  fence_after();
  // this CTA's QK-norm weight-gradient partial: the warps' slots, summed over all its items
  if (tid < 2 * HD) {
    const int col = tid & (HD - 1);
    float acc = 0.f;
    if (tid < HD) {
#pragma unroll
      for (int w = 0; w < 16; ++w) acc += S.wq[w][col];
      dqw_part[(int64_t)blockIdx.x * HD + col] = acc;
    } else {
#pragma unroll
      for (int w = 0; w < 16; ++w) acc += S.wk[w][col];
      dkw_part[(int64_t)blockIdx.x * HD + col] = acc;
    }
  }
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BWD_TMEM_COLS));
}

// ============================================================================ forward
// Persistent: one CTA (16 warps) per SM walks a contiguous range of (window, head) items, heads
// fastest (the backward's order).  The q, k and v rows of item i+1 arrive by TMA box loads into
// the second buffer set while item i computes.  Warp w reads TMEM lanes 32*(w%4).. and column
// group w/4, as in the backward.  Query tile 0 is rows [0,128), tile 1 rows [NK-128, NK) (its
// rows < 128 are computed again and not stored).  Per item:
//   QK-RMSNorm of the q and k rows in place (two threads per row)
//   S_t = Qhat_t Khat^T     both tiles issued at once -> TMEM s_col(t) (K-major operands)
//   softmax of tile t       row max and row sum combined over the four column groups through
//                           shared memory; P = exp2(S*scale*log2e + mask - max) packed to bf16
//                           into `ps` (K-major 128-byte-swizzled blocks of 64 keys)
//   O_t = P_t V             A = P K-major, B = V MN-major -> TMEM o_col(t); tile 0's O product
//                           runs during tile 1's softmax (P_1 is written once it has finished)
//   epilogue                O/rowsum to bf16 rows in shared memory, then whole 128-byte rows to
//                           each token's position; lse = max + log2(sum) in window order
constexpr int FWD_THREADS = 512;
constexpr int FWD_TMEM_COLS = 512;
// TMEM columns: S_0 [0, 176), O_0 [192, 256), S_1 [256, 432), O_1 [448, 512).
__device__ __forceinline__ uint32_t s_col(int t) { return t == 0 ? 0u : 256u; }
__device__ __forceinline__ uint32_t o_col(int t) { return t == 0 ? 192u : 448u; }

struct __align__(1024) SmemF {
  unsigned char q[2][ROWBUF];  // item-parity buffer sets; K-major SW128 rows, normalized in place
  unsigned char k[2][ROWBUF];
  unsigned char v[2][ROWBUF];  // MN-major B operand of O = P V (the same SW128 rows)
  unsigned char ps[3 * PS_BLOCK];  // P of the current query tile, [128 rows x 64 keys] SW128 blocks
  unsigned char stg[128 * ROW_B];   // bf16 O rows of one query tile
  int tok[2][MAXL];
  short wr[2][MAXL];  // window-order index of smem row j (the lse layout)
  signed char lab[2][MAXL];
  float red[2][4][128];  // per-column-group row max / row sum
  float qwv[HD];
  float kwv[HD];
  uint64_t bar_s[2];  // S of query tile 0 / 1 complete
  uint64_t bar_o[2];  // O of query tile 0 / 1 complete
  uint64_t bar_ld;    // an item's q/k/v rows landed
  uint32_t tmem_base;
};

// Scaled, masked logits (log2 domain; padding keys -inf) of this warp's 48 keys [16 c0, 16 c0 + 48)
// of one row, read from TMEM.  Keys at or beyond NK (the last group reads past the S columns into
// unused TMEM) are -inf without a label lookup.
__device__ __forceinline__ void logits(uint32_t taddr, const signed char* lab, int c0, int lr, float sl2, float ml2,
                                       int mixed, int L, int NK, float* sv) {
  ld_cols<3>(taddr + 16 * c0, sv);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const int j = c0 + c;
    if (16 * j >= NK) {
#pragma unroll
      for (int i = 0; i < 16; ++i) sv[16 * c + i] = -INFINITY;
    } else if (!mixed && 16 * j + 16 <= L) {
#pragma unroll
      for (int i = 0; i < 16; ++i) sv[16 * c + i] *= sl2;
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int lk = lab[16 * j + i];
        sv[16 * c + i] = lk < 0 ? -INFINITY : fmaf(sv[16 * c + i], sl2, lk != lr ? ml2 : 0.f);
      }
    }
  }
}

__device__ __forceinline__ float row_max(uint32_t taddr, const signed char* lab, int c0, int lr, float sl2, float ml2,
                                         int mixed, int L, int NK) {
  float sv[48];
  logits(taddr, lab, c0, lr, sl2, ml2, mixed, L, NK, sv);
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 48; ++i) m = fmaxf(m, sv[i]);
  return m;
}

// P = exp2(s - m) of the same keys (logits read again from TMEM rather than kept in registers
// across the block barrier), packed to bf16 pairs in pk; returns their fp32 sum.
__device__ __forceinline__ float probs(uint32_t taddr, const signed char* lab, int c0, int lr, float sl2, float ml2,
                                       int mixed, int L, int NK, float m, uint32_t* pk) {
  float sv[48];
  logits(taddr, lab, c0, lr, sl2, ml2, mixed, L, NK, sv);
  float l = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float p0 = ex2(sv[2 * i] - m), p1 = ex2(sv[2 * i + 1] - m);
    l += p0 + p1;
    pk[i] = pack_bf16(p0, p1);
  }
  return l;
}

// This row's P for keys [16 c0, 16 c0 + 48) into the K-major P tile (192 keys wide).
__device__ __forceinline__ void store_p(unsigned char* ps, int rt, int c0, const uint32_t* pk) {
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const int key = 16 * (c0 + c);
    *reinterpret_cast<uint4*>(ps + ps_off(rt, key)) = make_uint4(pk[8 * c], pk[8 * c + 1], pk[8 * c + 2], pk[8 * c + 3]);
    *reinterpret_cast<uint4*>(ps + ps_off(rt, key + 8)) =
        make_uint4(pk[8 * c + 4], pk[8 * c + 5], pk[8 * c + 6], pk[8 * c + 7]);
  }
}

__global__ void __launch_bounds__(FWD_THREADS, 1)
    fwd_kernel(const __grid_constant__ BoxMaps box_qkv, const float* __restrict__ qw, const float* __restrict__ kw,
               __nv_bfloat16* __restrict__ out, float* __restrict__ lse, AttnGeom g, int* err) {
  extern __shared__ unsigned char smem_raw[];
  SmemF& S = *reinterpret_cast<SmemF*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lg = warp & 3;   // TMEM lane quarter
  const int cg = warp >> 2;  // column group: keys [48 cg, 48 cg + 48), O columns [16 cg, 16 cg + 16)
  const int L = g.T * g.wh * g.ww;
  const int NK = (L + 15) & ~15;
  const int ntiles = (L + 127) / 128;
  const int nww = g.W / g.ww, nwh = g.H / g.wh;
  const int C = g.nh * HD;
  const int64_t n_items = (int64_t)g.B * nwh * nww * g.nh;
  const int64_t i_begin = n_items * blockIdx.x / gridDim.x;
  const int64_t i_end = n_items * (blockIdx.x + 1) / gridDim.x;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(FWD_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar_s[t])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar_o[t])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar_ld)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // rows [L, max(NK,128)) of every operand buffer stay zero (the loads write rows < L only)
  const int pad_rows = max(NK, 128);
  for (int idx = tid; idx < (pad_rows - L) * 8; idx += FWD_THREADS) {
    const int r = L + (idx >> 3), c = idx & 7;
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      *reinterpret_cast<uint4*>(S.q[b2] + swz(r, c)) = z;
      *reinterpret_cast<uint4*>(S.k[b2] + swz(r, c)) = z;
      *reinterpret_cast<uint4*>(S.v[b2] + swz(r, c)) = z;
    }
  }
  // rows of the P tile that no warp writes (padding rows) stay finite
  for (int idx = tid; idx < 3 * PS_BLOCK / 16; idx += FWD_THREADS)
    reinterpret_cast<uint4*>(S.ps)[idx] = make_uint4(0, 0, 0, 0);
  if (tid < HD) {
    S.qwv[tid] = qw[tid];
    S.kwv[tid] = kw[tid];
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  const uint32_t trow = tmem + ((uint32_t)(lg * 32) << 16);
  const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NK >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                        ((uint32_t)(128 >> 4) << 24);
  const float sl2 = g.scale * kLog2e;
  const float ml2 = -100.f * kLog2e;
  const int rt = lg * 32 + lane;  // row within a 128-row tile
  const int c0 = 3 * cg;
  uint32_t ph = 0, ld_parity = 0;
  bool ok = true;
  bool ld_pending = false;
  int tcur = 0;
  int64_t win = i_begin / g.nh;
  int mixed = 0;
  if (i_begin < i_end) {
    mixed = build_table(g, win, nww, nwh, L, S.tok[0], S.lab[0], tid, S.wr[0]);
    if (tid == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.bar_ld)),
                   "r"(3 * L * ROW_B)
                   : "memory");
    __syncthreads();
    ld_pending = true;
    if (lane == 0 && warp < 3) {
      const int h0 = (int)(i_begin - win * g.nh);
      unsigned char* buf = warp == 0 ? S.q[0] : warp == 1 ? S.k[0] : S.v[0];
      load_window(buf, box_qkv, &S.bar_ld, warp * C + h0 * HD, win_load(g, win, nww, nwh), g);
    }
  }

  int b = 0;  // buffer set of the current item
  for (int64_t item = i_begin; item < i_end && ok; ++item) {
    const int h = (int)(item - win * g.nh);
    const bool has_next = item + 1 < i_end;
    const int64_t nwin = (item + 1) / g.nh;
    const int ntab = nwin == win ? tcur : 1 - tcur;
    int mixed_n = mixed;
    const int* tok = S.tok[tcur];
    const short* wr = S.wr[tcur];
    const signed char* lab = S.lab[tcur];
    unsigned char* qb_ = S.q[b];
    unsigned char* kb_ = S.k[b];
    ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar_ld, ld_parity, err) : true);
    ld_parity ^= 1;
    ld_pending = false;
    if (!ok) break;
    // the next item's table and rows: its buffer set was last read by this CTA's previous
    // item, whose MMAs have all completed
    if (has_next) {
      if (nwin != win) mixed_n = build_table(g, nwin, nww, nwh, L, S.tok[ntab], S.lab[ntab], tid, S.wr[ntab]);
      if (tid == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.bar_ld)),
                     "r"(3 * L * ROW_B)
                     : "memory");
      __syncthreads();
      ld_pending = true;
      if (lane == 0 && warp < 3) {
        const int nh_ = (int)(item + 1 - nwin * g.nh);
        unsigned char* buf = warp == 0 ? S.q[1 - b] : warp == 1 ? S.k[1 - b] : S.v[1 - b];
        load_window(buf, box_qkv, &S.bar_ld, warp * C + nh_ * HD, win_load(g, nwin, nww, nwh), g);
      }
    }
    // QK-RMSNorm in place, two threads per row (four 16-byte chunks each)
    for (int base = 0; base < 4 * L; base += FWD_THREADS) {
      const int idx = base + tid;
      const bool act = idx < 4 * L;
      const int rr = act ? idx >> 1 : 0, half = idx & 1;
      const bool isq = rr < L;
      const int r = isq ? rr : rr - L;
      unsigned char* row = isq ? qb_ : kb_;
      const float* w = isq ? S.qwv : S.kwv;
      float f[4][8];
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(row + swz(r, 4 * half + c)), f[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[c][i] * f[c][i];
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rs = rsqrtf(ss / (float)HD + FLT_EPSILON);
      if (act) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 8; ++i) f[c][i] *= rs * w[(4 * half + c) * 8 + i];
          *reinterpret_cast<uint4*>(row + swz(r, 4 * half + c)) = pack8<__nv_bfloat16>(f[c]);
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      for (int t = 0; t < ntiles; ++t) {
        const int qrow = t == 0 ? 0 : NK - 128;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_ss(tmem + s_col(t), desc_kmajor(qb_ + qrow * ROW_B + ks * 32), desc_kmajor(kb_ + ks * 32), id_s,
                 ks > 0);
        commit(&S.bar_s[t]);
      }
    }
    __syncwarp();
    float m_t[2] = {0.f, 0.f}, l_t[2] = {1.f, 1.f};
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t >= ntiles) break;
      const int qrow = t == 0 ? 0 : NK - 128;
      const int lo = t * 128;
      const int r = qrow + rt;
      const int lr = r < L ? lab[r] : 0;
      // warps whose rows are all padding, or all recomputed rows of tile 1, skip the softmax:
      // each O row depends on its own P row only, and those rows are not stored
      const bool warp_live = qrow + lg * 32 + 31 >= lo && qrow + lg * 32 < L;  // warp-uniform
      ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar_s[t], ph, err) : true);
      if (!ok) break;
      fence_after();
      uint32_t pk[24];
      float mx = -INFINITY;
      const uint32_t ts = trow + s_col(t);
      if (warp_live && c0 * 16 < NK) mx = row_max(ts, lab, c0, lr, sl2, ml2, mixed, L, NK);
      S.red[0][cg][rt] = mx;
      __syncthreads();
      const float m = fmaxf(fmaxf(S.red[0][0][rt], S.red[0][1][rt]), fmaxf(S.red[0][2][rt], S.red[0][3][rt]));
      float ls = 0.f;
      if (warp_live && c0 * 16 < NK) ls = probs(ts, lab, c0, lr, sl2, ml2, mixed, L, NK, m, pk);
      S.red[1][cg][rt] = ls;
      // the P tile is free once the previous tile's O product has read it
      ok = __syncthreads_and((warp == 0 && t > 0) ? wait_bar(&S.bar_o[0], ph, err) : true);
      if (!ok) break;
      m_t[t] = m;
      l_t[t] = S.red[1][0][rt] + S.red[1][1][rt] + S.red[1][2][rt] + S.red[1][3][rt];
      if (warp_live && c0 * 16 < NK) store_p(S.ps, rt, c0, pk);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncthreads();
      if (tid == 0) {
        fence_after();
        for (int ks = 0; ks < NK / 16; ++ks)
          mma_ss(tmem + o_col(t), desc_kmajor(S.ps + (ks >> 2) * PS_BLOCK + (ks & 3) * 32),
                 desc_mnmajor(S.v[b] + ks * 16 * ROW_B), id_o, ks > 0);
        commit(&S.bar_o[t]);
      }
      __syncwarp();
    }
    if (!ok) break;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t >= ntiles) break;
      const int qrow = t == 0 ? 0 : NK - 128;
      const int lo = t * 128;
      const int r = qrow + rt;
      const bool warp_live = qrow + lg * 32 + 31 >= lo && qrow + lg * 32 < L;  // warp-uniform
      ok = __syncthreads_and(warp == 0 ? wait_bar(&S.bar_o[t], ph, err) : true);
      if (!ok) break;
      fence_after();
      unsigned char* st = S.stg;  // reused by tile 1 after the barrier above
      if (warp_live) {
        float o[16];
        ld16(trow + o_col(t) + 16 * cg, o);
        const float il = 1.f / l_t[t];
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= il;
        *reinterpret_cast<uint4*>(st + swz(rt, 2 * cg)) = pack8<__nv_bfloat16>(o);
        *reinterpret_cast<uint4*>(st + swz(rt, 2 * cg + 1)) = pack8<__nv_bfloat16>(o + 8);
        if (cg == 0 && r >= lo && r < L) lse[item * L + wr[r]] = m_t[t] + __log2f(l_t[t]);
      }
      __syncthreads();
      const int c = tid & 7;
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int row = (tid >> 3) + 64 * k2;
        const int rr = qrow + row;
        if (rr >= lo && rr < L)
          *reinterpret_cast<uint4*>(out + (int64_t)tok[rr] * g.out_stride + (int64_t)h * HD + 8 * c) =
              *reinterpret_cast<const uint4*>(st + swz(row, c));
      }
    }
    if (!ok) break;
    ph ^= 1;
    b ^= 1;
    tcur = ntab;
    win = nwin;
    mixed = mixed_n;
    fence_before();
    __syncthreads();  // S, O and the staging rows are rewritten by the next item
    fence_after();
  }
  // after an error, let loads still in flight land before the shared memory is released
  // (bounded; a second timeout is not recorded again)
  if (!ok && ld_pending && tid == 0) wait_bar(&S.bar_ld, ld_parity, nullptr);
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FWD_TMEM_COLS));
}

// ============================================================================ forward, warp-specialised
// Persistent, one CTA of 16 warps per SM walking a contiguous range of (window, head) items, heads
// fastest.  Unlike the kernel above (every warp takes every phase of one item, separated by block
// barriers), each role runs its own loop and the roles hand work to one another through mbarriers,
// so the elementwise work of one item overlaps the loads, the normalisation and the MMAs of others:
//   warp 0        producer: the window's tables (token row, window-order index, mask label and the
//                 per-key additive bias of every smem row) and TMA box loads of an item's q, k and v
//                 rows into stage (n % 3) of a three-stage ring;
//   warps 1, 2    MMA issuers (one elected lane each), one per softmax warpgroup:
//                 S_t = Qhat_t Khat^T (A, B K-major smem) and O_t = P_t V (A = P read from TMEM,
//                 B = V as an MN-major smem operand);
//   warps 4-7     QK-RMSNorm of a landed stage's q and k rows in place (one thread per row), and
//                 the norms of the normalised rows (a bound on the logits, below);
//   warps 8-11,   softmax + epilogue warpgroups; warpgroup w takes the items with (n & 1) == w and
//   12-15         owns TMEM columns [256 w, 256 w + 256): S at [0, 176) with P written back as
//                 packed bf16 pairs over its front (tcgen05.st), O at [192, 256).
// Each thread owns one query row (its TMEM lane), so the row max and row sum need no cross-warp
// reduction.  The max is replaced by the Cauchy-Schwarz bound sl2 * |qhat_i| * max_j |khat_j| when
// that bound is at most 48 (log2 units; P then stays a normal number), which skips one pass over S:
// softmax and lse do not depend on the shift used, only its overflow safety does.  Query tile 0 is
// rows [0, 128), tile 1 rows [NK - 128, NK), of which rows >= 128 are computed and stored.  O rows
// go from registers to their tokens' positions (whole 128-byte rows, 16-byte stores); lse (log2
// domain, window order) per row.  Every mbarrier wait is bounded and raises a CTA abort flag on
// expiry (kErrWaitTimeout in the device error word); all roles then leave their loops, wait
// (bounded) for their own TMA loads and MMAs, and the TMEM is freed.
constexpr int WS_THREADS = 512;
constexpr int WS_TMEM_COLS = 512;
constexpr int WS_STAGES = 3;
constexpr uint32_t WS_O_COL = 192;
constexpr float WS_MAX_BOUND = 48.f;
// wait budget in SM cycles (the SM clock, read without the latency of %globaltimer): 4e9 cycles
// are 2 to 3 s between the power-capped and the maximum clock
constexpr unsigned long long kWaitBudgetCycles = 4000000000ull;

struct __align__(1024) SmemWS {
  unsigned char q[WS_STAGES][ROWBUF];  // K-major SW128 rows, normalised in place
  unsigned char k[WS_STAGES][ROWBUF];
  unsigned char v[WS_STAGES][ROWBUF];  // MN-major B operand of O = P V
  // additive log2-domain bias of key j for a query row of label 0 / 1: 0 for the same label,
  // -100 log2(e) for the other, -inf for padding keys (j >= L, up to the last 32-key chunk)
  float kbias[WS_STAGES][2][MAXL + 16];
  int tok[WS_STAGES][MAXL];          // token row of smem row j
  short wr[WS_STAGES][MAXL];         // window-order index of smem row j
  signed char lab[WS_STAGES][MAXL];  // mask label of smem row j (-1: padding)
  float qn[WS_STAGES][MAXL];         // |qhat| of q row j
  float kn[WS_STAGES][4];            // max |khat| over each norm warp's k rows
  int mixed[WS_STAGES];
  float qwv[HD];
  float kwv[HD];
  uint64_t loaded[WS_STAGES];      // rows landed (TMA transaction count)
  uint64_t normed[WS_STAGES];      // q/k normalised, norms written (4 norm warps)
  uint64_t stage_free[WS_STAGES];  // MMAs done with the rows (commit) and tables read (4 warps)
  uint64_t s_full[2];              // warpgroup w: S of the current tile in TMEM (MMA commit)
  uint64_t p_ready[2];             // warpgroup w: P written to TMEM (4 warps)
  uint64_t o_full[2];              // warpgroup w: O of the current tile in TMEM (MMA commit)
  uint64_t o_free[2];              // warpgroup w: O drained from TMEM (4 warps)
  uint64_t mma_done[2];            // MMA issuer w: every product it issued has completed
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void mb_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mb_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Bounded wait of one thread on an mbarrier phase; false on timeout (error recorded, abort raised)
// or once another role has raised the abort flag.  With abort == nullptr the flag is not watched
// (clean-up waits) and a timeout records nothing.  Each try_wait carries a suspend-time hint, so a
// waiting thread sleeps in the barrier unit until the phase completes (or about a millisecond
// passes) instead of spinning: with fifteen waiting roles per CTA, spinning threads took most of
// the issue slots from the working warps.
__device__ __forceinline__ bool ws_wait1(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(1000000u)
        : "memory");
    if (ok) return true;
    if (abort && *abort) return false;
    if ((unsigned long long)(clock64() - t0) > kWaitBudgetCycles) {
      if (abort) {
        if (err) record_error(err, kErrWaitTimeout);
        *abort = 1;
      }
      return false;
    }
  }
}
// The same, polled by lane 0 and broadcast, so the warp leaves a loop as one.
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort, int lane) {
  int ok = 1;
  if (lane == 0) ok = ws_wait1(bar, parity, err, abort) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 32 columns of this warp's lane quarter without waiting, and the wait naming the registers (so no
// use of them is scheduled before it): the next chunk's load is in flight while one is processed.
__device__ __forceinline__ void ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void ld_wait32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Tables of window `w`'s smem rows, by one warp; returns whether the window mixes labels.
__device__ __forceinline__ int ws_table(const AttnGeom& g, int64_t w, int nww, int nwh, int L, int* tok,
                                        signed char* lab, short* wr, float (*kbias)[MAXL + 16], int lane) {
  WinPos p;
  p.wx = (int)(w % nww);
  p.wy = (int)((w / nww) % nwh);
  p.b = (int)(w / ((int64_t)nww * nwh));
  const WinLoad wl = win_load(g, w, nww, nwh);
  const int lab0 = label(g, p, 0);
  const float ml2 = -100.f * kLog2e;
  int mx = 0;
  for (int j = lane; j < MAXL + 16; j += 32) {
    const int i = j < L ? win_row(g, wl, j) : 0;
    const int lb = j < L ? label(g, p, i) : -1;
    if (j < MAXL) {
      wr[j] = (short)i;
      lab[j] = (signed char)lb;
      tok[j] = j < L ? (int)token(g, p, i) : 0;
    }
    kbias[0][j] = lb < 0 ? -INFINITY : (lb != 0 ? ml2 : 0.f);
    kbias[1][j] = lb < 0 ? -INFINITY : (lb != 1 ? ml2 : 0.f);
    mx |= (j < L && lb != lab0);
  }
  return __any_sync(0xffffffffu, mx);
}

// P = exp2(s - m) of 32 logits (raw S in v, columns [c, c + 32) of this thread's row) as bf16 pairs
// into TMEM columns [c/2, c/2 + 16); adds them to the row sum l.
__device__ __forceinline__ void ws_probs(const uint32_t* v, int c, int mixed, int L, float sl2, float m,
                                         const float* kb, uint32_t trow, float& l) {
  uint32_t pk[16];
  if (!mixed && c + 32 <= L) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float p0 = ex2(fmaf(__uint_as_float(v[2 * i]), sl2, -m));
      const float p1 = ex2(fmaf(__uint_as_float(v[2 * i + 1]), sl2, -m));
      l += p0 + p1;
      pk[i] = pack_bf16(p0, p1);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float4 b4 = *reinterpret_cast<const float4*>(kb + c + 2 * i);
      const float p0 = ex2(fmaf(__uint_as_float(v[2 * i]), sl2, b4.x - m));
      const float p1 = ex2(fmaf(__uint_as_float(v[2 * i + 1]), sl2, b4.y - m));
      const float p2 = ex2(fmaf(__uint_as_float(v[2 * i + 2]), sl2, b4.z - m));
      const float p3 = ex2(fmaf(__uint_as_float(v[2 * i + 3]), sl2, b4.w - m));
      l += (p0 + p1) + (p2 + p3);
      pk[i] = pack_bf16(p0, p1);
      pk[i + 1] = pack_bf16(p2, p3);
    }
  }
  st16(trow + (uint32_t)(c >> 1), pk);
}

// The CTAs walk the windows column-major (window row fastest), so that every CTA's contiguous range
// holds its share of the bottom window row, whose windows mix mask labels and cost more: in row-
// major order a few CTAs got only such windows and finished last.  Returns the item index
// (window * nh + head, the lse layout) of position j of that order.
__device__ __forceinline__ int64_t ws_item(const AttnGeom& g, int nww, int nwh, int64_t j, int64_t* win, int* h) {
  const int64_t wq = j / g.nh;
  *h = (int)(j - wq * g.nh);
  const int64_t per = (int64_t)nww * nwh;
  const int64_t b = wq / per, rem = wq - b * per;
  const int wx = (int)(rem / nwh), wy = (int)(rem - (int64_t)(rem / nwh) * nwh);
  *win = (b * nwh + wy) * nww + wx;
  return *win * g.nh + *h;
}

__global__ void __launch_bounds__(WS_THREADS, 1)
    fwd_ws_kernel(const __grid_constant__ BoxMaps box_qkv, const float* __restrict__ qw, const float* __restrict__ kw,
                  __nv_bfloat16* __restrict__ out, float* __restrict__ lse, AttnGeom g, int* err,
                  long long* __restrict__ stamps) {
  extern __shared__ unsigned char smem_raw[];
  SmemWS& S = *reinterpret_cast<SmemWS*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = g.T * g.wh * g.ww;
  const int NK = (L + 15) & ~15;
  const int ntiles = (L + 127) / 128;
  const int nww = g.W / g.ww, nwh = g.H / g.wh;
  const int C = g.nh * HD;
  const int64_t n_items = (int64_t)g.B * nwh * nww * g.nh;
  const int64_t i_begin = n_items * blockIdx.x / gridDim.x;
  const int64_t n_local = n_items * (blockIdx.x + 1) / gridDim.x - i_begin;
  volatile int* abort = &S.abort;
  // optional phase timestamps (SM clock) of the first 64 items of the first 16 CTAs; null in
  // production.  Slot k of item n: stamps[(blockIdx.x * 64 + n) * 16 + k].
  long long* st = (stamps && blockIdx.x < 16) ? stamps + (int64_t)blockIdx.x * 64 * 16 : nullptr;
#define WS_STAMP(n_, k_)                                   \
  do {                                                     \
    if (st && (n_) < 64) st[(n_) * 16 + (k_)] = clock64(); \
  } while (0)

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(WS_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < WS_STAGES; ++s) {
      mb_init(&S.loaded[s], 1);
      mb_init(&S.normed[s], 4);
      mb_init(&S.stage_free[s], 5);
    }
    for (int w = 0; w < 2; ++w) {
      mb_init(&S.s_full[w], 1);
      mb_init(&S.p_ready[w], 4);
      mb_init(&S.o_full[w], 1);
      mb_init(&S.o_free[w], 4);
      mb_init(&S.mma_done[w], 1);
    }
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // rows [L, 176) of every operand buffer stay zero (the loads write rows < L only)
  for (int idx = tid; idx < (MAXL - L) * 8; idx += WS_THREADS) {
    const int r = L + (idx >> 3), c = idx & 7;
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int s = 0; s < WS_STAGES; ++s) {
      *reinterpret_cast<uint4*>(S.q[s] + swz(r, c)) = z;
      *reinterpret_cast<uint4*>(S.k[s] + swz(r, c)) = z;
      *reinterpret_cast<uint4*>(S.v[s] + swz(r, c)) = z;
    }
  }
  if (tid < HD) {
    S.qwv[tid] = qw[tid];
    S.kwv[tid] = kw[tid];
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    int64_t tab_win[WS_STAGES] = {-1, -1, -1};
    int64_t issued[WS_STAGES] = {0, 0, 0};
    for (int64_t n = 0; n < n_local; ++n) {
      const int s = (int)(n % WS_STAGES);
      const int64_t use = n / WS_STAGES;
      if (lane == 0) WS_STAMP(n, 0);
      if (use > 0 && !ws_wait(&S.stage_free[s], (uint32_t)((use - 1) & 1), err, abort, lane)) break;
      int64_t win;
      int h;
      ws_item(g, nww, nwh, i_begin + n, &win, &h);
      if (win != tab_win[s]) {
        const int mx = ws_table(g, win, nww, nwh, L, S.tok[s], S.lab[s], S.wr[s], S.kbias[s], lane);
        if (lane == 0) S.mixed[s] = mx;
        tab_win[s] = win;
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) {
        mb_expect_tx(&S.loaded[s], (uint32_t)(3 * L * ROW_B));
        const WinLoad wl = win_load(g, win, nww, nwh);
        load_window(S.q[s], box_qkv, &S.loaded[s], h * HD, wl, g);
        load_window(S.k[s], box_qkv, &S.loaded[s], C + h * HD, wl, g);
        load_window(S.v[s], box_qkv, &S.loaded[s], 2 * C + h * HD, wl, g);
        WS_STAMP(n, 1);
      }
      __syncwarp();
      ++issued[s];
    }
    // loads still in flight land before the shared memory is released
    if (lane == 0)
      for (int s = 0; s < WS_STAGES; ++s)
        if (issued[s] > 0) ws_wait1(&S.loaded[s], (uint32_t)((issued[s] - 1) & 1), nullptr, nullptr);
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ---------------------------------------------------------------- MMA issuers
    const int w = warp - 1;
    if (lane == 0) {
      const uint32_t tb = tmem + 256u * (uint32_t)w;
      const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NK >> 3) << 17) |
                            ((uint32_t)(128 >> 4) << 24);
      const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                            ((uint32_t)(128 >> 4) << 24);
      uint32_t c_s = 0, c_o = 0;
      bool ok = true;
      for (int64_t n = w; n < n_local && ok; n += 2) {
        const int s = (int)(n % WS_STAGES);
        ok = ws_wait1(&S.normed[s], (uint32_t)((n / WS_STAGES) & 1), err, abort);
        WS_STAMP(n, 13);
        for (int t = 0; t < ntiles && ok; ++t) {
          // S_t overwrites the columns from which the previous O product read P
          if (c_o > 0) ok = ws_wait1(&S.o_full[w], (c_o - 1) & 1, err, abort);
          if (!ok) break;
          fence_after();
          const int qrow = t == 0 ? 0 : NK - 128;
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks)
            mma_ss(tb, desc_kmajor(S.q[s] + qrow * ROW_B + ks * 32), desc_kmajor(S.k[s] + ks * 32), id_s, ks > 0);
          commit(&S.s_full[w]);
          if (t == 0) WS_STAMP(n, 14);
          ++c_s;
          ok = ws_wait1(&S.p_ready[w], (c_s - 1) & 1, err, abort);
          // the previous O has been drained from its columns
          if (ok && c_o > 0) ok = ws_wait1(&S.o_free[w], (c_o - 1) & 1, err, abort);
          if (!ok) break;
          fence_after();
          for (int ks = 0; ks < NK / 16; ++ks)
            mma_ts(tb + WS_O_COL, tb + 8u * (uint32_t)ks, desc_mnmajor(S.v[s] + ks * 16 * ROW_B), id_o, ks > 0);
          commit(&S.o_full[w]);
          ++c_o;
        }
        WS_STAMP(n, 15);
        if (ok) commit(&S.stage_free[s]);  // arrives once this item's products have all completed
      }
      commit(&S.mma_done[w]);
      ws_wait1(&S.mma_done[w], 0, nullptr, nullptr);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- QK-RMSNorm
    const int nt = tid - 128, nw = warp - 4;
    for (int64_t n = 0; n < n_local; ++n) {
      const int s = (int)(n % WS_STAGES);
      if (!ws_wait(&S.loaded[s], (uint32_t)((n / WS_STAGES) & 1), err, abort, lane)) break;
      if (nt == 0) WS_STAMP(n, 2);
      float kmax = 0.f;
      // two threads per row (32 columns each), four partial sums per thread: the squares of x (for
      // rs) and of x * w (for |qhat| = rs * |x * w|) come from one pass over the row
      for (int base = 0; base < 4 * L; base += 128) {
        if (base + (nt & ~31) >= 4 * L) break;  // warp-uniform
        const int idx = base + nt;
        const bool act = idx < 4 * L;
        const int hr = act ? idx >> 1 : 0, half = idx & 1;
        const bool isq = hr < L;
        const int r = isq ? hr : hr - L;
        unsigned char* row = isq ? S.q[s] : S.k[s];
        const float* wv = (isq ? S.qwv : S.kwv) + 32 * half;
        float x[4][8];
        float ss[4] = {0.f, 0.f, 0.f, 0.f}, sw[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(row + swz(r, 4 * half + c)), x[c]);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float xw = x[c][i] * wv[8 * c + i];
            ss[i & 3] = fmaf(x[c][i], x[c][i], ss[i & 3]);
            sw[i & 3] = fmaf(xw, xw, sw[i & 3]);
            x[c][i] = xw;
          }
        }
        float ssum = (ss[0] + ss[1]) + (ss[2] + ss[3]);
        float swsum = (sw[0] + sw[1]) + (sw[2] + sw[3]);
        ssum += __shfl_xor_sync(0xffffffffu, ssum, 1);
        swsum += __shfl_xor_sync(0xffffffffu, swsum, 1);
        const float rs = rsqrtf(ssum * (1.f / HD) + FLT_EPSILON);
        if (act) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[c][i] *= rs;
            *reinterpret_cast<uint4*>(row + swz(r, 4 * half + c)) = pack8<__nv_bfloat16>(x[c]);
          }
          const float nrm = rs * sqrtf(swsum) * 1.01f;  // margin for the bf16 rounding of the operands
          if (half == 0) {
            if (isq) S.qn[s][r] = nrm;
            else kmax = fmaxf(kmax, nrm);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
      if (lane == 0) S.kn[s][nw] = kmax;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mb_arrive(&S.normed[s]);
      if (nt == 0) WS_STAMP(n, 3);
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int w = (warp - 8) >> 2;
    const int lg = warp & 3;
    const uint32_t tb = tmem + 256u * (uint32_t)w;
    const uint32_t trow = tb + ((uint32_t)(lg * 32) << 16);
    const float sl2 = g.scale * kLog2e;
    uint32_t c_s = 0, c_o = 0;
    bool ok = true;
    for (int64_t n = w; n < n_local && ok; n += 2) {
      const int s = (int)(n % WS_STAGES);
      int64_t win;
      int h;
      const int64_t item = ws_item(g, nww, nwh, i_begin + n, &win, &h);
      // the stage's tables were written before its loads; visible once its rows are normalised
      ok = ws_wait(&S.normed[s], (uint32_t)((n / WS_STAGES) & 1), err, abort, lane);
      if (!ok) break;
      const bool stamper = lg == 3 && lane == 0;
      if (stamper) WS_STAMP(n, 4);
      const int mixed = S.mixed[s];
      const float kmax = fmaxf(fmaxf(S.kn[s][0], S.kn[s][1]), fmaxf(S.kn[s][2], S.kn[s][3]));
      for (int t = 0; t < ntiles && ok; ++t) {
        const int qrow = t == 0 ? 0 : NK - 128;
        const int lo = t * 128;
        const int r = qrow + lg * 32 + lane;
        const bool live = r >= lo && r < L;
        const bool warp_live = qrow + lg * 32 + 31 >= lo && qrow + lg * 32 < L;  // warp-uniform
        ok = ws_wait(&S.s_full[w], c_s & 1, err, abort, lane);
        ++c_s;
        if (!ok) break;
        if (stamper) WS_STAMP(n, 5 + 4 * t);
        fence_after();
        float m = -INFINITY, l = 0.f;
        if (warp_live) {
          const int lr = r < L ? S.lab[s][r] : 0;
          const float* kb = S.kbias[s][lr > 0 ? 1 : 0];
          const float bound = sl2 * (r < L ? S.qn[s][r] : 0.f) * kmax;
          if (__all_sync(0xffffffffu, bound <= WS_MAX_BOUND)) {
            m = bound;
          } else {
            // exact row max of the scaled, biased logits (scale > 0: the raw maximum of a chunk
            // without bias, scaled once at the end)
            float mraw = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < NK; c += 32) {
              float v[32];
              ld32(trow + (uint32_t)c, v);
              if (!mixed && c + 32 <= L) {
#pragma unroll
                for (int i = 0; i < 32; ++i) mraw = fmaxf(mraw, v[i]);
              } else {
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                  const float4 b4 = *reinterpret_cast<const float4*>(kb + c + i);
                  m = fmaxf(m, fmaxf(fmaxf(fmaf(v[i], sl2, b4.x), fmaf(v[i + 1], sl2, b4.y)),
                                     fmaxf(fmaf(v[i + 2], sl2, b4.z), fmaf(v[i + 3], sl2, b4.w))));
                }
              }
            }
            m = fmaxf(m, mraw * sl2);
          }
          // P = exp2(s - m) as bf16 pairs over the front of S (columns c/2 < c: already read).  The
          // loop is kept rolled with one TMEM load in flight: unrolled, the four roles' loops no longer
          // fit the instruction caches (instruction-fetch stalls, 40% slower); with a second register
          // buffer the softmax warps spill at 128 registers (30% slower).
#pragma unroll 1
          for (int c = 0; c < NK; c += 32) {
            uint32_t v[32];
            ld32_async(trow + (uint32_t)c, v);
            ld_wait32(v);
            ws_probs(v, c, mixed, L, sl2, m, kb, trow, l);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&S.p_ready[w]);
        if (stamper) WS_STAMP(n, 6 + 4 * t);
        // ---- epilogue of tile t: O / rowsum to the token rows; lse per row
        ok = ws_wait(&S.o_full[w], c_o & 1, err, abort, lane);
        ++c_o;
        if (!ok) break;
        if (stamper) WS_STAMP(n, 7 + 4 * t);
        fence_after();
        if (warp_live) {
          const float il = 1.f / l;
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)S.tok[s][live ? r : 0] * g.out_stride + (int64_t)h * HD);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float o[32];
            ld32(trow + WS_O_COL + 32u * hf, o);
            if (live) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float f8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) f8[i] = o[8 * c + i] * il;
                dst[4 * hf + c] = pack8<__nv_bfloat16>(f8);
              }
            }
          }
          if (live) lse[item * L + S.wr[s][r]] = m + __log2f(l);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&S.o_free[w]);  // the next O product may start
        if (stamper) WS_STAMP(n, 8 + 4 * t);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mb_arrive(&S.stage_free[s]);  // this warp is done with the stage's tables
    }
    __syncwarp();
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(WS_TMEM_COLS));
#undef WS_STAMP
}

}  // namespace attn_tc

bool window_attn_fwd_tc_supported(const AttnGeom& g, int dtype) {
  const int L = g.T * g.wh * g.ww;
  return dtype == kBF16 && g.hd == 64 && L >= 1 && L <= attn_tc::MAXL && g.H % g.wh == 0 && g.W % g.ww == 0;
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 4-D view [B*T, H, W, ld] of a token-major bf16 tensor, box = [1, h, w, 64] (SWIZZLE_128B)
bool box_map(CUtensorMap* map, const void* ptr, const AttnGeom& g, int64_t ld, int w, int h) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)ld, (cuuint64_t)g.W, (cuuint64_t)g.H, (cuuint64_t)g.B * g.T};
  cuuint64_t strides[3] = {(cuuint64_t)(ld * 2), (cuuint64_t)(ld * 2 * g.W), (cuuint64_t)(ld * 2 * g.W * g.H)};
  cuuint32_t box[4] = {64, (cuuint32_t)w, (cuuint32_t)h, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Split of a window dimension at the grid edge: first-part size of the one window column (row)
// that wraps, 0 if none wraps (the grid is a whole number of windows, so all wrapping windows
// split the same way).
int wrap_split(int n, int wsize, int shift) {
  for (int w0 = 0; w0 < n; w0 += wsize) {
    int x0 = (w0 + shift) % n;
    if (x0 < 0) x0 += n;
    if (x0 + wsize > n) return n - x0;
  }
  return 0;
}

// The 3 x 3 box shapes {full, first part, second part} of width x height (see box_index).
bool window_box_maps(attn_tc::BoxMaps* maps, const void* ptr, const AttnGeom& g, int64_t ld) {
  const int ax = wrap_split(g.W, g.ww, g.sw), ay = wrap_split(g.H, g.wh, g.sh);
  const int ws[3] = {g.ww, ax, g.ww - ax}, hs[3] = {g.wh, ay, g.wh - ay};
  for (int yi = 0; yi < 3; ++yi)
    for (int xi = 0; xi < 3; ++xi) {
      CUtensorMap* m = &maps->m[yi * 3 + xi];
      memset(m, 0, sizeof(*m));
      if (ws[xi] <= 0 || hs[yi] <= 0 || ws[xi] > 256 || hs[yi] > 256) continue;
      if (!box_map(m, ptr, g, ld, ws[xi], hs[yi])) return false;
    }
  return true;
}
}  // namespace

cudaError_t window_attn_bwd_tc(const void* qkv, const float* qw, const float* kw, const void* out,
                               const void* dout, const float* lse, void* dqkv, float* dqw_part, float* dkw_part,
                               const AttnGeom& g, cudaStream_t s, long long* stamps) {
  const size_t smem = sizeof(attn_tc::SmemB) + 1024;
  auto k = attn_tc::bwd_kernel;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int dev = 0, sms = 0;
  NSW_CUDA_CHECK(cudaGetDevice(&dev));
  NSW_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t n_tok = (int64_t)g.B * g.T * g.H * g.W;
  if (n_tok >= (1LL << 31) - 1) return cudaErrorInvalidValue;
  (void)out;  // D = rowsum(P dP) is formed in the kernel; O itself is not read
  attn_tc::BoxMaps b_qkv, b_dout;
  if (!window_box_maps(&b_qkv, qkv, g, g.qkv_stride) || !window_box_maps(&b_dout, dout, g, g.out_stride))
    return cudaErrorInvalidValue;
  const int64_t items = (int64_t)g.B * (g.H / g.wh) * (g.W / g.ww) * g.nh;
  const int grid = (int)std::min<int64_t>(items, sms);
  k<<<grid, attn_tc::BWD_THREADS, smem, s>>>(b_qkv, b_dout, (const __nv_bfloat16*)qkv, qw, kw,
                                             (const __nv_bfloat16*)dout, lse,
                                             (__nv_bfloat16*)dqkv, dqw_part, dkw_part, g, device_error_flag(),
                                             stamps);
  return cudaGetLastError();
}

cudaError_t window_attn_fwd_ws(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                               const AttnGeom& g, cudaStream_t s, long long* stamps) {
  if (!(g.scale > 0.f)) return cudaErrorInvalidValue;  // the row max is taken on unscaled logits
  const size_t smem = sizeof(attn_tc::SmemWS) + 1024;
  auto k = attn_tc::fwd_ws_kernel;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int dev = 0, sms = 0;
  NSW_CUDA_CHECK(cudaGetDevice(&dev));
  NSW_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t n_tok = (int64_t)g.B * g.T * g.H * g.W;
  if (n_tok >= (1LL << 31) - 1) return cudaErrorInvalidValue;
  attn_tc::BoxMaps b_qkv;
  if (!window_box_maps(&b_qkv, qkv, g, g.qkv_stride)) return cudaErrorInvalidValue;
  const int64_t items = (int64_t)g.B * (g.H / g.wh) * (g.W / g.ww) * g.nh;
  const int grid = (int)std::min<int64_t>(items, sms);
  k<<<grid, attn_tc::WS_THREADS, smem, s>>>(b_qkv, qw, kw, (__nv_bfloat16*)out, lse, g, device_error_flag(),
                                            stamps);
  return cudaGetLastError();
}

cudaError_t window_attn_fwd_tc(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                               const AttnGeom& g, cudaStream_t s) {
  const size_t smem = sizeof(attn_tc::SmemF) + 1024;
  auto k = attn_tc::fwd_kernel;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int dev = 0, sms = 0;
  NSW_CUDA_CHECK(cudaGetDevice(&dev));
  NSW_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t n_tok = (int64_t)g.B * g.T * g.H * g.W;
  if (n_tok >= (1LL << 31) - 1) return cudaErrorInvalidValue;
  attn_tc::BoxMaps b_qkv;
  if (!window_box_maps(&b_qkv, qkv, g, g.qkv_stride)) return cudaErrorInvalidValue;
  const int64_t items = (int64_t)g.B * (g.H / g.wh) * (g.W / g.ww) * g.nh;
  const int grid = (int)std::min<int64_t>(items, sms);
  k<<<grid, attn_tc::FWD_THREADS, smem, s>>>(b_qkv, qw, kw, (__nv_bfloat16*)out, lse, g, device_error_flag());
  return cudaGetLastError();
}

}  // namespace nsw
