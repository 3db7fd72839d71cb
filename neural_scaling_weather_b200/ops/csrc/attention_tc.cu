// Shifted-window attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract and numerics as the mma.sync forward in attention.cu (gathered window
// tokens by index arithmetic, QK-RMSNorm in shared memory, additive -100 latitude-wrap
// mask, exp2-domain softmax, log2-domain LSE for the backward), specialised for the
// production geometry: head_dim 64 and windows of at most 176 tokens (T*wh*ww <= 176).
//
// One CTA of 4 warps owns one (window, head); two CTAs fit per SM (76 KB smem, 256 TMEM
// columns each).  Per 128-row query tile t (one or two tiles):
//   S_t = Qhat_t Khat^T        tcgen05.mma kind::f16, M=128, N=NK (keys rounded to 16),
//                              both operands K-major 128-byte-swizzled smem, fp32 in TMEM;
//   softmax                    each thread owns one query row (its TMEM lane): reads S in
//                              16-column chunks (tcgen05.ld), row max, exp2, row sum, and
//                              writes P as packed bf16 pairs back over the front of S
//                              (tcgen05.st) -- P never touches shared memory;
//   O_t = P_t V                tcgen05.mma with A read from TMEM and B = V as an MN-major
//                              swizzled smem operand (V rows are keys with d contiguous,
//                              exactly the MN-major canonical layout), fp32 in TMEM;
//   epilogue                   tcgen05.ld of the O row, 1/rowsum, bf16, 16-byte stores to
//                              the token's grid position; LSE per row.
// One mbarrier tracks the MMA completions (tcgen05.commit); its waits are bounded by a
// %globaltimer budget and record kErrWaitTimeout in the device error word on expiry.
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace nsw {
namespace attn_tc {

constexpr int HD = 64;
constexpr int ROW_B = HD * 2;        // 128 bytes per row (one swizzle row)
constexpr int MAXL = 176;            // keys padded to a multiple of 16, at most 176
constexpr int Q_ROWS = 256;          // two query tiles of 128
constexpr int O_COL = 192;           // TMEM column of the O accumulator
constexpr int TMEM_COLS = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr unsigned long long kWaitBudgetNs = 2000000000ull;

struct __align__(1024) Smem {
  unsigned char q[Q_ROWS * ROW_B];  // 32 KB, K-major SW128 (two M=128 tiles)
  unsigned char k[MAXL * ROW_B];    // 22 KB, K-major SW128 (B of S = Q K^T)
  unsigned char v[MAXL * ROW_B];    // 22 KB, MN-major SW128 (B of O = P V)
  int tok[MAXL];
  signed char lab[MAXL];
  uint64_t bar;
  uint32_t tmem_base;
  int aborted;
};

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
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void ld32(uint32_t taddr, float* f) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

__global__ void __launch_bounds__(128, 2)
    fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
               __nv_bfloat16* __restrict__ out, float* __restrict__ lse, AttnGeom g, int* err) {
  extern __shared__ unsigned char smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = g.T * g.wh * g.ww;
  const int NK = (L + 15) & ~15;
  const int ntiles = (L + 127) / 128;
  const int bw = blockIdx.x, h = blockIdx.y;
  const int nww = g.W / g.ww, nwh = g.H / g.wh;
  WinPos p;
  p.wx = bw % nww;
  p.wy = (bw / nww) % nwh;
  p.b = bw / (nww * nwh);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&S.bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // token table and labels
  const int lab0 = label(g, p, 0);
  int mixed = 0;
  for (int i = tid; i < MAXL; i += blockDim.x) {
    S.tok[i] = i < L ? (int)token(g, p, i) : 0;
    const int lb = i < L ? label(g, p, i) : -1;
    S.lab[i] = (signed char)lb;
    mixed |= (i < L && lb != lab0);
  }
  mixed = __syncthreads_or(mixed);

  // gather Q (256 rows), K and V (NK rows) into the swizzled layouts; zero the padding
  const int64_t C = (int64_t)g.nh * HD;
  const __nv_bfloat16* base = qkv + (int64_t)h * HD;
  for (int idx = tid; idx < (Q_ROWS + 2 * MAXL) * 8; idx += blockDim.x) {
    const int row_all = idx >> 3, c = idx & 7;
    unsigned char* dst;
    int r, part;
    if (row_all < Q_ROWS) {
      r = row_all;
      part = 0;
      dst = S.q + swz(r, c);
    } else if (row_all < Q_ROWS + MAXL) {
      r = row_all - Q_ROWS;
      part = 1;
      dst = S.k + swz(r, c);
    } else {
      r = row_all - Q_ROWS - MAXL;
      part = 2;
      dst = S.v + swz(r, c);
    }
    if (r < L) {
      const __nv_bfloat16* src = base + (int64_t)S.tok[r] * g.qkv_stride + part * C + c * 8;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // QK-RMSNorm in place (thread per row)
  for (int rr = tid; rr < 2 * L; rr += blockDim.x) {
    const bool isq = rr < L;
    const int r = isq ? rr : rr - L;
    unsigned char* row = isq ? S.q : S.k;
    const float* w = isq ? qw : kw;
    float f[8][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(row + swz(r, c)), f[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[c][i] * f[c][i];
    }
    const float rs = rsqrtf(ss / (float)HD + FLT_EPSILON);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[c][i] *= rs * __ldg(w + c * 8 + i);
      *reinterpret_cast<uint4*>(row + swz(r, c)) = pack8<__nv_bfloat16>(f[c]);
    }
  }
  // generic-proxy smem writes -> visible to the tensor core (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NK >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                        ((uint32_t)(128 >> 4) << 24);
  const float sl2 = g.scale * kLog2e;
  const float ml2 = -100.f * kLog2e;
  uint32_t parity = 0;
  bool ok = true;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  for (int t = 0; t < ntiles && ok; ++t) {
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks)
        mma_ss(tmem, desc_kmajor(S.q + t * 128 * ROW_B + ks * 32), desc_kmajor(S.k + ks * 32), id_s, ks > 0);
      commit(&S.bar);
    }
    __syncwarp();
    ok = __syncthreads_and(wait_bar(&S.bar, parity, err));  // CTA-uniform outcome
    parity ^= 1;
    if (!ok) break;
    fence_after();
    // ---- softmax of row r (this thread's TMEM lane)
    const int r = t * 128 + warp * 32 + lane;
    const int lr = r < L ? S.lab[r] : 0;
    const uint32_t trow = tmem + lane_base;
    float m = -INFINITY;
    for (int j = 0; j < NK / 16; ++j) {
      float v[16];
      ld16(trow + 16 * j, v);
      const bool plain = !mixed && 16 * j + 16 <= L;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float s = v[i] * sl2;
        if (!plain) {
          const int key = 16 * j + i;
          const int lk = S.lab[key];
          if (lk < 0) s = -INFINITY;
          else if (lk != lr) s += ml2;
        }
        m = fmaxf(m, s);
      }
    }
    float l = 0.f;
    for (int j = 0; j < NK / 16; ++j) {
      float v[16];
      ld16(trow + 16 * j, v);
      const bool plain = !mixed && 16 * j + 16 <= L;
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        float s0 = v[i] * sl2, s1 = v[i + 1] * sl2;
        if (!plain) {
          const int k0 = 16 * j + i;
          const int l0 = S.lab[k0], l1 = S.lab[k0 + 1];
          if (l0 < 0) s0 = -INFINITY;
          else if (l0 != lr) s0 += ml2;
          if (l1 < 0) s1 = -INFINITY;
          else if (l1 != lr) s1 += ml2;
        }
        const float p0 = ex2(s0 - m), p1 = ex2(s1 - m);
        l += p0 + p1;
        pk[i >> 1] = pack_bf16(p0, p1);
      }
      st8(trow + 8 * j, pk);  // P over the front of S: column 8j < 16j, already read
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    fence_before();
    __syncthreads();
    // ---- O = P V
    if (tid == 0) {
      fence_after();
      for (int ks = 0; ks < NK / 16; ++ks)
        mma_ts(tmem + O_COL, tmem + 8 * ks, desc_mnmajor(S.v + ks * 16 * ROW_B), id_o, ks > 0);
      commit(&S.bar);
    }
    __syncwarp();
    ok = __syncthreads_and(wait_bar(&S.bar, parity, err));
    parity ^= 1;
    if (!ok) break;
    fence_after();
    float o[64];
    ld32(trow + O_COL, o);
    ld32(trow + O_COL + 32, o + 32);
    if (r < L) {
      const float il = 1.f / l;
      __nv_bfloat16* dst = out + (int64_t)S.tok[r] * g.out_stride + (int64_t)h * HD;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float f8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f8[i] = o[c * 8 + i] * il;
        reinterpret_cast<uint4*>(dst)[c] = pack8<__nv_bfloat16>(f8);
      }
      lse[((int64_t)bw * g.nh + h) * L + r] = m + __log2f(l);
    }
    fence_before();
    __syncthreads();  // S/P and O columns are reused by the next tile
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

}  // namespace attn_tc

bool window_attn_fwd_tc_supported(const AttnGeom& g, int dtype) {
  const int L = g.T * g.wh * g.ww;
  return dtype == kBF16 && g.hd == 64 && L >= 1 && L <= attn_tc::MAXL && g.H % g.wh == 0 && g.W % g.ww == 0;
}

cudaError_t window_attn_fwd_tc(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                               const AttnGeom& g, cudaStream_t s) {
  const size_t smem = sizeof(attn_tc::Smem) + 1024;
  auto k = attn_tc::fwd_kernel;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(g.B * (g.H / g.wh) * (g.W / g.ww), g.nh);
  k<<<grid, 128, smem, s>>>((const __nv_bfloat16*)qkv, qw, kw, (__nv_bfloat16*)out, lse, g, device_error_flag());
  return cudaGetLastError();
}

}  // namespace nsw
