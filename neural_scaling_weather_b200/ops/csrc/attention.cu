// Shifted-window multi-head attention with fused QK-RMSNorm (forward and backward).
//
// One CTA owns one (batch, window, head).  Its L = T*wh*ww tokens are gathered straight
// from the token-major qkv tensor by index arithmetic: window token (t, iy, ix) of window
// (wy, wx) reads grid token ((wy*wh + iy + sh) mod H, (wx*ww + ix + sw) mod W), which is
// the reference's roll(-shift) + window_partition (models/swin_helpers.py:26-77, 399-433),
// and the output goes back to the same grid position (window_reverse + roll(+shift)).
// The latitude-wrap mask (models/swin_helpers.py:322-397) is recomputed from row
// indices: tokens whose global rolled row is >= h_global - mask_shift form region 1,
// and scores between tokens of different regions get -100 added (the reference adds
// -100, not -inf).  Padding keys beyond L are excluded.
//
// QK-RMSNorm (eps = FLT_EPSILON, fp32 math, result rounded to the compute type) is
// applied while the window sits in shared memory.  Scores and P.V use mma.sync
// m16n8k16 with fp32 accumulation; softmax runs in the exp2 domain with the scale
// folded in.  The whole window (<= 16 query tiles of 16) lives in shared memory, so the
// forward needs no re-reads and the backward recomputes scores from shared memory:
// phase A (a warp per 16 keys) produces dK and dV, phase B (a warp per 16 queries)
// produces dQ; both then apply the RMSNorm backward with the raw q/k rows and write
// raw-q/k/v gradients into dqkv at the tokens' grid positions.  Per-CTA partial
// gradients of the two norm weights are reduced by the caller in a fixed order.
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace nsw {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, const uint32_t* a, uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two floats -> one packed pair of 16-bit values in a single conversion instruction.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Hardware base-2 exponential (ex2.approx.ftz: ~2 ulp), ample for probabilities that are
// rounded to 16 bits before the P.V product.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct WinPos {
  int b, wy, wx;
};

__device__ __forceinline__ WinPos win_pos(const AttnGeom& g, int bw) {
  const int nww = g.W / g.ww, nwh = g.H / g.wh;
  WinPos p;
  p.wx = bw % nww;
  p.wy = (bw / nww) % nwh;
  p.b = bw / (nww * nwh);
  return p;
}

__device__ __forceinline__ int64_t win_token(const AttnGeom& g, const WinPos& p, int i) {
  const int wa = g.wh * g.ww;
  const int t = i / wa;
  const int r = i - t * wa;
  const int iy = r / g.ww, ix = r - (r / g.ww) * g.ww;
  int gy = (p.wy * g.wh + iy + g.sh) % g.H;
  int gx = (p.wx * g.ww + ix + g.sw) % g.W;
  if (gy < 0) gy += g.H;
  if (gx < 0) gx += g.W;
  return ((int64_t)(p.b * g.T + t) * g.H + gy) * g.W + gx;
}

__device__ __forceinline__ int win_label(const AttnGeom& g, const WinPos& p, int i) {
  if (!g.mask || g.mask_shift <= 0) return 0;
  const int wa = g.wh * g.ww;
  const int iy = (i % wa) / g.ww;
  const int row_g = g.row_offset + p.wy * g.wh + iy;
  return row_g >= g.h_global - g.mask_shift ? 1 : 0;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// Grid-token index and region label of every window position (the only place with
// integer division).  Returns, to every thread, whether the window mixes two regions
// (only then does the -100 mask apply anywhere in it).
__device__ __forceinline__ bool fill_tokens(int* sTok, signed char* sLab, const AttnGeom& g, const WinPos& p,
                                            int L, int rows_pad) {
  const int lab0 = win_label(g, p, 0);
  int mixed = 0;
  for (int i = threadIdx.x; i < rows_pad; i += blockDim.x) {
    sTok[i] = i < L ? (int)win_token(g, p, i) : 0;
    const int lab = i < L ? win_label(g, p, i) : -1;
    sLab[i] = (signed char)lab;
    mixed |= (i < L && lab != lab0);
  }
  return __syncthreads_or(mixed) != 0;
}

// Issue asynchronous 16-byte copies of rows [0, L) of one of q/k/v/dO into smem (row
// stride HD+8) and zero rows [L, rows_pad); completion is awaited by cp_async_wait_all.
template <typename T, int HD>
__device__ __forceinline__ void load_rows(T* s, const T* base, int64_t stride, int64_t col0,
                                          const int* sTok, int L, int rows_pad) {
  constexpr int CH = HD / 8;
  for (int idx = threadIdx.x; idx < rows_pad * CH; idx += blockDim.x) {
    const int i = idx / CH, c = idx - i * CH;
    T* dst = s + i * (HD + 8) + c * 8;
    if (i < L) {
      const int64_t tok = sTok[i];
      cp_async16(dst, base + tok * stride + col0 + c * 8);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
}

// In-place RMSNorm of rows [0, L) of an smem tile; writes rstd per row if requested.
template <typename T, int HD>
__device__ __forceinline__ void norm_rows(T* s, const float* w, int L, float* rstd_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  constexpr int PER = HD / 32 > 0 ? HD / 32 : 1;
  for (int i = warp; i < L; i += nw) {
    T* row = s + i * (HD + 8);
    float v[PER];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = lane + 32 * k;
      v[k] = c < HD ? to_f(row[c]) : 0.f;
      ss += v[k] * v[k];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)HD + FLT_EPSILON);
    if (rstd_out && lane == 0) rstd_out[i] = rs;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = lane + 32 * k;
      if (c < HD) row[c] = from_f<T>(v[k] * rs * w[c]);
    }
  }
}

// ============================================================================= forward
template <typename T, int HD>
__global__ void __launch_bounds__(256, 2) fwd_kernel(const T* __restrict__ qkv, const float* __restrict__ qw,
                                                  const float* __restrict__ kw, T* __restrict__ out,
                                                  float* __restrict__ lse, AttnGeom g) {
  constexpr int RS = HD + 8;  // smem row stride (elements); +16 B breaks bank conflicts
  constexpr int KS = HD / 16;
  constexpr int DT = HD / 8;
  extern __shared__ __align__(16) unsigned char smem[];
  const int L = g.T * g.wh * g.ww;
  const int nqt = (L + 15) / 16;
  const int lq = nqt * 16;
  const int lk = ((L + 63) / 64) * 64;
  T* sQ = reinterpret_cast<T*>(smem);
  T* sK = sQ + lq * RS;
  T* sV = sK + lk * RS;
  int* sTok = reinterpret_cast<int*>(sV + lk * RS);
  signed char* sLab = reinterpret_cast<signed char*>(sTok + lk);

  const int bw = blockIdx.x, h = blockIdx.y;
  const WinPos p = win_pos(g, bw);
  const int64_t C = (int64_t)g.nh * HD;
  const bool mixed = fill_tokens(sTok, sLab, g, p, L, lk);
  load_rows<T, HD>(sQ, qkv, g.qkv_stride, 0 * C + (int64_t)h * HD, sTok, L, lq);
  load_rows<T, HD>(sK, qkv, g.qkv_stride, 1 * C + (int64_t)h * HD, sTok, L, lk);
  load_rows<T, HD>(sV, qkv, g.qkv_stride, 2 * C + (int64_t)h * HD, sTok, L, lk);
  cp_async_wait_all();
  __syncthreads();
  norm_rows<T, HD>(sQ, qw, L, nullptr);
  norm_rows<T, HD>(sK, kw, L, nullptr);
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const float sl2 = g.scale * kLog2e;
  const float ml2 = -100.f * kLog2e;

  for (int qt = warp; qt < nqt; qt += nw) {
    uint32_t qa[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int r = qt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = ks * 16 + (lane >> 4) * 8;
      ldsm_x4(smem_u32(sQ + r * RS + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    }
    const int r0 = qt * 16 + gq, r1 = r0 + 8;
    const int lab0 = sLab[r0] < 0 ? 0 : sLab[r0];
    const int lab1 = sLab[r1] < 0 ? 0 : sLab[r1];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[DT][4];
#pragma unroll
    for (int d = 0; d < DT; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;

    for (int kc = 0; kc < lk; kc += 64) {
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
          uint32_t b0, b1, b2, b3;
          const int r = kc + pr * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = ks * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(smem_u32(sK + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(s[2 * pr], qa[ks], b0, b1);
          mma16816<T>(s[2 * pr + 1], qa[ks], b2, b3);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
      if (!mixed && kc + 64 <= L) {
        // no mask and no padding in this chunk (the common case)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            s[j][e] *= sl2;
            s[j][2 + e] *= sl2;
            mx0 = fmaxf(mx0, s[j][e]);
            mx1 = fmaxf(mx1, s[j][2 + e]);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = kc + j * 8 + 2 * tq + e;
            const int lc = sLab[col];
            float v0 = s[j][e] * sl2, v1 = s[j][2 + e] * sl2;
            if (lc < 0) {
              v0 = -INFINITY;
              v1 = -INFINITY;
            } else {
              if (lc != lab0) v0 += ml2;
              if (lc != lab1) v1 += ml2;
            }
            s[j][e] = v0;
            s[j][2 + e] = v1;
            mx0 = fmaxf(mx0, v0);
            mx1 = fmaxf(mx1, v1);
          }
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float c0 = fast_exp2(m0 - mn0), c1 = fast_exp2(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 *= c0;
      l1 *= c1;
#pragma unroll
      for (int d = 0; d < DT; ++d) {
        o[d][0] *= c0;
        o[d][1] *= c0;
        o[d][2] *= c1;
        o[d][3] *= c1;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = fast_exp2(s[j][0] - mn0);
        s[j][1] = fast_exp2(s[j][1] - mn0);
        s[j][2] = fast_exp2(s[j][2] - mn1);
        s[j][3] = fast_exp2(s[j][3] - mn1);
        l0 += s[j][0] + s[j][1];
        l1 += s[j][2] + s[j][3];
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int r = kc + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(smem_u32(sV + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(o[2 * dp], pa, b0, b1);
          mma16816<T>(o[2 * dp + 1], pa, b2, b3);
        }
      }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float il0 = 1.f / l0, il1 = 1.f / l1;
    // stage the 16 x HD output tile in this warp's own Q rows, then store 16-byte chunks
    __syncwarp();
#pragma unroll
    for (int d = 0; d < DT; ++d) {
      const int c = d * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(sQ + r0 * RS + c) = pack2<T>(o[d][0] * il0, o[d][1] * il0);
      *reinterpret_cast<uint32_t*>(sQ + r1 * RS + c) = pack2<T>(o[d][2] * il1, o[d][3] * il1);
    }
    if (tq == 0) {
      const int64_t base = ((int64_t)bw * g.nh + h) * L;
      if (r0 < L) lse[base + r0] = m0 + log2f(l0);
      if (r1 < L) lse[base + r1] = m1 + log2f(l1);
    }
    __syncwarp();
    for (int idx = lane; idx < 16 * DT; idx += 32) {
      const int rr = idx / DT, cc = idx - rr * DT;
      const int i = qt * 16 + rr;
      if (i < L) {
        const int64_t tok = sTok[i];
        *reinterpret_cast<uint4*>(out + tok * g.out_stride + (int64_t)h * HD + cc * 8) =
            *reinterpret_cast<const uint4*>(sQ + i * RS + cc * 8);
      }
    }
  }
}

// ============================================================================= backward
template <typename T, int HD>
__device__ __forceinline__ void norm_backward_store(
    float (*acc)[4], int row0, int lane, const T* __restrict__ raw_base, int64_t stride,
    int64_t col0, const float* __restrict__ w, const float* s_rstd, const int* sTok, int L,
    T* __restrict__ dst, float* wacc) {
  // acc: gradient w.r.t. the normed rows (16 rows x HD) in mma C layout.
  constexpr int DT = HD / 8;
  const int gq = lane >> 2, tq = lane & 3;
  const int rows[2] = {row0 + gq, row0 + gq + 8};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int i = rows[half];
    const bool valid = i < L;
    const int64_t tok = valid ? sTok[i] : 0;
    const float rs = valid ? s_rstd[i] : 0.f;
    float xr[DT][2];
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < DT; ++d) {
      const int c = d * 8 + 2 * tq;
      if (valid) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(raw_base + tok * stride + col0 + c);
        const T* hv = reinterpret_cast<const T*>(&u);
        xr[d][0] = to_f(hv[0]);
        xr[d][1] = to_f(hv[1]);
      } else {
        xr[d][0] = xr[d][1] = 0.f;
      }
      dot += w[c] * acc[d][2 * half] * xr[d][0] + w[c + 1] * acc[d][2 * half + 1] * xr[d][1];
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    const float k3 = rs * rs * rs * dot / (float)HD;
#pragma unroll
    for (int d = 0; d < DT; ++d) {
      const int c = d * 8 + 2 * tq;
      const float g0 = acc[d][2 * half], g1 = acc[d][2 * half + 1];
      wacc[2 * d] += g0 * xr[d][0] * rs;
      wacc[2 * d + 1] += g1 * xr[d][1] * rs;
      if (valid) {
        const float o0 = rs * w[c] * g0 - xr[d][0] * k3;
        const float o1 = rs * w[c + 1] * g1 - xr[d][1] * k3;
        *reinterpret_cast<uint32_t*>(dst + tok * stride + col0 + c) = pack2<T>(o0, o1);
      }
    }
  }
}

template <typename T, int HD>
__device__ __forceinline__ void store_rows_c(float (*acc)[4], int row0, int lane, int64_t stride,
                                             int64_t col0, const int* sTok, int L, T* __restrict__ dst) {
  constexpr int DT = HD / 8;
  const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int i = row0 + gq + 8 * half;
    if (i >= L) continue;
    const int64_t tok = sTok[i];
#pragma unroll
    for (int d = 0; d < DT; ++d) {
      const int c = d * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(dst + tok * stride + col0 + c) =
          pack2<T>(acc[d][2 * half], acc[d][2 * half + 1]);
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(192, 2) bwd_kernel(const T* __restrict__ qkv, const float* __restrict__ qw,
                                                  const float* __restrict__ kw, const T* __restrict__ out,
                                                  const T* __restrict__ dout, const float* __restrict__ lse,
                                                  T* __restrict__ dqkv, float* __restrict__ dqw_part,
                                                  float* __restrict__ dkw_part, AttnGeom g) {
  constexpr int RS = HD + 8;
  constexpr int KS = HD / 16;
  constexpr int DT = HD / 8;
  extern __shared__ __align__(16) unsigned char smem[];
  const int L = g.T * g.wh * g.ww;
  const int nt = (L + 15) / 16;
  const int lp = nt * 16;
  T* sQ = reinterpret_cast<T*>(smem);
  T* sK = sQ + lp * RS;
  T* sV = sK + lp * RS;
  T* sG = sV + lp * RS;  // dO
  float* sLse = reinterpret_cast<float*>(sG + lp * RS);
  float* sD = sLse + lp;
  float* sRq = sD + lp;
  float* sRk = sRq + lp;
  float* sWq = sRk + lp;  // [HD] partial dqw
  float* sWk = sWq + HD;  // [HD] partial dkw
  int* sTok = reinterpret_cast<int*>(sWk + HD);
  signed char* sLab = reinterpret_cast<signed char*>(sTok + lp);

  const int bw = blockIdx.x, h = blockIdx.y;
  const WinPos p = win_pos(g, bw);
  const int64_t C = (int64_t)g.nh * HD;
  const bool mixed = fill_tokens(sTok, sLab, g, p, L, lp);
  load_rows<T, HD>(sQ, qkv, g.qkv_stride, 0 * C + (int64_t)h * HD, sTok, L, lp);
  load_rows<T, HD>(sK, qkv, g.qkv_stride, 1 * C + (int64_t)h * HD, sTok, L, lp);
  load_rows<T, HD>(sV, qkv, g.qkv_stride, 2 * C + (int64_t)h * HD, sTok, L, lp);
  load_rows<T, HD>(sG, dout, g.out_stride, (int64_t)h * HD, sTok, L, lp);
  const int64_t lse_base = ((int64_t)bw * g.nh + h) * L;
  for (int i = threadIdx.x; i < lp; i += blockDim.x) sLse[i] = i < L ? lse[lse_base + i] : INFINITY;
  for (int i = threadIdx.x; i < HD; i += blockDim.x) {
    sWq[i] = 0.f;
    sWk[i] = 0.f;
  }
  {  // D_i = sum_d dO_i,d * O_i,d
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = warp; i < lp; i += nw) {
      float acc = 0.f;
      if (i < L) {
        const int64_t tok = sTok[i];
        for (int c = lane; c < HD; c += 32)
          acc += to_f(dout[tok * g.out_stride + (int64_t)h * HD + c]) *
                 to_f(out[tok * g.out_stride + (int64_t)h * HD + c]);
      }
      acc = warp_sum(acc);
      if (lane == 0) sD[i] = acc;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  norm_rows<T, HD>(sQ, qw, L, sRq);
  norm_rows<T, HD>(sK, kw, L, sRk);
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const float sl2 = g.scale * kLog2e;
  const float ml2 = -100.f * kLog2e;
  float wq[2 * DT], wk[2 * DT];
#pragma unroll
  for (int i = 0; i < 2 * DT; ++i) wq[i] = wk[i] = 0.f;

  for (int task = warp; task < 2 * nt; task += nw) {
    if (task < nt) {
      // ---------------- phase A: 16 keys -> dK, dV
      const int kt = task;
      uint32_t ka[KS][4], va[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32(sK + r * RS + c), ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3]);
        ldsm_x4(smem_u32(sV + r * RS + c), va[ks][0], va[ks][1], va[ks][2], va[ks][3]);
      }
      const int kr0 = kt * 16 + gq, kr1 = kr0 + 8;
      const int klab0 = sLab[kr0], klab1 = sLab[kr1];
      float dv[DT][4], dk[DT][4];
#pragma unroll
      for (int d = 0; d < DT; ++d)
#pragma unroll
        for (int e = 0; e < 4; ++e) dv[d][e] = dk[d][e] = 0.f;
      for (int qc = 0; qc < lp; qc += 16) {
        float st[2][4], dpt[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0, b1, b2, b3;
          const int r = qc + (lane & 7) + (lane >> 4) * 8;
          const int c = ks * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(smem_u32(sQ + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(st[0], ka[ks], b0, b1);
          mma16816<T>(st[1], ka[ks], b2, b3);
          ldsm_x4(smem_u32(sG + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(dpt[0], va[ks], b0, b1);
          mma16816<T>(dpt[1], va[ks], b2, b3);
        }
        // P^T and dS^T (rows = keys, cols = queries)
        const bool plain = !mixed && qc + 16 <= L && kt * 16 + 16 <= L;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = qc + j * 8 + 2 * tq + e;
            const float lq = sLse[q];
            const float dq = sD[q];
            float v0 = st[j][e] * sl2, v1 = st[j][2 + e] * sl2;
            float p0, p1;
            if (plain) {
              p0 = fast_exp2(v0 - lq);
              p1 = fast_exp2(v1 - lq);
            } else {
              const int ql = sLab[q];
              if (ql >= 0) {
                if (klab0 != ql) v0 += ml2;
                if (klab1 != ql) v1 += ml2;
              }
              p0 = (klab0 < 0) ? 0.f : fast_exp2(v0 - lq);
              p1 = (klab1 < 0) ? 0.f : fast_exp2(v1 - lq);
            }
            st[j][e] = p0;
            st[j][2 + e] = p1;
            dpt[j][e] = p0 * (dpt[j][e] - dq);
            dpt[j][2 + e] = p1 * (dpt[j][2 + e] - dq);
          }
        }
        uint32_t pa[4], sa[4];
        pa[0] = pack2<T>(st[0][0], st[0][1]);
        pa[1] = pack2<T>(st[0][2], st[0][3]);
        pa[2] = pack2<T>(st[1][0], st[1][1]);
        pa[3] = pack2<T>(st[1][2], st[1][3]);
        sa[0] = pack2<T>(dpt[0][0], dpt[0][1]);
        sa[1] = pack2<T>(dpt[0][2], dpt[0][3]);
        sa[2] = pack2<T>(dpt[1][0], dpt[1][1]);
        sa[3] = pack2<T>(dpt[1][2], dpt[1][3]);
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int r = qc + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(smem_u32(sG + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(dv[2 * dp], pa, b0, b1);
          mma16816<T>(dv[2 * dp + 1], pa, b2, b3);
          ldsm_x4_t(smem_u32(sQ + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(dk[2 * dp], sa, b0, b1);
          mma16816<T>(dk[2 * dp + 1], sa, b2, b3);
        }
      }
#pragma unroll
      for (int d = 0; d < DT; ++d)
#pragma unroll
        for (int e = 0; e < 4; ++e) dk[d][e] *= g.scale;
      store_rows_c<T, HD>(dv, kt * 16, lane, g.qkv_stride, 2 * C + (int64_t)h * HD, sTok, L, dqkv);
      norm_backward_store<T, HD>(dk, kt * 16, lane, qkv, g.qkv_stride, 1 * C + (int64_t)h * HD, kw,
                                 sRk, sTok, L, dqkv, wk);
    } else {
      // ---------------- phase B: 16 queries -> dQ
      const int qt = task - nt;
      uint32_t qa[KS][4], ga[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int r = qt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32(sQ + r * RS + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
        ldsm_x4(smem_u32(sG + r * RS + c), ga[ks][0], ga[ks][1], ga[ks][2], ga[ks][3]);
      }
      const int qr0 = qt * 16 + gq, qr1 = qr0 + 8;
      const int qlab0 = sLab[qr0], qlab1 = sLab[qr1];
      const float lq0 = sLse[qr0], lq1 = sLse[qr1];
      const float d0 = sD[qr0], d1 = sD[qr1];
      float dq[DT][4];
#pragma unroll
      for (int d = 0; d < DT; ++d) dq[d][0] = dq[d][1] = dq[d][2] = dq[d][3] = 0.f;
      for (int kc = 0; kc < lp; kc += 16) {
        float s[2][4], dpm[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[j][e] = dpm[j][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0, b1, b2, b3;
          const int r = kc + (lane & 7) + (lane >> 4) * 8;
          const int c = ks * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(smem_u32(sK + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(s[0], qa[ks], b0, b1);
          mma16816<T>(s[1], qa[ks], b2, b3);
          ldsm_x4(smem_u32(sV + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(dpm[0], ga[ks], b0, b1);
          mma16816<T>(dpm[1], ga[ks], b2, b3);
        }
        const bool plain = !mixed && kc + 16 <= L;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float v0 = s[j][e] * sl2, v1 = s[j][2 + e] * sl2;
            float p0 = 0.f, p1 = 0.f;
            if (plain) {
              p0 = fast_exp2(v0 - lq0);
              p1 = fast_exp2(v1 - lq1);
            } else {
              const int k = kc + j * 8 + 2 * tq + e;
              const int kl = sLab[k];
              if (kl >= 0) {
                if (kl != (qlab0 < 0 ? 0 : qlab0)) v0 += ml2;
                if (kl != (qlab1 < 0 ? 0 : qlab1)) v1 += ml2;
                p0 = fast_exp2(v0 - lq0);
                p1 = fast_exp2(v1 - lq1);
              }
            }
            s[j][e] = p0 * (dpm[j][e] - d0);
            s[j][2 + e] = p1 * (dpm[j][2 + e] - d1);
          }
        }
        uint32_t sa[4];
        sa[0] = pack2<T>(s[0][0], s[0][1]);
        sa[1] = pack2<T>(s[0][2], s[0][3]);
        sa[2] = pack2<T>(s[1][0], s[1][1]);
        sa[3] = pack2<T>(s[1][2], s[1][3]);
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int r = kc + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(smem_u32(sK + r * RS + c), b0, b1, b2, b3);
          mma16816<T>(dq[2 * dp], sa, b0, b1);
          mma16816<T>(dq[2 * dp + 1], sa, b2, b3);
        }
      }
#pragma unroll
      for (int d = 0; d < DT; ++d)
#pragma unroll
        for (int e = 0; e < 4; ++e) dq[d][e] *= g.scale;
      norm_backward_store<T, HD>(dq, qt * 16, lane, qkv, g.qkv_stride, 0 * C + (int64_t)h * HD, qw,
                                 sRq, sTok, L, dqkv, wq);
    }
  }
  // reduce the norm-weight partials: over the 8 row groups of the warp, then the CTA
#pragma unroll
  for (int i = 0; i < 2 * DT; ++i) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      wq[i] += __shfl_xor_sync(0xffffffffu, wq[i], o);
      wk[i] += __shfl_xor_sync(0xffffffffu, wk[i], o);
    }
  }
  if (gq == 0) {
#pragma unroll
    for (int d = 0; d < DT; ++d) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        atomicAdd(&sWq[d * 8 + 2 * tq + e], wq[2 * d + e]);
        atomicAdd(&sWk[d * 8 + 2 * tq + e], wk[2 * d + e]);
      }
    }
  }
  __syncthreads();
  const int64_t cta = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  for (int i = threadIdx.x; i < HD; i += blockDim.x) {
    dqw_part[cta * HD + i] = sWq[i];
    dkw_part[cta * HD + i] = sWk[i];
  }
}

template <typename T, int HD>
static cudaError_t launch_fwd(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                              const AttnGeom& g, cudaStream_t s) {
  const int L = g.T * g.wh * g.ww;
  const int nqt = (L + 15) / 16;
  const int lk = ((L + 63) / 64) * 64;
  const size_t smem = (size_t)(nqt * 16 + 2 * lk) * (HD + 8) * sizeof(T) + (size_t)lk * (sizeof(int) + 1);
  int nw = nqt < 8 ? nqt : 8;
  if (nw < 1) nw = 1;
  auto k = fwd_kernel<T, HD>;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(g.B * (g.H / g.wh) * (g.W / g.ww), g.nh);
  k<<<grid, nw * 32, smem, s>>>((const T*)qkv, qw, kw, (T*)out, lse, g);
  return cudaGetLastError();
}

template <typename T, int HD>
static cudaError_t launch_bwd(const void* qkv, const float* qw, const float* kw, const void* out,
                              const void* dout, const float* lse, void* dqkv, float* dqw_part,
                              float* dkw_part, const AttnGeom& g, cudaStream_t s) {
  const int L = g.T * g.wh * g.ww;
  const int nt = (L + 15) / 16;
  const int lp = nt * 16;
  const size_t smem = (size_t)4 * lp * (HD + 8) * sizeof(T) + (size_t)4 * lp * sizeof(float) +
                      2 * HD * sizeof(float) + (size_t)lp * (sizeof(int) + 1);
  int nw = 2 * nt < 6 ? 2 * nt : 6;
  auto k = bwd_kernel<T, HD>;
  NSW_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(g.B * (g.H / g.wh) * (g.W / g.ww), g.nh);
  k<<<grid, nw * 32, smem, s>>>((const T*)qkv, qw, kw, (const T*)out, (const T*)dout, lse, (T*)dqkv,
                                dqw_part, dkw_part, g);
  return cudaGetLastError();
}

}  // namespace attn

#define NSW_ATTN_DISPATCH(FN, ...)                                              \
  do {                                                                          \
    if (dtype == kBF16) {                                                       \
      if (g.hd == 64) return attn::FN<__nv_bfloat16, 64>(__VA_ARGS__);          \
      if (g.hd == 32) return attn::FN<__nv_bfloat16, 32>(__VA_ARGS__);          \
      if (g.hd == 16) return attn::FN<__nv_bfloat16, 16>(__VA_ARGS__);          \
      if (g.hd == 128) return attn::FN<__nv_bfloat16, 128>(__VA_ARGS__);        \
    } else if (dtype == kF16) {                                                 \
      if (g.hd == 64) return attn::FN<__half, 64>(__VA_ARGS__);                 \
      if (g.hd == 32) return attn::FN<__half, 32>(__VA_ARGS__);                 \
      if (g.hd == 16) return attn::FN<__half, 16>(__VA_ARGS__);                 \
      if (g.hd == 128) return attn::FN<__half, 128>(__VA_ARGS__);               \
    }                                                                           \
    return cudaErrorInvalidValue;                                               \
  } while (0)

cudaError_t window_attn_fwd(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                            const AttnGeom& g, int dtype, cudaStream_t s) {
  const int L = g.T * g.wh * g.ww;
  if (L > 192 || L <= 0 || g.H % g.wh || g.W % g.ww) return cudaErrorInvalidValue;
  NSW_ATTN_DISPATCH(launch_fwd, qkv, qw, kw, out, lse, g, s);
}

cudaError_t window_attn_bwd(const void* qkv, const float* qw, const float* kw, const void* out,
                            const void* dout, const float* lse, void* dqkv, float* dqw_part,
                            float* dkw_part, const AttnGeom& g, int dtype, cudaStream_t s) {
  const int L = g.T * g.wh * g.ww;
  if (L > 192 || L <= 0 || g.H % g.wh || g.W % g.ww) return cudaErrorInvalidValue;
  NSW_ATTN_DISPATCH(launch_bwd, qkv, qw, kw, out, dout, lse, dqkv, dqw_part, dkw_part, g, s);
}

}  // namespace nsw
