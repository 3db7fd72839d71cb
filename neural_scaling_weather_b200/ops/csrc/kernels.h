// Host-side launch interface of the sm_100a kernels (no torch types; raw pointers).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nsw {

enum DType : int { kBF16 = 0, kF16 = 1, kF32 = 2 };

int* device_error_flag();  // per-device error word (lazily allocated)

// ---- norms -------------------------------------------------------------------
cudaError_t rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n,
                        float eps, int dtype, cudaStream_t s);
cudaError_t rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                        float* dw_partial, int partial_rows, int64_t rows, int n, int dtype,
                        cudaStream_t s, float eps = -1.f, const void* add = nullptr);

// ---- elementwise epilogues -----------------------------------------------------
// y = act(acc + bias) + residual (residual row index = row % res_period)
cudaError_t bias_act_residual(const void* acc, int acc_dtype, const float* bias, const void* residual,
                              int64_t res_period, void* y, void* preact, int64_t rows, int n,
                              int act, int dtype, cudaStream_t s);
cudaError_t gelu_bwd(const void* dy, const void* u, void* du, int64_t n, int dtype, cudaStream_t s);
// column sums of a [rows, n] matrix in fp32 (deterministic two-pass)
// out_b[:] (+)= sum over rows of part[b, :, :] (fp32, rows in order); out_b = out + b * n, except
// out_1 = out1 when given (separate destinations, e.g. two parameters' gradients); accumulate adds
// to the destination instead of overwriting it
cudaError_t sum_rows(const float* part, int64_t batches, int64_t rows, int64_t n, float* out, cudaStream_t s,
                     bool accumulate = false, float* out1 = nullptr);
cudaError_t col_sum(const void* x, float* out, float* partial, int partial_rows, int64_t rows, int n,
                    int dtype, cudaStream_t s);

// ---- patch embed / head layout ------------------------------------------------
cudaError_t im2col_patch(const void* x, int x_dtype, void* cols, int N, int C, int H, int W, int p,
                         int dtype, cudaStream_t s);
cudaError_t col2im_patch(const void* dcols, void* dx, int x_dtype, int N, int C, int H, int W, int p,
                         int dtype, cudaStream_t s);
cudaError_t unpatchify(const void* y2, void* out, int BT, int h, int w, int p, int C, int dtype,
                       cudaStream_t s);
cudaError_t patchify(const void* dout, void* dy2, int BT, int h, int w, int p, int C, int dtype,
                     cudaStream_t s);

// ---- losses ----------------------------------------------------------------------
cudaError_t weighted_sse(const void* x, int x_dtype, const void* y, int y_dtype, const float* area_w,
                         const float* ch_w, float* partial, int partial_n, float* out, int64_t lead,
                         int C, int H, int W, cudaStream_t s);
cudaError_t weighted_sse_bwd(const void* x, int x_dtype, const void* y, int y_dtype,
                             const float* area_w, const float* ch_w, const float* gscale, void* dx,
                             int64_t lead, int C, int H, int W, cudaStream_t s);
cudaError_t weighted_se_per_plane(const void* x, int x_dtype, const void* y, int y_dtype,
                                  const float* area_w, float* out, int64_t planes, int H, int W,
                                  cudaStream_t s);

// ---- optimizer -----------------------------------------------------------------
cudaError_t adamw_step(float* p, const float* g, float* m, float* v, void* shadow, int shadow_dtype,
                       const float* gscale, const int* skip, int64_t n, float lr, float b1, float b2,
                       float eps, float wd, float bc1, float bc2, bool decoupled, cudaStream_t s);
cudaError_t segment_sumsq(const float* x, const int64_t* block_lo, const int64_t* block_hi,
                          const int* block_cls, int nblocks, int ncls, float* partial, float* out,
                          cudaStream_t s);

// ---- window attention ------------------------------------------------------------
struct AttnGeom {
  int B, T, H, W;      // token grid (local)
  int nh, hd;          // local heads, head dim
  int wh, ww;          // window
  int sh, sw;          // index shift
  int mask, mask_shift, row_offset, h_global;
  float scale;
  int64_t qkv_stride;  // elements between consecutive tokens in qkv (3*nh*hd)
  int64_t out_stride;  // elements between tokens in out / dout (nh*hd)
};
cudaError_t window_attn_fwd(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                            const AttnGeom& g, int dtype, cudaStream_t s);
// tcgen05/TMEM forward (bf16, head_dim 64, T*wh*ww <= 176); same outputs as window_attn_fwd
bool window_attn_fwd_tc_supported(const AttnGeom& g, int dtype);
cudaError_t window_attn_fwd_tc(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                               const AttnGeom& g, cudaStream_t s);
// warp-specialised tcgen05 forward (same contract and support as window_attn_fwd_tc)
cudaError_t window_attn_fwd_ws(const void* qkv, const float* qw, const float* kw, void* out, float* lse,
                               const AttnGeom& g, cudaStream_t s, long long* stamps = nullptr);
// RMSNorm, one warp per row with the row in registers (n <= 2048); rmsnorm_fwd/bwd use the TMA
// version below where it applies and these otherwise
cudaError_t rmsnorm_fwd_rows(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n,
                             float eps, int dtype, cudaStream_t s);
cudaError_t rmsnorm_bwd_rows(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                             float* dw_partial, int partial_rows, int64_t rows, int n, int dtype,
                             cudaStream_t s);
// RMSNorm with TMA bulk-copy row tiles (16-bit types, n % 8 == 0, n <= 4096)
bool rmsnorm_tma_supported(int64_t rows, int n, int dtype);
cudaError_t rmsnorm_fwd_tma(const void* x, const float* w, void* y, float* rstd, int64_t rows, int n, float eps,
                            int dtype, int grid, cudaStream_t s);
// eps >= 0: rstd is recomputed from x (as the forward computed it); eps < 0: read from rstd
cudaError_t rmsnorm_bwd_tma(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dw_partial, int partial_rows, int64_t rows, int n, int dtype, float eps,
                            cudaStream_t s, const void* add = nullptr);  // add: optional [rows, n] added to dx
// dqw_part / dkw_part: one row of head_dim partial sums per CTA, min(items, SM count) rows
cudaError_t window_attn_bwd_tc(const void* qkv, const float* qw, const float* kw, const void* out,
                               const void* dout, const float* lse, void* dqkv, float* dqw_part, float* dkw_part,
                               const AttnGeom& g, cudaStream_t s, long long* stamps = nullptr);
cudaError_t window_attn_bwd(const void* qkv, const float* qw, const float* kw, const void* out,
                            const void* dout, const float* lse, void* dqkv, float* dqw_part,
                            float* dkw_part, const AttnGeom& g, int dtype, cudaStream_t s);

// ---- tcgen05 GEMM ----------------------------------------------------------------
struct GemmArgs {
  const void* A;        // [M, K] row-major (K contiguous)
  const void* B;        // [N, K] row-major (K contiguous)
  void* D;              // [M, N] row-major output (ldd elements)
  int64_t M, N, K;
  int64_t lda, ldb, ldd;
  const float* bias;    // [N] or null
  const void* residual; // [*, N] (ldr) or null; row index = m % res_period
  int64_t ldr, res_period;
  void* preact;         // optional [M, N] pre-activation output (ldd)
  int act;              // 0 none, 1 gelu, 2 * gelu'(residual), 3 gelu + gelu'(u) as preact, 4 * residual
  int dtype;            // kBF16 / kF16 (A, B, D, residual, preact)
  int out_f32;          // D in fp32 instead of dtype
  float alpha;
  int accumulate;       // D += result (fp32 output only)
  // tensor-parallel all-reduce fused into the epilogue (ar_world > 1): ar_part[r] / ar_flags[r]
  // are rank r's symmetric partial buffer (ar_world slots of [M, N] in dtype, slot s receiving
  // rank s's partial) and flag words (peer pointers)
  int ar_world;
  int ar_rank;
  void* ar_part[8];
  uint32_t* ar_flags[8];
  // optional (nullptr: off): %globaltimer stamps of the fused all-reduce epilogue's phases, eight per
  // tile for the first 32 tiles of CTAs 0..3, at [(cta * 32 + i) * 8 + phase]
  long long* ar_stamps;
};
cudaError_t gemm_tcgen05(const GemmArgs& a, cudaStream_t s, int impl = 0);
int gemm_tcgen05_supported(const GemmArgs& a);

// Weight (and bias) gradient of a linear layer on the tensor cores:
//   D[m, n] (+)= sum_t dy[t, m] * x[t, n]   (fp32),   db[m] (+)= sum_t dy[t, m]   (fp32)
// dy [T, M] and x [T, N] token-major (features contiguous, leading dimensions ldy / ldx).
// D and db may be split into up to four row segments of seg_rows rows (separate buffers, e.g. the
// q / k / v weights of a fused projection); seg_rows = 0 means one segment of M rows.
struct WgradArgs {
  const void* dy;
  int64_t ldy;
  const void* x;
  int64_t ldx;
  int64_t T, M, N;
  float* D[4];
  int64_t ldd;
  int64_t seg_rows;
  int accumulate;
  float* db[4];  // db[0] null: no bias gradient
  int db_accumulate;
  int dtype;
  float* ws;   // wgrad_workspace_floats(M, N, plan) floats (none needed when that is 0)
  int splits;  // set from the plan
  int k1;      // set from the plan
};
// Work schedule: `splits` k-splits (uniform), or with k1 > 0 the balanced schedule (each tile's first
// k1 k-blocks on a pair of its own, the rest in `splits` pieces on the remaining pairs); `pairs` is
// the number of CTA pairs it was planned for.
struct WgradPlan {
  int splits, k1, pairs;
};
WgradPlan wgrad_plan(int64_t M, int64_t N, int64_t T);
int64_t wgrad_workspace_floats(int64_t M, int64_t N, const WgradPlan& plan);
int wgrad_tcgen05_supported(const WgradArgs& a);
cudaError_t wgrad_tcgen05(const WgradArgs& a, const WgradPlan& plan, cudaStream_t s);

// Data-parallel reduction / sharded AdamW over peer memory (dp_fused.cu).  Every rank's buffers:
// grad / data fp32 flat buffers, shadow 16-bit (or null), flags uint32 [kDpFlagBase + world * slots]
// (flag word of (rank r, slot) at kDpFlagBase + r * slots + slot in every rank's array).
constexpr int kDpFlagBase = 16;
struct DpPeers {
  float* grad[8];
  float* data[8];
  void* shadow[8];
  uint32_t* flags[8];
  int world, rank, slots;
};
cudaError_t dp_reduce(const DpPeers& pr, int slot, uint32_t epoch, int64_t lo, int64_t hi, float scale,
                      cudaStream_t s);
cudaError_t dp_adamw(const DpPeers& pr, const int64_t* rlo, const int64_t* rhi, const int64_t* rstart, int nranges,
                     int64_t total4, float* m, float* v, int shadow_dtype, const float* gscale, const int* skip,
                     float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, bool decoupled,
                     cudaStream_t s);
cudaError_t dp_barrier(const DpPeers& pr, int slot, uint32_t epoch, cudaStream_t s);

// Cyclic roll of a (B*T, H_l, W_l, C) activation sharded over an n1 x n2 (sp1 x sp2) grid of one node's
// GPUs (halo_roll.cu): band buffers and flag words in symmetric memory, one entry per group rank.
// Flag words of each rank: [kHaloEpoch] rolls completed, [kHaloPackCount] / [kHaloDoneCount] block
// counters, [kHaloReady + r] / [kHaloAck + r] the last epoch rank r published.
constexpr int kHaloEpoch = 0, kHaloPackCount = 1, kHaloDoneCount = 2, kHaloReady = 16, kHaloAck = 32;
constexpr int kHaloFlagWords = 48;
struct HaloArgs {
  const void* x;
  void* out;
  void* band[8];
  uint32_t* flags[8];
  int world, rank, n1, n2;
  int coord1[8], coord2[8];  // (sp1, sp2) shard of each group rank
  int grid_rank[8];          // group rank holding shard (i, j), at i * n2 + j
  int h_off[9], w_off[9];    // shard offsets along H (n1 + 1 entries) and W (n2 + 1)
  int bt, row_vec, sh, sw;   // B*T, 16-byte vectors per row of C elements, shifts along H and W
};
int64_t halo_band_bytes(const HaloArgs& a, int shard);
cudaError_t halo_roll(const HaloArgs& a, cudaStream_t s);

// Legendre part of the real SHT (sht.cu): table P[m, l, k] = w_k Pbar_l^m(x_k) for orders
// m0 .. m0 + m_count - 1 (packed: order index mi's rows l = m .. L-1 start at row row_off[mi]),
// and the batched contractions C[mi, l, :] = sum_k P F[mi, k, :] / dF[mi, k, :] = sum_l P dC[mi, l, :].
cudaError_t legendre_table(const double* x, const double* w, int m0, int m_count, int L, int K,
                           const int64_t* row_off, float* P, int csphase, cudaStream_t s);
cudaError_t legendre_fwd(const float* P, const int64_t* row_off, const float* F, float* C, int m0, int m_count, int L,
                         int K, int N, cudaStream_t s);
cudaError_t legendre_bwd(const float* P, const int64_t* row_off, const float* dC, float* dF, int m0, int m_count, int L,
                         int K, int N, cudaStream_t s);

}  // namespace nsw
