#include <cstdlib>
// PyTorch bindings of the sm_100a kernels: argument checks, output allocation and the
// current CUDA stream; the kernels themselves live in the .cu files (no torch headers).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "kernels.h"

namespace {

using torch::Tensor;

int dt_code(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return nsw::kBF16;
    case at::kHalf: return nsw::kF16;
    case at::kFloat: return nsw::kF32;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

at::ScalarType scalar_of(int code) {
  return code == nsw::kBF16 ? at::kBFloat16 : (code == nsw::kF16 ? at::kHalf : at::kFloat);
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

void need_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

const float* opt_f32(const c10::optional<Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->is_cuda(), "expected fp32 CUDA tensor");
  return t->data_ptr<float>();
}

// ------------------------------------------------------------------------------ misc
int read_error_flag(bool clear) {
  int* f = nsw::device_error_flag();
  int v = 0;
  check(cudaMemcpy(&v, f, sizeof(int), cudaMemcpyDeviceToHost), "read_error_flag");
  if (clear && v) check(cudaMemset(f, 0, sizeof(int)), "clear_error_flag");
  return v;
}

// The device error word as a one-element int32 tensor (a view: no copy, not owned), so the
// host can read it with an asynchronous copy alongside other per-step results.
Tensor error_word() {
  int dev = 0;
  check(cudaGetDevice(&dev), "cudaGetDevice");
  int* f = nsw::device_error_flag();
  TORCH_CHECK(f != nullptr, "device error word unavailable");
  return torch::from_blob(f, {1}, torch::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
}

// Writes a code into the device error word (what a kernel does when a bounded wait runs
// out); lets tests check that the host-side checks stop a run without any kernel failing.
void set_error_flag(int code) {
  int* f = nsw::device_error_flag();
  check(cudaMemcpy(f, &code, sizeof(int), cudaMemcpyHostToDevice), "set_error_flag");
}

// ------------------------------------------------------------------------------ norms
std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor w, double eps) {
  need_cuda(x, "x");
  need_cuda(w, "w");
  const int n = (int)x.size(-1);
  const int64_t rows = x.numel() / n;
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  check(nsw::rmsnorm_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), rows,
                         n, (float)eps, dt_code(x), stream()),
        "rmsnorm_fwd");
  return {y, rstd};
}

// eps >= 0: the kernel recomputes rstd from x with this eps (the forward's value); else it reads rstd
// add (optional, [rows, n] like x): added to dx in the same pass (skip-connection gradient)
// dw_into (optional, fp32 [n] contiguous): the weight gradient is added into it (the optimizer's gradient
// buffer) and returned; otherwise a fresh tensor
std::vector<Tensor> rmsnorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor rstd, double eps, c10::optional<Tensor> add,
                                c10::optional<Tensor> dw_into) {
  need_cuda(dy, "dy");
  need_cuda(x, "x");
  const int n = (int)x.size(-1);
  const int64_t rows = x.numel() / n;
  auto dx = torch::empty_like(x);
  const bool fused_add = add.has_value() && nsw::rmsnorm_tma_supported(rows, n, dt_code(x));
  if (add) TORCH_CHECK(add->is_contiguous() && add->scalar_type() == x.scalar_type() && add->numel() == x.numel(),
                       "rmsnorm_bwd: add must be a contiguous tensor like x");
  // one partial weight-gradient row per CTA: one persistent CTA per SM for the TMA kernel
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  int parts = nsw::rmsnorm_tma_supported(rows, n, dt_code(x)) ? sms : 3 * sms;
  if (rows < parts * 8) parts = (int)std::max<int64_t>(1, (rows + 7) / 8);
  auto part = torch::empty({parts, n}, x.options().dtype(at::kFloat));
  check(nsw::rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(),
                         dx.data_ptr(), part.data_ptr<float>(), parts, rows, n, dt_code(x), stream(), (float)eps,
                         fused_add ? add->data_ptr() : nullptr),
        "rmsnorm_bwd");
  if (add && !fused_add) dx.add_(*add);
  if (dw_into)
    TORCH_CHECK(dw_into->is_cuda() && dw_into->scalar_type() == at::kFloat && dw_into->is_contiguous() &&
                    dw_into->numel() == n,
                "rmsnorm_bwd: dw_into must be a contiguous fp32 CUDA tensor of n elements");
  auto dw = dw_into ? *dw_into : torch::empty({(int64_t)n}, x.options().dtype(at::kFloat));
  check(nsw::sum_rows(part.data_ptr<float>(), 1, parts, n, dw.data_ptr<float>(), stream(), dw_into.has_value()),
        "sum_rows");
  return {dx, dw};
}

// ------------------------------------------------------------------------------ GEMM + all-reduce
// D = sum over the ranks of A_r B_r^T (+ bias + residual), the reduction done in the GEMM's
// epilogue over NVLink peer memory.  part_ptrs / flag_ptrs: every rank's symmetric partial
// buffer (one [M, N] slot per rank: >= W * M * N elements of A's dtype) and flag words, in rank
// order; rank: this rank.
Tensor gemm_allreduce(Tensor A, Tensor B, c10::optional<Tensor> bias, c10::optional<Tensor> residual,
                      std::vector<int64_t> part_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                      c10::optional<Tensor> stamps) {
  need_cuda(A, "A");
  need_cuda(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_allreduce: A [M,K], B [N,K]");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous(), "gemm_allreduce: contiguous operands");
  TORCH_CHECK(part_ptrs.size() == flag_ptrs.size() && part_ptrs.size() >= 2 && part_ptrs.size() <= 8,
              "gemm_allreduce: 2..8 ranks");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  auto D = torch::empty({M, N}, A.options());
  nsw::GemmArgs g{};
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.D = D.data_ptr();
  g.M = M;
  g.N = N;
  g.K = K;
  g.lda = K;
  g.ldb = K;
  g.ldd = N;
  g.alpha = 1.f;
  g.dtype = dt_code(A);
  g.res_period = M;
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N, "gemm_allreduce: fp32 bias [N]");
    g.bias = bias->data_ptr<float>();
  }
  if (residual) {
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == M * N && residual->scalar_type() == A.scalar_type(),
                "gemm_allreduce: residual [M, N] in A's dtype");
    g.residual = residual->data_ptr();
    g.ldr = N;
  }
  g.ar_world = (int)part_ptrs.size();
  g.ar_rank = (int)rank;
  for (int r = 0; r < g.ar_world; ++r) {
    g.ar_part[r] = reinterpret_cast<void*>(part_ptrs[r]);
    g.ar_flags[r] = reinterpret_cast<uint32_t*>(flag_ptrs[r]);
  }
  if (stamps) {
    TORCH_CHECK(stamps->is_cuda() && stamps->scalar_type() == at::kLong && stamps->numel() >= 4 * 32 * 8,
                "gemm_allreduce: stamps must be an int64 CUDA tensor of >= 1024 elements");
    g.ar_stamps = reinterpret_cast<long long*>(stamps->data_ptr<int64_t>());
  }
  TORCH_CHECK(nsw::gemm_tcgen05_supported(g), "gemm_allreduce: shape/alignment not supported");
  check(nsw::gemm_tcgen05(g, stream(), 1), "gemm_allreduce");
  return D;
}

// ------------------------------------------------------------------------------ GEMM
Tensor gemm(Tensor A, Tensor B, c10::optional<Tensor> bias, c10::optional<Tensor> residual,
            int64_t res_period, int64_t act, c10::optional<Tensor> preact, bool out_f32, double alpha,
            c10::optional<Tensor> out, bool accumulate, int64_t impl) {
  need_cuda(A, "A");
  need_cuda(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm: A [M,K], B [N,K]");
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "gemm: A and B must share a dtype");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous(), "gemm: A and B must be contiguous");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  const auto out_type = out_f32 ? at::kFloat : A.scalar_type();
  Tensor D;
  if (out.has_value() && out->defined()) {
    D = *out;
    need_cuda(D, "out");
    // the kernel writes M x N elements with leading dimension N from D's first element
    TORCH_CHECK(D.dim() == 2 && D.size(0) == M && D.size(1) == N && D.is_contiguous(),
                "gemm: out must be a contiguous [M, N] tensor");
    TORCH_CHECK(D.scalar_type() == out_type, "gemm: out dtype must be fp32 with out_f32, else A's dtype");
  } else {
    D = torch::empty({M, N}, A.options().dtype(out_f32 ? at::kFloat : A.scalar_type()));
  }
  nsw::GemmArgs g{};
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.D = D.data_ptr();
  g.M = M;
  g.N = N;
  g.K = K;
  g.lda = K;
  g.ldb = K;
  g.ldd = N;
  g.bias = opt_f32(bias);
  if (residual.has_value() && residual->defined()) {
    need_cuda(*residual, "residual");
    TORCH_CHECK(residual->scalar_type() == A.scalar_type(), "residual dtype");
    g.res_period = res_period > 0 ? res_period : M;
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == g.res_period * N,
                "gemm: residual must be a contiguous [res_period (or M), N] tensor");
    g.residual = residual->data_ptr();
    g.ldr = N;
  }
  if (preact.has_value() && preact->defined()) {
    need_cuda(*preact, "preact");
    TORCH_CHECK(preact->is_contiguous() && preact->numel() == M * N && preact->scalar_type() == A.scalar_type(),
                "gemm: preact must be a contiguous [M, N] tensor of A's dtype");
    g.preact = preact->data_ptr();
  }
  TORCH_CHECK(!g.bias || bias->numel() == N, "gemm: bias must have N elements");
  g.act = (int)act;
  g.dtype = dt_code(A);
  g.out_f32 = out_f32 ? 1 : 0;
  g.alpha = (float)alpha;
  g.accumulate = accumulate ? 1 : 0;
  TORCH_CHECK(nsw::gemm_tcgen05_supported(g), "gemm: shape/alignment not supported by the tcgen05 kernel");
  check(nsw::gemm_tcgen05(g, stream(), (int)impl), "gemm_tcgen05");
  return D;
}

bool gemm_supported(Tensor A, Tensor B, bool out_f32) {
  nsw::GemmArgs g{};
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.D = A.data_ptr();
  g.M = A.size(0);
  g.N = B.size(0);
  g.K = A.size(1);
  g.lda = A.stride(0);
  g.ldb = B.stride(0);
  g.ldd = B.size(0);
  g.dtype = dt_code(A);
  g.out_f32 = out_f32;
  return A.is_contiguous() && B.is_contiguous() && nsw::gemm_tcgen05_supported(g);
}

std::vector<Tensor> bias_act_residual(Tensor acc, c10::optional<Tensor> bias, c10::optional<Tensor> residual,
                                      int64_t res_period, int64_t act, bool want_preact, int64_t out_dtype) {
  need_cuda(acc, "acc");
  const int n = (int)acc.size(-1);
  const int64_t rows = acc.numel() / n;
  auto y = torch::empty(acc.sizes(), acc.options().dtype(scalar_of((int)out_dtype)));
  Tensor pre;
  if (want_preact) pre = torch::empty_like(y);
  const void* res = nullptr;
  if (residual.has_value() && residual->defined()) {
    need_cuda(*residual, "residual");
    res = residual->data_ptr();
  }
  check(nsw::bias_act_residual(acc.data_ptr(), dt_code(acc), opt_f32(bias), res, res_period,
                               y.data_ptr(), want_preact ? pre.data_ptr() : nullptr, rows, n, (int)act,
                               (int)out_dtype, stream()),
        "bias_act_residual");
  return {y, pre};
}

Tensor gelu_bwd(Tensor dy, Tensor u) {
  need_cuda(dy, "dy");
  need_cuda(u, "u");
  auto du = torch::empty_like(u);
  check(nsw::gelu_bwd(dy.data_ptr(), u.data_ptr(), du.data_ptr(), u.numel(), dt_code(u), stream()),
        "gelu_bwd");
  return du;
}

// Weight gradient D (+)= dy^T x (fp32 [M, N]) and optionally the bias gradient db (+)= colsum(dy)
// (fp32 [M]) on the tensor cores.  dy [T, M] and x [T, N] may be column slices (row stride >= width,
// unit column stride).  `out` / `db` (fp32, contiguous) are written, or accumulated into.
bool wgrad_supported(const Tensor& dy, const Tensor& x) {
  if (!dy.is_cuda() || !x.is_cuda() || dy.dim() != 2 || x.dim() != 2 || dy.scalar_type() != x.scalar_type())
    return false;
  if (dy.stride(1) != 1 || x.stride(1) != 1 || dy.size(0) != x.size(0)) return false;
  nsw::WgradArgs a{};
  a.dy = dy.data_ptr();
  a.ldy = dy.stride(0);
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.T = dy.size(0);
  a.M = dy.size(1);
  a.N = x.size(1);
  a.D[0] = reinterpret_cast<float*>(16);  // placeholder: only the operands are checked here
  a.ldd = a.N;
  a.dtype = dt_code(dy);
  return nsw::wgrad_tcgen05_supported(a) != 0;
}

static void check_f32_out(const Tensor& t, int64_t numel, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == numel &&
                  (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "wgrad: ", what, " must be a contiguous, 16-byte aligned fp32 tensor of ", numel, " elements");
}

// dy's M columns form len(outs) equal row segments of dW: segment i (M / len(outs) rows) goes to
// outs[i] (and its feature sums to dbs[i]).  Returns outs.
std::vector<Tensor> wgrad_segments(Tensor dy, Tensor x, std::vector<Tensor> outs, bool accumulate,
                                   c10::optional<std::vector<Tensor>> dbs, bool db_accumulate) {
  TORCH_CHECK(wgrad_supported(dy, x), "wgrad: unsupported operands (bf16/fp16 [T, M] and [T, N] with unit column "
                                      "stride, row strides multiples of 8, 16-byte aligned)");
  const int64_t T = dy.size(0), M = dy.size(1), N = x.size(1);
  const int nseg = (int)outs.size();
  TORCH_CHECK(nseg >= 1 && nseg <= 4 && M % nseg == 0, "wgrad: 1 to 4 equal row segments");
  const int64_t seg = M / nseg;
  nsw::WgradArgs a{};
  for (int i = 0; i < nseg; ++i) {
    check_f32_out(outs[i], seg * N, "out");
    a.D[i] = outs[i].data_ptr<float>();
  }
  if (dbs.has_value()) {
    TORCH_CHECK((int)dbs->size() == nseg, "wgrad: one db per segment");
    for (int i = 0; i < nseg; ++i) {
      check_f32_out((*dbs)[i], seg, "db");
      a.db[i] = (*dbs)[i].data_ptr<float>();
    }
  }
  a.dy = dy.data_ptr();
  a.ldy = dy.stride(0);
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.T = T;
  a.M = M;
  a.N = N;
  a.ldd = N;
  a.seg_rows = seg;
  a.accumulate = accumulate ? 1 : 0;
  a.db_accumulate = db_accumulate ? 1 : 0;
  a.dtype = dt_code(dy);
  const nsw::WgradPlan plan = nsw::wgrad_plan(M, N, T);
  Tensor ws;
  const int64_t wsn = nsw::wgrad_workspace_floats(M, N, plan);
  if (wsn > 0) {
    ws = torch::empty({wsn}, dy.options().dtype(at::kFloat));
    a.ws = ws.data_ptr<float>();
  }
  check(nsw::wgrad_tcgen05(a, plan, stream()), "wgrad_tcgen05");
  return outs;
}

Tensor wgrad(Tensor dy, Tensor x, c10::optional<Tensor> out, bool accumulate, c10::optional<Tensor> db,
             bool db_accumulate) {
  const int64_t M = dy.size(1), N = x.size(1);
  Tensor D;
  if (out.has_value() && out->defined()) {
    D = *out;
  } else {
    TORCH_CHECK(!accumulate, "wgrad: accumulate needs out");
    D = torch::empty({M, N}, dy.options().dtype(at::kFloat));
  }
  c10::optional<std::vector<Tensor>> dbs;
  if (db.has_value() && db->defined()) dbs = std::vector<Tensor>{*db};
  wgrad_segments(dy, x, {D.view({-1})}, accumulate, dbs, db_accumulate);
  return D.view({M, N});
}

std::vector<int64_t> wgrad_plan(int64_t M, int64_t N, int64_t T) {
  const nsw::WgradPlan p = nsw::wgrad_plan(M, N, T);
  return {p.splits, p.k1, p.pairs};
}

// ------------------------------------------------------------------------------ data-parallel fused path
static nsw::DpPeers dp_peers(const std::vector<int64_t>& grad, const std::vector<int64_t>& data,
                             const std::vector<int64_t>& shadow, const std::vector<int64_t>& flags, int64_t rank,
                             int64_t slots) {
  const int world = (int)grad.size();
  TORCH_CHECK(world >= 1 && world <= 8 && (int)data.size() == world && (int)flags.size() == world &&
                  (shadow.empty() || (int)shadow.size() == world) && rank >= 0 && rank < world,
              "dp: 1..8 ranks with one pointer each");
  nsw::DpPeers pr{};
  for (int r = 0; r < world; ++r) {
    pr.grad[r] = reinterpret_cast<float*>(grad[r]);
    pr.data[r] = reinterpret_cast<float*>(data[r]);
    pr.shadow[r] = shadow.empty() ? nullptr : reinterpret_cast<void*>(shadow[r]);
    pr.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
    TORCH_CHECK((grad[r] & 15) == 0 && (data[r] & 15) == 0 && (shadow.empty() || (shadow[r] & 7) == 0),
                "dp: buffers must be 16-byte aligned");
  }
  pr.world = world;
  pr.rank = (int)rank;
  pr.slots = (int)slots;
  return pr;
}

void dp_reduce(std::vector<int64_t> grad, std::vector<int64_t> data, std::vector<int64_t> shadow,
               std::vector<int64_t> flags, int64_t rank, int64_t slots, int64_t slot, int64_t epoch, int64_t lo,
               int64_t hi, double scale) {
  const auto pr = dp_peers(grad, data, shadow, flags, rank, slots);
  check(nsw::dp_reduce(pr, (int)slot, (uint32_t)epoch, lo, hi, (float)scale, stream()), "dp_reduce");
}

void dp_adamw(std::vector<int64_t> grad, std::vector<int64_t> data, std::vector<int64_t> shadow,
              std::vector<int64_t> flags, int64_t rank, int64_t slots, Tensor rlo, Tensor rhi, Tensor rstart,
              int64_t total4, Tensor m, Tensor v, int64_t shadow_dtype, Tensor gscale, Tensor skip, double lr,
              double b1, double b2, double eps, double wd, double bc1, double bc2, bool decoupled) {
  const auto pr = dp_peers(grad, data, shadow, flags, rank, slots);
  TORCH_CHECK(rlo.scalar_type() == at::kLong && rhi.scalar_type() == at::kLong && rstart.scalar_type() == at::kLong &&
                  rlo.is_cuda() && rlo.numel() == rhi.numel() && rlo.numel() == rstart.numel(),
              "dp_adamw: int64 CUDA range tables");
  need_cuda(m, "m");
  need_cuda(v, "v");
  check(nsw::dp_adamw(pr, rlo.data_ptr<int64_t>(), rhi.data_ptr<int64_t>(), rstart.data_ptr<int64_t>(),
                      (int)rlo.numel(), total4, m.data_ptr<float>(), v.data_ptr<float>(), (int)shadow_dtype,
                      gscale.data_ptr<float>(), skip.data_ptr<int>(), (float)lr, (float)b1, (float)b2, (float)eps,
                      (float)wd, (float)bc1, (float)bc2, decoupled, stream()),
        "dp_adamw");
}

void dp_barrier(std::vector<int64_t> grad, std::vector<int64_t> data, std::vector<int64_t> shadow,
                std::vector<int64_t> flags, int64_t rank, int64_t slots, int64_t slot, int64_t epoch) {
  const auto pr = dp_peers(grad, data, shadow, flags, rank, slots);
  check(nsw::dp_barrier(pr, (int)slot, (uint32_t)epoch, stream()), "dp_barrier");
}

// ------------------------------------------------------------------------------ sharded roll (halo)
// x, out: contiguous (..., H_l, W_l, C) CUDA tensors of this rank's shard; C * element size a multiple of
// 16 bytes.  geom = [n1, n2, sh, sw, rank]; h_off / w_off: shard offsets (n1 + 1 / n2 + 1 entries);
// coord1 / coord2: shard of each group rank; band / flags: every group rank's symmetric buffers.
static nsw::HaloArgs halo_args(const Tensor& x, const Tensor& out, std::vector<int64_t> geom,
                               std::vector<int64_t> h_off, std::vector<int64_t> w_off, std::vector<int64_t> coord1,
                               std::vector<int64_t> coord2, std::vector<int64_t> band, std::vector<int64_t> flags) {
  TORCH_CHECK(geom.size() == 5, "halo_roll: geom = [n1, n2, sh, sw, rank]");
  nsw::HaloArgs a{};
  a.n1 = (int)geom[0];
  a.n2 = (int)geom[1];
  a.sh = (int)geom[2];
  a.sw = (int)geom[3];
  a.rank = (int)geom[4];
  a.world = (int)band.size();
  TORCH_CHECK(a.world >= 2 && a.world <= 8 && a.n1 * a.n2 == a.world && (int)flags.size() == a.world &&
                  (int)coord1.size() == a.world && (int)coord2.size() == a.world &&
                  (int)h_off.size() == a.n1 + 1 && (int)w_off.size() == a.n2 + 1 && a.rank >= 0 && a.rank < a.world,
              "halo_roll: inconsistent group description");
  for (int i = 0; i < 8; ++i) a.grid_rank[i] = -1;
  for (int r = 0; r < a.world; ++r) {
    a.band[r] = reinterpret_cast<void*>(band[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
    a.coord1[r] = (int)coord1[r];
    a.coord2[r] = (int)coord2[r];
    TORCH_CHECK(a.coord1[r] >= 0 && a.coord1[r] < a.n1 && a.coord2[r] >= 0 && a.coord2[r] < a.n2,
                "halo_roll: shard coordinate out of range");
    a.grid_rank[a.coord1[r] * a.n2 + a.coord2[r]] = r;
  }
  for (int i = 0; i < a.n1 * a.n2; ++i) TORCH_CHECK(a.grid_rank[i] >= 0, "halo_roll: a shard has no rank");
  for (int i = 0; i <= a.n1; ++i) a.h_off[i] = (int)h_off[i];
  for (int j = 0; j <= a.n2; ++j) a.w_off[j] = (int)w_off[j];
  need_cuda(x, "x");
  need_cuda(out, "out");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.sizes() == out.sizes() &&
                  x.scalar_type() == out.scalar_type() && x.dim() >= 3,
              "halo_roll: x and out contiguous (..., H_l, W_l, C) of one shape and dtype");
  const int64_t rowb = x.size(-1) * x.element_size();
  TORCH_CHECK(rowb % 16 == 0, "halo_roll: C * element size must be a multiple of 16 bytes");
  const int i1 = a.coord1[a.rank], i2 = a.coord2[a.rank];
  TORCH_CHECK(x.size(-3) == a.h_off[i1 + 1] - a.h_off[i1] && x.size(-2) == a.w_off[i2 + 1] - a.w_off[i2],
              "halo_roll: x is not this rank's shard");
  a.x = x.data_ptr();
  a.out = out.data_ptr();
  a.row_vec = (int)(rowb / 16);
  a.bt = (int)(x.numel() / (x.size(-3) * x.size(-2) * x.size(-1)));
  return a;
}

int64_t halo_band_bytes(Tensor x, std::vector<int64_t> geom, std::vector<int64_t> h_off, std::vector<int64_t> w_off,
                        std::vector<int64_t> coord1, std::vector<int64_t> coord2) {
  // size of the largest band buffer any rank of the group needs (no pointers involved)
  std::vector<int64_t> fake(coord1.size(), 16);
  int64_t best = 0;
  const auto a = halo_args(x, x, geom, h_off, w_off, coord1, coord2, fake, fake);
  for (int r = 0; r < a.world; ++r) best = std::max(best, nsw::halo_band_bytes(a, r));
  return best;
}

void halo_roll(Tensor x, Tensor out, std::vector<int64_t> geom, std::vector<int64_t> h_off,
               std::vector<int64_t> w_off, std::vector<int64_t> coord1, std::vector<int64_t> coord2,
               std::vector<int64_t> band, std::vector<int64_t> flags) {
  const auto a = halo_args(x, out, geom, h_off, w_off, coord1, coord2, band, flags);
  check(nsw::halo_roll(a, stream()), "halo_roll");
}

// ------------------------------------------------------------------------------ SHT (Legendre part)
// x, w: float64 [K] (this rank's colatitude nodes and quadrature weights); orders m0 .. m0 + m_count - 1;
// returns (P packed float32 [rows, K], row_off int64 [m_count]).
std::vector<Tensor> legendre_table(Tensor x, Tensor w, int64_t m0, int64_t m_count, int64_t L, bool csphase) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kDouble && w.scalar_type() == at::kDouble &&
                  x.is_contiguous() && w.is_contiguous() && x.numel() == w.numel(),
              "legendre_table: x, w float64 CUDA vectors of equal length");
  const int64_t K = x.numel();
  std::vector<int64_t> off(m_count);
  int64_t rows = 0;
  for (int64_t i = 0; i < m_count; ++i) {
    off[i] = rows;
    rows += std::max<int64_t>(0, L - (m0 + i));
  }
  auto row_off = torch::from_blob(off.data(), {m_count}, torch::kInt64).to(x.device());
  auto P = torch::zeros({std::max<int64_t>(rows, 1), K}, x.options().dtype(at::kFloat));
  check(nsw::legendre_table(x.data_ptr<double>(), w.data_ptr<double>(), (int)m0, (int)m_count, (int)L, (int)K,
                            row_off.data_ptr<int64_t>(), P.data_ptr<float>(), csphase ? 1 : 0, stream()),
        "legendre_table");
  return {P, row_off};
}

// F float32 [m_count, K, N] -> C float32 [m_count, L, N]
Tensor legendre_fwd(Tensor P, Tensor row_off, Tensor F, int64_t m0, int64_t L) {
  need_cuda(P, "P");
  need_cuda(F, "F");
  TORCH_CHECK(F.dim() == 3 && F.scalar_type() == at::kFloat, "legendre_fwd: F float32 [m, K, N]");
  const int64_t mc = F.size(0), K = F.size(1), N = F.size(2);
  TORCH_CHECK(row_off.numel() == mc && P.size(1) == K, "legendre_fwd: table shape");
  auto C = torch::empty({mc, L, N}, F.options());
  check(nsw::legendre_fwd(P.data_ptr<float>(), row_off.data_ptr<int64_t>(), F.data_ptr<float>(), C.data_ptr<float>(),
                          (int)m0, (int)mc, (int)L, (int)K, (int)N, stream()),
        "legendre_fwd");
  return C;
}

// dC float32 [m_count, L, N] -> dF float32 [m_count, K, N]
Tensor legendre_bwd(Tensor P, Tensor row_off, Tensor dC, int64_t m0, int64_t K) {
  need_cuda(P, "P");
  need_cuda(dC, "dC");
  TORCH_CHECK(dC.dim() == 3 && dC.scalar_type() == at::kFloat, "legendre_bwd: dC float32 [m, L, N]");
  const int64_t mc = dC.size(0), L = dC.size(1), N = dC.size(2);
  TORCH_CHECK(row_off.numel() == mc && P.size(1) == K, "legendre_bwd: table shape");
  auto dF = torch::empty({mc, K, N}, dC.options());
  check(nsw::legendre_bwd(P.data_ptr<float>(), row_off.data_ptr<int64_t>(), dC.data_ptr<float>(),
                          dF.data_ptr<float>(), (int)m0, (int)mc, (int)L, (int)K, (int)N, stream()),
        "legendre_bwd");
  return dF;
}

Tensor col_sum(Tensor x) {
  need_cuda(x, "x");
  const int n = (int)x.size(-1);
  const int64_t rows = x.numel() / n;
  // partial rows: up to 8 blocks per SM for the vector path, 4 for the scalar one
  int parts = (n % 8 == 0 && x.scalar_type() != at::kFloat) ? 8 * 148 : 4 * 148;
  if (rows < parts) parts = (int)std::max<int64_t>(1, rows);
  auto part = torch::empty({parts, n}, x.options().dtype(at::kFloat));
  auto out = torch::empty({n}, x.options().dtype(at::kFloat));
  check(nsw::col_sum(x.data_ptr(), out.data_ptr<float>(), part.data_ptr<float>(), parts, rows, n,
                     dt_code(x), stream()),
        "col_sum");
  return out;
}

// ------------------------------------------------------------------------------ patches
Tensor im2col(Tensor x, int64_t p, int64_t out_dtype) {
  need_cuda(x, "x");
  const int N = (int)x.size(0), C = (int)x.size(1), H = (int)x.size(2), W = (int)x.size(3);
  auto cols = torch::empty({(int64_t)N * (H / p) * (W / p), (int64_t)C * p * p},
                           x.options().dtype(scalar_of((int)out_dtype)));
  check(nsw::im2col_patch(x.data_ptr(), dt_code(x), cols.data_ptr(), N, C, H, W, (int)p, (int)out_dtype,
                          stream()),
        "im2col");
  return cols;
}

Tensor col2im(Tensor dcols, int64_t N, int64_t C, int64_t H, int64_t W, int64_t p, int64_t x_dtype) {
  need_cuda(dcols, "dcols");
  auto dx = torch::empty({N, C, H, W}, dcols.options().dtype(scalar_of((int)x_dtype)));
  check(nsw::col2im_patch(dcols.data_ptr(), dx.data_ptr(), (int)x_dtype, (int)N, (int)C, (int)H, (int)W,
                          (int)p, dt_code(dcols), stream()),
        "col2im");
  return dx;
}

Tensor unpatchify(Tensor y2, int64_t B, int64_t T, int64_t h, int64_t w, int64_t p, int64_t C) {
  need_cuda(y2, "y2");
  auto out = torch::empty({B, T, C, h * p, w * p}, y2.options());
  check(nsw::unpatchify(y2.data_ptr(), out.data_ptr(), (int)(B * T), (int)h, (int)w, (int)p, (int)C,
                        dt_code(y2), stream()),
        "unpatchify");
  return out;
}

Tensor patchify(Tensor dout, int64_t h, int64_t w, int64_t p, int64_t C) {
  need_cuda(dout, "dout");
  const int64_t BT = dout.numel() / (C * h * p * w * p);
  auto dy2 = torch::empty({BT * h * w, p * p * C}, dout.options());
  check(nsw::patchify(dout.data_ptr(), dy2.data_ptr(), (int)BT, (int)h, (int)w, (int)p, (int)C,
                      dt_code(dout), stream()),
        "patchify");
  return dy2;
}

// ------------------------------------------------------------------------------ losses
Tensor weighted_sse(Tensor x, Tensor y, c10::optional<Tensor> aw, c10::optional<Tensor> cw) {
  need_cuda(x, "x");
  need_cuda(y, "y");
  TORCH_CHECK(x.sizes() == y.sizes(), "weighted_sse: shape mismatch");
  const int W = (int)x.size(-1), H = (int)x.size(-2), C = (int)x.size(-3);
  const int64_t lead = x.numel() / ((int64_t)C * H * W);
  const int parts = 4 * 148;
  auto part = torch::empty({parts}, x.options().dtype(at::kFloat));
  auto out = torch::empty({}, x.options().dtype(at::kFloat));
  check(nsw::weighted_sse(x.data_ptr(), dt_code(x), y.data_ptr(), dt_code(y), opt_f32(aw), opt_f32(cw),
                          part.data_ptr<float>(), parts, out.data_ptr<float>(), lead, C, H, W, stream()),
        "weighted_sse");
  return out;
}

Tensor weighted_sse_bwd(Tensor x, Tensor y, c10::optional<Tensor> aw, c10::optional<Tensor> cw, Tensor gscale) {
  need_cuda(x, "x");
  need_cuda(y, "y");
  const int W = (int)x.size(-1), H = (int)x.size(-2), C = (int)x.size(-3);
  const int64_t lead = x.numel() / ((int64_t)C * H * W);
  auto dx = torch::empty_like(x);
  check(nsw::weighted_sse_bwd(x.data_ptr(), dt_code(x), y.data_ptr(), dt_code(y), opt_f32(aw), opt_f32(cw),
                              gscale.data_ptr<float>(), dx.data_ptr(), lead, C, H, W, stream()),
        "weighted_sse_bwd");
  return dx;
}

Tensor weighted_se_per_plane(Tensor x, Tensor y, Tensor aw) {
  need_cuda(x, "x");
  need_cuda(y, "y");
  const int W = (int)x.size(-1), H = (int)x.size(-2);
  const int64_t planes = x.numel() / ((int64_t)H * W);
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end() - 2);
  auto out = torch::empty(shape, x.options().dtype(at::kFloat));
  check(nsw::weighted_se_per_plane(x.data_ptr(), dt_code(x), y.data_ptr(), dt_code(y),
                                   aw.data_ptr<float>(), out.data_ptr<float>(), planes, H, W, stream()),
        "weighted_se_per_plane");
  return out;
}

// ------------------------------------------------------------------------------ optimizer
void adamw_step(Tensor p, Tensor g, Tensor m, Tensor v, Tensor shadow, Tensor gscale, Tensor skip, double lr,
                double b1, double b2, double eps, double wd, double bc1, double bc2, bool decoupled) {
  need_cuda(p, "p");
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat, "adamw: fp32 buffers");
  void* sh = shadow.numel() ? shadow.data_ptr() : nullptr;
  const int shd = shadow.numel() ? dt_code(shadow) : nsw::kF32;
  check(nsw::adamw_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), sh,
                        shd, gscale.data_ptr<float>(), skip.data_ptr<int>(), p.numel(), (float)lr, (float)b1,
                        (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2, decoupled, stream()),
        "adamw_step");
}

Tensor segment_sumsq(Tensor x, Tensor block_lo, Tensor block_hi, Tensor block_cls, int64_t ncls) {
  need_cuda(x, "x");
  const int nb = (int)block_lo.numel();
  auto part = torch::empty({nb}, x.options().dtype(at::kFloat));
  auto out = torch::empty({ncls}, x.options().dtype(at::kFloat));
  check(nsw::segment_sumsq(x.data_ptr<float>(), block_lo.data_ptr<int64_t>(), block_hi.data_ptr<int64_t>(),
                           block_cls.data_ptr<int>(), nb, (int)ncls, part.data_ptr<float>(), out.data_ptr<float>(),
                           stream()),
        "segment_sumsq");
  return out;
}

// ------------------------------------------------------------------------------ attention
nsw::AttnGeom make_geom(const std::vector<int64_t>& gi, double scale) {
  TORCH_CHECK(gi.size() == 14, "geometry: 14 ints expected");
  nsw::AttnGeom g{};
  g.B = (int)gi[0];
  g.T = (int)gi[1];
  g.H = (int)gi[2];
  g.W = (int)gi[3];
  g.nh = (int)gi[4];
  g.hd = (int)gi[5];
  g.wh = (int)gi[6];
  g.ww = (int)gi[7];
  g.sh = (int)gi[8];
  g.sw = (int)gi[9];
  g.mask = (int)gi[10];
  g.mask_shift = (int)gi[11];
  g.row_offset = (int)gi[12];
  g.h_global = (int)gi[13];
  g.scale = (float)scale;
  g.qkv_stride = 3LL * g.nh * g.hd;
  g.out_stride = (int64_t)g.nh * g.hd;
  return g;
}

std::vector<Tensor> window_attn_fwd(Tensor qkv, Tensor qw, Tensor kw, std::vector<int64_t> gi, double scale,
                                    int64_t impl, c10::optional<Tensor> stamps) {
  need_cuda(qkv, "qkv");
  auto g = make_geom(gi, scale);
  const int64_t tokens = (int64_t)g.B * g.T * g.H * g.W;
  TORCH_CHECK(qkv.numel() == tokens * g.qkv_stride, "qkv size");
  auto out = torch::empty({tokens, (int64_t)g.nh * g.hd}, qkv.options());
  const int L = g.T * g.wh * g.ww;
  const int64_t nwin = (int64_t)g.B * (g.H / g.wh) * (g.W / g.ww);
  auto lse = torch::empty({nwin * g.nh * L}, qkv.options().dtype(at::kFloat));
  // impl: 0 = default (the warp-specialised tcgen05 kernel where it applies, else mma.sync),
  // 1 = mma.sync, 2 = persistent tcgen05 (every warp in every phase), 3 = warp-specialised tcgen05.
  // Measured at 64800 tokens x 16 heads: 0.37 / 0.44 / 0.66 ms for impl 3 / 1 / 2.
  const bool tc_ok = nsw::window_attn_fwd_tc_supported(g, dt_code(qkv));
  TORCH_CHECK(impl != 2 || tc_ok, "window_attn_fwd: tcgen05 path needs bf16, head_dim 64, window <= 176 tokens");
  TORCH_CHECK(impl != 3 || tc_ok, "window_attn_fwd: tcgen05 path needs bf16, head_dim 64, window <= 176 tokens");
  if (tc_ok && (impl == 3 || impl == 0))
    check(nsw::window_attn_fwd_ws(qkv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), out.data_ptr(),
                                  lse.data_ptr<float>(), g, stream(),
                                  stamps ? reinterpret_cast<long long*>(stamps->data_ptr<int64_t>()) : nullptr),
          "window_attn_fwd_ws");
  else if (tc_ok && impl == 2)
    check(nsw::window_attn_fwd_tc(qkv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), out.data_ptr(),
                                  lse.data_ptr<float>(), g, stream()),
          "window_attn_fwd_tc");
  else
    check(nsw::window_attn_fwd(qkv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), out.data_ptr(),
                               lse.data_ptr<float>(), g, dt_code(qkv), stream()),
          "window_attn_fwd");
  return {out, lse};
}

std::vector<Tensor> window_attn_bwd(Tensor qkv, Tensor qw, Tensor kw, Tensor out, Tensor dout, Tensor lse,
                                    std::vector<int64_t> gi, double scale, int64_t impl,
                                    c10::optional<Tensor> stamps, c10::optional<Tensor> dqw_into,
                                    c10::optional<Tensor> dkw_into) {
  need_cuda(qkv, "qkv");
  need_cuda(dout, "dout");
  auto g = make_geom(gi, scale);
  auto dqkv = torch::empty_like(qkv);
  const int64_t nwin = (int64_t)g.B * (g.H / g.wh) * (g.W / g.ww);
  // impl: 0 = default (tcgen05 where supported), 1 = mma.sync, 2 = tcgen05/TMEM
  const bool tc_ok = nsw::window_attn_fwd_tc_supported(g, dt_code(qkv));
  TORCH_CHECK(impl != 2 || tc_ok, "window_attn_bwd: tcgen05 path needs bf16, head_dim 64, window <= 176 tokens");
  const bool tc = tc_ok && impl != 1;
  // QK-norm weight-gradient partial rows: one per CTA of the persistent tcgen05 kernel
  // (min(items, SMs) CTAs), one per (window, head) item for the mma.sync kernel; q and k partials
  // share one tensor so a single reduction sums both
  const int64_t items = nwin * g.nh;
  const int64_t rows = tc ? std::min<int64_t>(items, at::cuda::getCurrentDeviceProperties()->multiProcessorCount) : items;
  auto part = torch::empty({2, rows, (int64_t)g.hd}, qkv.options().dtype(at::kFloat));
  float* qp = part.data_ptr<float>();
  float* kp = qp + rows * g.hd;
  if (tc)
    check(nsw::window_attn_bwd_tc(qkv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), out.data_ptr(),
                                  dout.data_ptr(), lse.data_ptr<float>(), dqkv.data_ptr(), qp, kp, g, stream(),
                                  stamps ? reinterpret_cast<long long*>(stamps->data_ptr<int64_t>()) : nullptr),
          "window_attn_bwd_tc");
  else
    check(nsw::window_attn_bwd(qkv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), out.data_ptr(),
                               dout.data_ptr(), lse.data_ptr<float>(), dqkv.data_ptr(), qp, kp, g, dt_code(qkv),
                               stream()),
          "window_attn_bwd");
  // QK-norm weight gradients: added into the given fp32 gradient buffers (both or neither), else fresh
  if (dqw_into || dkw_into) {
    TORCH_CHECK(dqw_into && dkw_into, "window_attn_bwd: dqw_into and dkw_into go together");
    for (const Tensor* t : {&*dqw_into, &*dkw_into})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == g.hd,
                  "window_attn_bwd: QK-norm gradient buffers must be contiguous fp32 CUDA tensors of head_dim");
    check(nsw::sum_rows(part.data_ptr<float>(), 2, rows, g.hd, dqw_into->data_ptr<float>(), stream(), true,
                        dkw_into->data_ptr<float>()),
          "sum_rows");
    return {dqkv, *dqw_into, *dkw_into};
  }
  auto sums = torch::empty({2, (int64_t)g.hd}, qkv.options().dtype(at::kFloat));
  check(nsw::sum_rows(part.data_ptr<float>(), 2, rows, g.hd, sums.data_ptr<float>(), stream()), "sum_rows");
  return {dqkv, sums[0], sums[1]};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of neural_scaling_weather_b200";
  m.def("read_error_flag", &read_error_flag, py::arg("clear") = true);
  m.def("wgrad_supported", &wgrad_supported, py::arg("dy"), py::arg("x"));
  m.def("legendre_table", &legendre_table);
  m.def("dp_reduce", &dp_reduce);
  m.def("dp_adamw", &dp_adamw);
  m.def("dp_barrier", &dp_barrier);
  m.def("halo_band_bytes", &halo_band_bytes);
  m.def("halo_roll", &halo_roll);
  m.def("legendre_fwd", &legendre_fwd);
  m.def("legendre_bwd", &legendre_bwd);
  m.def("wgrad", &wgrad, py::arg("dy"), py::arg("x"), py::arg("out") = py::none(), py::arg("accumulate") = false,
        py::arg("db") = py::none(), py::arg("db_accumulate") = false);
  m.def("wgrad_segments", &wgrad_segments, py::arg("dy"), py::arg("x"), py::arg("outs"), py::arg("accumulate"),
        py::arg("dbs") = py::none(), py::arg("db_accumulate") = false);
  m.def("wgrad_plan", &wgrad_plan, py::arg("M"), py::arg("N"), py::arg("T"));
  m.def("error_word", &error_word);
  m.def("set_error_flag", &set_error_flag);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("eps") = -1.0, py::arg("add") = py::none(), py::arg("dw_into") = py::none());
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("res_period") = 0, py::arg("act") = 0, py::arg("preact") = py::none(), py::arg("out_f32") = false,
        py::arg("alpha") = 1.0, py::arg("out") = py::none(), py::arg("accumulate") = false, py::arg("impl") = 0);
  m.def("gemm_supported", &gemm_supported);
  m.def("gemm_allreduce", &gemm_allreduce, py::arg("A"), py::arg("B"), py::arg("bias") = py::none(),
        py::arg("residual") = py::none(), py::arg("part_ptrs"), py::arg("flag_ptrs"), py::arg("rank"),
        py::arg("stamps") = py::none());
  m.def("bias_act_residual", &bias_act_residual);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("col_sum", &col_sum);
  m.def("im2col", &im2col);
  m.def("col2im", &col2im);
  m.def("unpatchify", &unpatchify);
  m.def("patchify", &patchify);
  m.def("weighted_sse", &weighted_sse);
  m.def("weighted_sse_bwd", &weighted_sse_bwd);
  m.def("weighted_se_per_plane", &weighted_se_per_plane);
  m.def("adamw_step", &adamw_step);
  m.def("segment_sumsq", &segment_sumsq);
  m.def("window_attn_fwd", &window_attn_fwd, py::arg("qkv"), py::arg("qw"), py::arg("kw"), py::arg("geom"),
        py::arg("scale"), py::arg("impl") = 0, py::arg("stamps") = py::none());
  m.def("window_attn_bwd", &window_attn_bwd, py::arg("qkv"), py::arg("qw"), py::arg("kw"), py::arg("out"),
        py::arg("dout"), py::arg("lse"), py::arg("geom"), py::arg("scale"), py::arg("impl") = 0,
        py::arg("stamps") = py::none(), py::arg("dqw_into") = py::none(), py::arg("dkw_into") = py::none());
}
