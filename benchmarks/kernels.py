"""Kernel microbenchmarks with roofline fractions.

``python benchmarks/kernels.py <kernel> [--iters N] [shape flags]``

Each kernel is timed with CUDA events on the launching stream after warm-up, with a
synchronize on both sides; the inputs of the default shapes are larger than the 126 MB L2.
The fraction is taken against ``MEASURED_PEAKS.json`` when present (copy bandwidth and
cuBLAS bf16 throughput measured on this pool), otherwise against fixed fallback peaks.
Also used, with a small ``--iters``, as the command profiled by ``ncu``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from neural_scaling_weather_b200.ops import _ext  # noqa: E402
from neural_scaling_weather_b200.ops.geometry import WindowGeometry  # noqa: E402


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "of measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "of fallback"}


def timeit(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def report(name, ms, flops=None, nbytes=None, extra=None):
    pk = peaks()
    out = {"kernel": name, "ms": round(ms, 4)}
    if flops:
        tf = flops / ms / 1e9
        out["tflops"] = round(tf, 1)
        out["frac_tensor"] = f"{tf / pk['bf16_tflops']:.3f} {pk['src']}"
    if nbytes:
        gbs = nbytes / ms / 1e6
        out["gbs"] = round(gbs, 1)
        out["frac_hbm"] = f"{gbs / pk['hbm_gbs']:.3f} {pk['src']}"
    if extra:
        out.update(extra)
    print(json.dumps(out))
    return out


def bench_gemm(a):
    ext = _ext.require()
    M, N, K = a.M, a.N, a.K
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(N, device="cuda") if a.epilogue in ("bias", "gelu", "gelu_grad") else None
    pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16) if a.epilogue in ("gelu", "gelu_grad") else None
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16) if a.epilogue in ("residual", "aux") else None
    act = {"gelu": 1, "gelu_grad": 3, "aux": 4}.get(a.epilogue, 0)
    fn = lambda: ext.gemm(A, B, bias, res, 0, act, pre, impl=a.impl)  # noqa: E731
    ms = timeit(fn, a.iters)
    nbytes = 2 * (M * K + N * K + M * N * (1 + (pre is not None) + (res is not None)))
    r = report(f"gemm_tcgen05[{a.epilogue}] {M}x{N}x{K}", ms, 2.0 * M * N * K, nbytes)
    if a.compare:
        ms2 = timeit(lambda: torch.mm(A, B.t()), a.iters)
        report(f"cublas torch.mm {M}x{N}x{K}", ms2, 2.0 * M * N * K, 2 * (M * K + N * K + M * N))
    return r


def bench_block_gemms(a):
    """The eight tcgen05 GEMMs of one transformer block (forward and data-gradient)."""
    ext = _ext.require()
    M, E = a.M, 1024
    bf = dict(device="cuda", dtype=torch.bfloat16)
    x = torch.randn(M, E, **bf)
    h4 = torch.randn(M, 4 * E, **bf)
    u = torch.randn(M, 4 * E, **bf)
    res = torch.randn(M, E, **bf)
    W = {n: torch.randn(*shape, **bf) * 0.02 for n, shape in
         [("qkv", (3 * E, E)), ("proj", (E, E)), ("fc1", (4 * E, E)), ("fc2", (E, 4 * E))]}
    Wt = {n: w.t().contiguous() for n, w in W.items()}
    b = {n: torch.randn(w.shape[0], device="cuda") for n, w in W.items()}
    g3 = torch.randn(M, 3 * E, **bf)
    pre = torch.empty(M, 4 * E, **bf)
    cases = [
        ("fwd qkv +bias", lambda: ext.gemm(x, W["qkv"], b["qkv"], impl=a.impl), M, 3 * E, E),
        ("fwd proj +bias+res", lambda: ext.gemm(x, W["proj"], b["proj"], res, impl=a.impl), M, E, E),
        ("fwd fc1 +bias+gelu(+preact)", lambda: ext.gemm(x, W["fc1"], b["fc1"], None, 0, 1, pre, impl=a.impl), M, 4 * E, E),
        ("fwd fc1 +bias+gelu(+gelu')", lambda: ext.gemm(x, W["fc1"], b["fc1"], None, 0, 3, pre, impl=a.impl), M, 4 * E, E),
        ("fwd fc2 +bias+res", lambda: ext.gemm(h4, W["fc2"], b["fc2"], res, impl=a.impl), M, E, 4 * E),
        ("dgrad qkv", lambda: ext.gemm(g3, Wt["qkv"], impl=a.impl), M, E, 3 * E),
        ("dgrad proj", lambda: ext.gemm(x, Wt["proj"], impl=a.impl), M, E, E),
        ("dgrad fc2 *gelu'(u)", lambda: ext.gemm(x, Wt["fc2"], None, u, 0, 2, impl=a.impl), M, 4 * E, E),
        ("dgrad fc2 *aux", lambda: ext.gemm(x, Wt["fc2"], None, u, 0, 4, impl=a.impl), M, 4 * E, E),
        ("dgrad fc2 plain", lambda: ext.gemm(x, Wt["fc2"], impl=a.impl), M, 4 * E, E),
        ("dgrad fc1", lambda: ext.gemm(h4, Wt["fc1"], impl=a.impl), M, E, 4 * E),
        ("wgrad fc1 cublas", lambda: torch.mm(h4.t(), x, out_dtype=torch.float32), 4 * E, E, M),
    ]
    tot = 0.0
    for name, fn, m, n, k in cases:
        ms = timeit(fn, a.iters)
        if "plain" not in name and "wgrad" not in name and "(+preact)" not in name and "gelu'(u)" not in name:
            tot += ms
        report(name, ms, 2.0 * m * n * k, None)
    print(json.dumps({"block_fwd_plus_dgrad_ms": round(tot, 3)}))


def bench_attention(a):
    B, H, W, nh, hd = 1, a.H, a.W, a.heads, 64
    C = nh * hd
    geom = WindowGeometry(window=(9, 18), shift=(4, 9), mask=True, mask_shift=4, row_offset=0, h_global=H)
    qkv = torch.randn(B, 1, H, W, 3 * C, device="cuda", dtype=torch.bfloat16)
    qw = torch.ones(hd, device="cuda")
    kw = torch.ones(hd, device="cuda")
    ext = _ext.require()
    gi = [B, 1, H, W, nh, hd, 9, 18, 4, 9, 1, 4, 0, H]
    out, lse = ext.window_attn_fwd(qkv.view(-1, 3 * C), qw, kw, gi, hd ** -0.5)
    tokens = B * H * W
    L = 162
    flops = 4.0 * tokens * L * hd * nh  # QK^T and PV
    fimpls = [(i, t) for i, t in ((1, "mma.sync"), (2, "tcgen05"), (3, "tcgen05-ws")) if a.impl in (0, i)]
    for impl, tag in fimpls:
        ms = timeit(lambda: ext.window_attn_fwd(qkv.view(-1, 3 * C), qw, kw, gi, hd ** -0.5, impl), a.iters)
        report(f"window_attn_fwd[{tag}] tokens={tokens} heads={nh}", ms, flops, 2 * tokens * 4 * C)
    dout = torch.randn_like(out)
    impls = [(i, t) for i, t in ((1, "mma.sync"), (2, "tcgen05")) if a.impl in (0, i)]
    for impl, tag in impls:
        ms = timeit(lambda: ext.window_attn_bwd(qkv.view(-1, 3 * C), qw, kw, out, dout, lse, gi, hd ** -0.5,
                                                impl), a.iters)
        report(f"window_attn_bwd[{tag}] tokens={tokens} heads={nh}", ms, 2.5 * flops, 2 * tokens * 8 * C)


def bench_wgrad(a):
    """Weight-gradient GEMMs of one Swin block (dW = dy^T x, fp32 out) against cuBLAS (torch.mm)."""
    ext = _ext.require()
    T, E = a.M, 1024
    shapes = [("qkv", 3 * E, E), ("proj", E, E), ("fc1", 4 * E, E), ("fc2", E, 4 * E)]
    for name, m, n in shapes:
        dy = torch.randn(T, m, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(T, n, device="cuda", dtype=torch.bfloat16)
        out = torch.zeros(m, n, device="cuda")
        db = torch.zeros(m, device="cuda")
        flops = 2.0 * T * m * n
        ms = timeit(lambda: ext.wgrad(dy, x, out, True, db, True), a.iters)
        report(f"wgrad[tcgen05 +db] {name} T={T} M={m} N={n} splits={ext.wgrad_plan(m, n, T)}", ms, flops,
               2 * T * (m + n))
        ms = timeit(lambda: torch.mm(dy.t(), x, out_dtype=torch.float32), a.iters)
        report(f"wgrad[cublas] {name} T={T} M={m} N={n}", ms, flops, 2 * T * (m + n))


def bench_amse(a):
    """AMSE loss forward + backward on 70 x 720 x 1440 fields (device SHT: rFFT, fp32 Legendre kernels)."""
    import numpy as np

    from neural_scaling_weather_b200.losses import AMSELoss

    H, W, C = 720, 1440, 70
    lat = np.linspace(90, -90, H + 1)[:-1]
    lon = np.arange(W) * 360.0 / W
    loss_fn = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[H], [W]])
    x = torch.randn(1, 1, C, H, W, device="cuda", requires_grad=True)
    y = torch.randn(1, 1, C, H, W, device="cuda")

    def step():
        loss_fn(x, y).backward()

    ms = timeit(step, a.iters)
    # Legendre contraction FLOPs (triangular, forward for x and y, adjoint for x) plus the rFFTs
    L, M, N = H, W // 2 + 1, 2 * C
    flops = 3 * 2.0 * sum(L - m for m in range(min(M, L))) * H * N
    report(f"amse fwd+bwd {C}x{H}x{W}", ms, flops, 4 * 3 * C * H * W)


def bench_rmsnorm(a):
    ext = _ext.require()
    x = torch.randn(a.M, a.N, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(a.N, device="cuda")
    ms = timeit(lambda: ext.rmsnorm_fwd(x, w, 1e-7), a.iters)
    report(f"rmsnorm_fwd {a.M}x{a.N}", ms, None, 4 * a.M * a.N)
    y, r = ext.rmsnorm_fwd(x, w, 1e-7)
    ms = timeit(lambda: ext.rmsnorm_bwd(y, x, w, r, 1e-7), a.iters)
    report(f"rmsnorm_bwd {a.M}x{a.N}", ms, None, 6 * a.M * a.N)


def bench_adamw(a):
    ext = _ext.require()
    n = a.M
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    one = torch.ones(1, device="cuda")
    zero = torch.zeros(1, device="cuda", dtype=torch.int32)
    fn = lambda: ext.adamw_step(p, g, m, v, sh, one, zero, 1e-4, 0.9, 0.95, 1e-8, 1e-4, 0.5, 0.5, True)  # noqa
    ms = timeit(fn, a.iters)
    report(f"adamw_step n={n}", ms, None, n * (4 * 4 + 3 * 4 + 2))


def bench_sse(a):
    ext = _ext.require()
    x = torch.randn(1, 1, 70, 720, 1440, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(1, 1, 70, 720, 1440, device="cuda")
    aw = torch.rand(720, device="cuda")
    ms = timeit(lambda: ext.weighted_sse(x, y, aw, None), a.iters)
    report("weighted_sse 70x720x1440", ms, None, x.numel() * 6)
    g = torch.ones(1, device="cuda")
    ms = timeit(lambda: ext.weighted_sse_bwd(x, y, aw, None, g), a.iters)
    report("weighted_sse_bwd 70x720x1440", ms, None, x.numel() * 8)


def bench_patch(a):
    """Patch embedding im2col / col2im and head unpatchify / patchify at 73 (70) x 720 x 1440, patch 4."""
    ext = _ext.require()
    x = torch.randn(1, 73, 720, 1440, device="cuda")
    ms = timeit(lambda: ext.im2col(x, 4, 0), a.iters)
    report("im2col fp32->bf16 73x720x1440 p4", ms, None, x.numel() * (4 + 2))
    cols = ext.im2col(x, 4, 0)
    ms = timeit(lambda: ext.col2im(cols, 1, 73, 720, 1440, 4, 2), a.iters)
    report("col2im bf16->fp32 73x720x1440 p4", ms, None, x.numel() * (2 + 4))
    y2 = torch.randn(180 * 360, 16 * 70, device="cuda", dtype=torch.bfloat16)
    ms = timeit(lambda: ext.unpatchify(y2, 1, 1, 180, 360, 4, 70), a.iters)
    report("unpatchify bf16 70x720x1440 p4", ms, None, y2.numel() * 4)
    out = ext.unpatchify(y2, 1, 1, 180, 360, 4, 70)
    ms = timeit(lambda: ext.patchify(out, 180, 360, 4, 70), a.iters)
    report("patchify bf16 70x720x1440 p4", ms, None, y2.numel() * 4)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "block", "attention", "wgrad", "amse", "rmsnorm", "adamw", "sse",
                                       "patch", "colsum", "all"])
    ap.add_argument("--M", type=int, default=64800)
    ap.add_argument("--N", type=int, default=3072)
    ap.add_argument("--K", type=int, default=1024)
    ap.add_argument("--H", type=int, default=180)
    ap.add_argument("--W", type=int, default=360)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--epilogue", default="bias", choices=["none", "bias", "gelu", "gelu_grad", "residual", "aux"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--compare", action="store_true")
    ap.add_argument("--impl", type=int, default=0,
                    help="attention: 1 = mma.sync only, 2 = tcgen05 only, 3 = warp-specialised tcgen05 forward only; block GEMMs: 1 = one CTA per tile, "
                         "2 = CTA pair, 0 = default dispatch")
    a = ap.parse_args()
    if a.kernel in ("gemm", "all"):
        bench_gemm(a)
    if a.kernel == "block":
        bench_block_gemms(a)
    if a.kernel in ("colsum", "all"):
        ext = _ext.require()
        for n in (1024, 3072, 4096):
            t = torch.randn(a.M, n, device="cuda", dtype=torch.bfloat16)
            ms = timeit(lambda: ext.col_sum(t), a.iters)
            report(f"col_sum {a.M}x{n}", ms, None, 2 * a.M * n)
    if a.kernel in ("attention", "all"):
        bench_attention(a)
    if a.kernel in ("wgrad", "all"):
        bench_wgrad(a)
    if a.kernel in ("amse", "all"):
        bench_amse(a)
    if a.kernel in ("patch", "all"):
        bench_patch(a)
    if a.kernel in ("rmsnorm", "all"):
        a2 = argparse.Namespace(**vars(a))
        if a.kernel == "all":
            a2.N = 1024
        bench_rmsnorm(a2)
    if a.kernel in ("adamw", "all"):
        a3 = argparse.Namespace(**vars(a))
        a3.M = 204_000_000 if a.kernel == "all" else a.M
        bench_adamw(a3)
    if a.kernel in ("sse", "all"):
        bench_sse(a)
    err = _ext.require().read_error_flag(True)
    if err:
        raise SystemExit(f"device error flag {err}")


if __name__ == "__main__":
    main()
