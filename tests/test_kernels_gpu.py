"""Numerics of every sm_100a kernel against a plain-PyTorch fp32 reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.importorskip("torch").cuda
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from neural_scaling_weather_b200 import ops  # noqa: E402
from neural_scaling_weather_b200.ops import _ext, reference  # noqa: E402
from neural_scaling_weather_b200.ops.geometry import WindowGeometry  # noqa: E402

DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _ext_loaded():
    ext = _ext.require()
    yield ext
    assert ext.read_error_flag(True) == 0


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


# --------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 1120, 1168), (1000, 3072, 1024),
                                   (777, 128, 64), (129, 40, 96), (4096, 4096, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("impl", [1, 2])
def test_gemm_plain(M, N, K, dtype, impl, _ext_loaded):
    """impl 1: one CTA per 128 x BN tile; impl 2: CTA pair (cta_group::2) per 256 x 256 tile."""
    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV, dtype=dtype)
    b = torch.randn(N, K, device=DEV, dtype=dtype)
    d = _ext_loaded.gemm(a, b, impl=impl)
    ref = a.float() @ b.float().t()
    assert rel(d, ref) < 1e-2


@pytest.mark.parametrize("impl", [1, 2, 4])
def test_gemm_epilogues(impl, _ext_loaded):
    """impl 1: single CTA; 2: CTA pair; 4: single CTA with twelve epilogue warps for the GELU
    epilogues."""
    torch.manual_seed(1)
    M, N, K = 515, 512, 256
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.1
    bias = torch.randn(N, device=DEV)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    pre = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    y = _ext_loaded.gemm(a, b, bias, None, 0, 1, pre, impl=impl)
    u = a.float() @ b.float().t() + bias
    assert rel(pre, u) < 1e-2
    assert rel(y, torch.nn.functional.gelu(u)) < 1e-2
    y2 = _ext_loaded.gemm(a, b, bias, res, impl=impl)
    assert rel(y2, u + res.float()) < 1e-2
    # act 3: GELU with GELU'(u) as the saved tensor; act 4: multiply by the saved tensor
    g = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    y4 = _ext_loaded.gemm(a, b, bias, None, 0, 3, g, impl=impl)
    uu = u.clone().requires_grad_()
    torch.nn.functional.gelu(uu).sum().backward()
    assert rel(y4, torch.nn.functional.gelu(u)) < 1e-2
    assert rel(g, uu.grad) < 1e-2
    y5 = _ext_loaded.gemm(a, b, None, g, 0, 4, impl=impl)
    assert rel(y5, (a.float() @ b.float().t()) * g.float()) < 1e-2
    # broadcast residual (period)
    pos = torch.randn(128, N, device=DEV, dtype=torch.bfloat16)
    a3 = a[:512].contiguous()
    y3 = _ext_loaded.gemm(a3, b, None, pos, 128, impl=impl)
    ref3 = (a3.float() @ b.float().t()).view(4, 128, N) + pos.float()
    assert rel(y3, ref3.view(512, N)) < 1e-2
    # fp32 output with accumulation
    out = torch.randn(M, N, device=DEV)
    base = out.clone()
    _ext_loaded.gemm(a, b, None, None, 0, 0, None, True, 0.5, out, True, impl=impl)
    assert rel(out, base + 0.5 * (a.float() @ b.float().t())) < 1e-3


@pytest.mark.parametrize("M,N", [(512, 512), (1024, 1000), (4096, 4096)])
@pytest.mark.parametrize("impl", [1, 3, 4])
def test_gemm_residual_epilogues(M, N, impl, _ext_loaded):
    """impl 1 (M % 32 == 0, N > 128): residual / aux tiles arrive by TMA into the epilogue buffers;
    impl 3: the fallback that loads them with plain loads in the drain; impl 4: TMA residual
    tiles with twelve epilogue warps for the GELU forms."""
    torch.manual_seed(2)
    K = 256
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.1
    bias = torch.randn(N, device=DEV)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    acc = a.float() @ b.float().t()
    u = acc + bias
    assert rel(_ext_loaded.gemm(a, b, bias, res, impl=impl), u + res.float()) < 1e-2
    assert rel(_ext_loaded.gemm(a, b, None, res, 0, 4, impl=impl), acc * res.float()) < 1e-2
    r = res.float().requires_grad_()
    torch.nn.functional.gelu(r).sum().backward()
    assert rel(_ext_loaded.gemm(a, b, None, res, 0, 2, impl=impl), acc * r.grad) < 1e-2
    assert rel(_ext_loaded.gemm(a, b, bias, res, 0, 1, impl=impl), torch.nn.functional.gelu(u) + res.float()) < 1e-2


# --------------------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("rows,n", [(333, 64), (333, 1024), (333, 2048), (777, 4096), (20011, 1024),
                                    (70000, 1024)])
def test_rmsnorm(rows, n):
    """TMA row-tile kernels (ring of three tiles per CTA, partial last tile) against fp32."""
    torch.manual_seed(0)
    x = torch.randn(rows, n, device=DEV).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(n, device=DEV)).requires_grad_()
    y = ops.rms_norm(x, w)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    yr = reference.rms_norm(xr, wr)
    assert rel(y, yr) < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    assert rel(x.grad, xr.grad) < 2e-2
    assert rel(w.grad, wr.grad) < 2e-2


# --------------------------------------------------------------------------- attention
ATTN_CASES = [
    # B, T, H, W, nh, hd, window, shift, mask
    (1, 1, 18, 36, 2, 64, (9, 18), (0, 0), False),
    (1, 1, 18, 36, 2, 64, (9, 18), (4, 9), True),
    (2, 1, 8, 16, 4, 16, (4, 8), (2, 4), True),
    (1, 2, 8, 16, 2, 32, (4, 8), (2, 4), True),
    (1, 1, 12, 24, 2, 128, (4, 8), (2, 4), True),
]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_window_attention(case):
    B, T, H, W, nh, hd, win, shift, mask = case
    torch.manual_seed(0)
    C = nh * hd
    geom = WindowGeometry(window=win, shift=shift, mask=mask, mask_shift=shift[0], row_offset=0,
                          h_global=H)
    qkv = torch.randn(B, T, H, W, 3 * C, device=DEV).bfloat16().requires_grad_()
    qw = (1 + 0.1 * torch.randn(hd, device=DEV)).requires_grad_()
    kw = (1 + 0.1 * torch.randn(hd, device=DEV)).requires_grad_()
    scale = hd ** -0.5
    out = ops.window_attention(qkv, qw, kw, nh, hd, geom, scale)
    qr = qkv.detach().float().requires_grad_()
    qwr = qw.detach().clone().requires_grad_()
    kwr = kw.detach().clone().requires_grad_()
    ref = reference.window_attention(qr, qwr, kwr, nh, hd, geom, scale)
    assert rel(out, ref) < 2e-2
    g = torch.randn_like(ref)
    out.backward(g.bfloat16())
    ref.backward(g)
    assert rel(qkv.grad, qr.grad) < 4e-2
    assert rel(qw.grad, qwr.grad) < 4e-2
    assert rel(kw.grad, kwr.grad) < 4e-2


# --------------------------------------------------------------------------- linear op
@pytest.mark.parametrize("act,residual", [(None, False), ("gelu", False), (None, True)])
def test_linear_op(act, residual):
    torch.manual_seed(0)
    x = torch.randn(2, 3, 40, 64, device=DEV).bfloat16().requires_grad_()
    w1 = (0.05 * torch.randn(96, 64, device=DEV)).requires_grad_()
    w2 = (0.05 * torch.randn(32, 64, device=DEV)).requires_grad_()
    b1 = torch.randn(96, device=DEV).requires_grad_()
    b2 = torch.randn(32, device=DEV).requires_grad_()
    res = torch.randn(2, 3, 40, 128, device=DEV).bfloat16().requires_grad_() if residual else None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ops.linear(x, [w1, w2], [b1, b2], residual=res, activation=act)
    xr = x.detach().float().requires_grad_()
    ws = [t.detach().clone().requires_grad_() for t in (w1, w2, b1, b2)]
    rr = res.detach().float().requires_grad_() if residual else None
    yr = reference.linear(xr, torch.cat(ws[:2]), torch.cat(ws[2:]), rr, act)
    assert rel(y, yr) < 2e-2
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    assert rel(x.grad, xr.grad) < 3e-2
    for a, b in zip((w1, w2, b1, b2), ws):
        assert rel(a.grad, b.grad) < 3e-2
    if residual:
        assert rel(res.grad, rr.grad) < 1e-2


# --------------------------------------------------------------------------- patch embed / head
def test_patch_embed_and_head():
    torch.manual_seed(0)
    N, C, H, W, p, E = 2, 13, 24, 48, 4, 64
    x = torch.randn(N, C, H, W, device=DEV).requires_grad_()
    w = (0.05 * torch.randn(E, C, p, p, device=DEV)).requires_grad_()
    b = torch.randn(E, device=DEV).requires_grad_()
    add = torch.randn(1, H // p, W // p, E, device=DEV).bfloat16().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ops.patch_embed(x, w, b, p, add=add)
    xr = x.detach().clone().requires_grad_()
    wr, br = w.detach().clone().requires_grad_(), b.detach().clone().requires_grad_()
    ar = add.detach().float().requires_grad_()
    yr = reference.patch_embed(xr, wr, br, p, add=ar)
    assert rel(y, yr) < 2e-2
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    for a, r in ((x, xr), (w, wr), (b, br), (add, ar)):
        assert rel(a.grad, r.grad) < 3e-2

    Co = 10
    t = torch.randn(N, 1, H // p, W // p, E, device=DEV).bfloat16().requires_grad_()
    hw = (0.05 * torch.randn(Co * p * p, E, device=DEV)).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        o = ops.head_unpatchify(t, hw, p, Co)
    tr = t.detach().float().requires_grad_()
    hwr = hw.detach().clone().requires_grad_()
    orf = reference.head_unpatchify(tr, hwr, p, Co)
    assert o.shape == orf.shape
    assert rel(o, orf) < 2e-2
    g = torch.randn_like(orf)
    o.backward(g.bfloat16())
    orf.backward(g)
    assert rel(t.grad, tr.grad) < 3e-2
    assert rel(hw.grad, hwr.grad) < 3e-2


@pytest.mark.parametrize("B,T,h,w,p,C", [(1, 1, 180, 360, 4, 70), (2, 1, 5, 12, 4, 10), (1, 2, 3, 22, 4, 8),
                                          (1, 1, 4, 7, 2, 6)])
def test_patch_layout_kernels_exact(B, T, h, w, p, C):
    """unpatchify / patchify / im2col are pure re-layouts: equal to the PyTorch permutes bit for bit (the
    tiled shared-memory forms, ragged last tile included, and the per-element fallback)."""
    from neural_scaling_weather_b200.ops import _ext
    from neural_scaling_weather_b200.ops.fused import DT

    ext = _ext.require()
    torch.manual_seed(0)
    y2 = torch.randn(B * T * h * w, p * p * C, device=DEV).bfloat16()
    out = ext.unpatchify(y2, B, T, h, w, p, C)
    ref = y2.view(B, T, h, w, p, p, C).permute(0, 1, 6, 2, 4, 3, 5).reshape(B, T, C, h * p, w * p)
    assert torch.equal(out, ref)
    d = torch.randn(B, T, C, h * p, w * p, device=DEV).bfloat16()
    dy2 = ext.patchify(d, h, w, p, C)
    refd = d.view(B, T, C, h, p, w, p).permute(0, 1, 3, 5, 4, 6, 2).reshape(B * T * h * w, p * p * C)
    assert torch.equal(dy2, refd)
    N = B * T
    x = torch.randn(N, C, h * p, w * p, device=DEV)
    cols = ext.im2col(x, p, DT[torch.bfloat16])
    refc = x.view(N, C, h, p, w, p).permute(0, 2, 4, 1, 3, 5).reshape(N * h * w, C * p * p).bfloat16()
    assert torch.equal(cols, refc)


def test_coord_pos_embed_cached_per_weight_version():
    """The coordinate positional embedding equals the plain patch projection (values and weight / bias
    gradients), is served from the cache while the weights are unchanged, and is rebuilt after an
    in-place weight update (version bump)."""
    torch.manual_seed(0)
    T, H, W, p, E = 1, 24, 48, 4, 64
    coords = torch.randn(T, 4, H, W, device=DEV)
    w = torch.nn.Parameter(0.05 * torch.randn(E, 4, p, p, device=DEV))
    b = torch.nn.Parameter(torch.randn(E, device=DEV))
    wr, br = (torch.nn.Parameter(t.detach().clone()) for t in (w, b))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a = ops.coord_pos_embed(coords, w, b, p)
        r = ops.patch_embed(coords, wr, br, p)
    assert a.shape == r.shape and rel(a, r) < 1e-2
    g = torch.randn_like(r.float())
    a.backward(g.to(a.dtype))
    r.backward(g.to(r.dtype))
    assert rel(w.grad, wr.grad) < 2e-2 and rel(b.grad, br.grad) < 2e-2
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a2 = ops.coord_pos_embed(coords, w, b, p)
    assert a2.data_ptr() == a.data_ptr()  # cache hit: no recomputation
    with torch.no_grad():
        w.add_(0.01)
        wr.add_(0.01)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a3 = ops.coord_pos_embed(coords, w, b, p)
        r3 = ops.patch_embed(coords, wr, br, p)
    assert rel(a3, r3) < 1e-2 and rel(a3, a) > 1e-3
    # weights change, then a validation-style forward rebuilds the cache under inference mode: the next
    # training forward still sends gradients to the embedding weights
    with torch.no_grad():
        w.add_(0.01)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        ops.coord_pos_embed(coords, w, b, p)
    w.grad, b.grad = None, None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a4 = ops.coord_pos_embed(coords, w, b, p)
    a4.float().sum().backward()
    assert w.grad is not None and b.grad is not None and torch.isfinite(w.grad).all()


# --------------------------------------------------------------------------- losses
def test_weighted_sse():
    torch.manual_seed(0)
    x = torch.randn(2, 1, 7, 33, 65, device=DEV).bfloat16().requires_grad_()
    y = torch.randn(2, 1, 7, 33, 65, device=DEV)
    aw = torch.rand(33, 1, device=DEV)
    cw = torch.rand(7, 1, 1, device=DEV)
    s = ops.weighted_sse(x, y, aw, cw)
    xr = x.detach().float().requires_grad_()
    sr = reference.weighted_sse(xr, y, aw, cw)
    assert abs(s.item() - sr.item()) / sr.item() < 1e-4
    (3 * s).backward()
    (3 * sr).backward()
    assert rel(x.grad, xr.grad) < 1e-2
    pc = ops.weighted_se_per_channel(x.detach(), y, aw)
    pcr = reference.weighted_se_per_channel(x.detach().float(), y, aw)
    assert rel(pc, pcr) < 1e-4


# --------------------------------------------------------------------------- optimizer and norm
def test_fused_adamw_matches_torch():
    from neural_scaling_weather_b200.training.optimizer import FusedAdamW

    torch.manual_seed(0)
    shapes = [(33, 17), (64,), (5, 3, 2)]
    ps = [torch.nn.Parameter(torch.randn(*s, device=DEV)) for s in shapes]
    qs = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    opt = FusedAdamW(ps, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, shadow_dtype=torch.bfloat16)
    ref = torch.optim.AdamW(qs, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(5):
        for p, q in zip(ps, qs):
            g = torch.randn_like(p)
            p.grad.copy_(g)
            q.grad = g.clone()
        opt.step()
        ref.step()
    for p, q in zip(ps, qs):
        assert torch.allclose(p, q, atol=1e-5, rtol=1e-5)
    sd = opt.state_dict()
    assert set(sd["state"][0].keys()) == {"step", "exp_avg", "exp_avg_sq"}
    assert torch.allclose(opt.space.shadow.float(), opt.space.data, atol=1e-2, rtol=1e-2)


def test_sharded_norm_kernel():
    from neural_scaling_weather_b200.training.grad_norm import ShardedNorm
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace

    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(s, device=DEV)) for s in (100000, 7, 70000)]
    for p in ps:
        p.comm_metadata = {"sharded": [], "shared": [], "reduce": []}
    space = FlatParamSpace(ps)
    for p in ps:
        p.grad.copy_(torch.randn_like(p))
    n = ShardedNorm(space).norm("grad")
    ref = torch.sqrt(sum((p.grad.double() ** 2).sum() for p in ps))
    assert abs(n.item() - ref.item()) / ref.item() < 1e-5


# --------------------------------------------------------------------------- fused MLP
@pytest.mark.parametrize("residual", [False, True])
def test_fused_mlp(residual):
    torch.manual_seed(0)
    x = torch.randn(3, 100, 64, device=DEV).bfloat16().requires_grad_()
    w1 = (0.05 * torch.randn(256, 64, device=DEV)).requires_grad_()
    b1 = (0.1 * torch.randn(256, device=DEV)).requires_grad_()
    w2 = (0.05 * torch.randn(64, 256, device=DEV)).requires_grad_()
    b2 = (0.1 * torch.randn(64, device=DEV)).requires_grad_()
    res = torch.randn(3, 100, 64, device=DEV).bfloat16().requires_grad_() if residual else None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ops.mlp(x, w1, b1, w2, b2, res)
    xr = x.detach().float().requires_grad_()
    ps = [t.detach().clone().requires_grad_() for t in (w1, b1, w2, b2)]
    rr = res.detach().float().requires_grad_() if residual else None
    yr = reference.linear(reference.linear(xr, ps[0], ps[1], activation="gelu"), ps[2], ps[3], residual=rr)
    assert rel(y, yr) < 2e-2
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    assert rel(x.grad, xr.grad) < 3e-2
    for a, b in zip((w1, b1, w2, b2), ps):
        assert rel(a.grad, b.grad) < 3e-2
    if residual:
        assert rel(res.grad, rr.grad) < 1e-2


# --------------------------------------------------------------------------- tcgen05 attention forward
TC_CASES = [
    (1, 1, 18, 36, 2, (9, 18), (0, 0), False),
    (1, 1, 18, 36, 2, (9, 18), (4, 9), True),
    (2, 1, 27, 36, 3, (9, 18), (4, 9), True),
    (1, 1, 16, 32, 2, (8, 16), (4, 8), True),
    (1, 2, 8, 16, 2, (4, 8), (2, 4), True),
    # several (window, head) items per persistent CTA: head and window changes, next-item loads
    (1, 1, 90, 360, 4, (9, 18), (4, 9), True),
]


@pytest.mark.parametrize("case", TC_CASES)
def test_window_attention_tcgen05_forward(case, _ext_loaded):
    B, T, H, W, nh, win, shift, mask = case
    hd = 64
    torch.manual_seed(0)
    C = nh * hd
    geom = WindowGeometry(window=win, shift=shift, mask=mask, mask_shift=shift[0], row_offset=0, h_global=H)
    qkv = torch.randn(B, T, H, W, 3 * C, device=DEV).bfloat16()
    qw = 1 + 0.1 * torch.randn(hd, device=DEV)
    kw = 1 + 0.1 * torch.randn(hd, device=DEV)
    gi = [B, T, H, W, nh, hd, win[0], win[1], shift[0], shift[1], int(mask), shift[0], 0, H]
    out_mma, lse_mma = _ext_loaded.window_attn_fwd(qkv.view(-1, 3 * C), qw, kw, gi, hd ** -0.5, 1)
    ref = reference.window_attention(qkv.float(), qw, kw, nh, hd, geom, hd ** -0.5)
    for impl in (2, 3):  # persistent tcgen05; warp-specialised tcgen05
        out_tc, lse_tc = _ext_loaded.window_attn_fwd(qkv.view(-1, 3 * C), qw, kw, gi, hd ** -0.5, impl)
        assert _ext_loaded.read_error_flag(True) == 0, impl
        assert rel(out_tc.view_as(ref), ref) < 2e-2, impl
        assert rel(out_tc, out_mma) < 1e-2, impl
        assert torch.allclose(lse_tc, lse_mma, atol=2e-2, rtol=1e-3), impl


@pytest.mark.parametrize("case", TC_CASES)
def test_window_attention_tcgen05_backward(case, _ext_loaded):
    B, T, H, W, nh, win, shift, mask = case
    hd = 64
    torch.manual_seed(1)
    C = nh * hd
    geom = WindowGeometry(window=win, shift=shift, mask=mask, mask_shift=shift[0], row_offset=0, h_global=H)
    qkv = torch.randn(B, T, H, W, 3 * C, device=DEV).bfloat16()
    qw = 1 + 0.1 * torch.randn(hd, device=DEV)
    kw = 1 + 0.1 * torch.randn(hd, device=DEV)
    gi = [B, T, H, W, nh, hd, win[0], win[1], shift[0], shift[1], int(mask), shift[0], 0, H]
    out, lse = _ext_loaded.window_attn_fwd(qkv.view(-1, 3 * C), qw, kw, gi, hd ** -0.5, 1)
    dout = torch.randn_like(out)
    args = (qkv.view(-1, 3 * C), qw, kw, out, dout, lse, gi, hd ** -0.5)
    dq_tc, dqw_tc, dkw_tc = _ext_loaded.window_attn_bwd(*args, 2)
    dq_mma, dqw_mma, dkw_mma = _ext_loaded.window_attn_bwd(*args, 1)
    assert _ext_loaded.read_error_flag(True) == 0
    xr = qkv.float().requires_grad_()
    qwr = qw.clone().requires_grad_()
    kwr = kw.clone().requires_grad_()
    ref = reference.window_attention(xr, qwr, kwr, nh, hd, geom, hd ** -0.5)
    ref.backward(dout.float().view_as(ref))
    assert rel(dq_tc.view_as(xr), xr.grad) < 3e-2
    assert rel(dq_tc, dq_mma) < 2e-2
    assert rel(dqw_tc, qwr.grad) < 3e-2
    assert rel(dkw_tc, kwr.grad) < 3e-2


def test_rms_norm_with_skip_gradients():
    """(norm(x), x) from one node: dx sums both paths inside the RMSNorm backward kernel."""
    torch.manual_seed(3)
    x = torch.randn(4097, 1024, device=DEV).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(1024, device=DEV)).requires_grad_()
    y, skip = ops.rms_norm_with_skip(x, w)
    g1, g2 = torch.randn_like(y), torch.randn_like(skip)
    (y * g1 + skip * g2).float().sum().backward()
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    yr = reference.rms_norm(xr, wr)
    (yr * g1.float() + xr * g2.float()).sum().backward()
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 2e-2
    assert rel(w.grad, wr.grad) < 2e-2


# --------------------------------------------------------------------------- weight-gradient GEMM
WGRAD_CASES = [
    # T, M, N, col_offset (dy a column slice at this offset of a wider tensor), with bias
    (777, 200, 136, 0, True),       # ragged everywhere, one split
    (4099, 1024, 1024, 0, True),    # split-K with the last-arriver reduction
    (8192, 1024, 1024, 1024, True),  # dy a column slice (row stride 3072)
    (6000, 4096, 264, 0, False),    # ragged N, many m tiles
]


@pytest.mark.parametrize("case", WGRAD_CASES)
def test_wgrad_matches_fp32(case, _ext_loaded):
    """dW = dy^T x and db = colsum(dy) on the tcgen05 kernel (MN-major TMA operands, CTA pair,
    split-K) against fp32 PyTorch; accumulation into a sentinel-guarded output, deterministic reruns."""
    T, M, N, off, with_bias = case
    torch.manual_seed(11)
    width = off + M + (1024 if off else 0)
    dy_full = torch.randn(T, width, device=DEV).bfloat16()
    dy = dy_full[:, off:off + M]
    x = torch.randn(T, N, device=DEV).bfloat16()
    ref = dy.float().t() @ x.float()
    ref_b = dy.float().sum(0)
    pad = 1024
    buf = torch.full((M * N + 2 * pad,), 12345.0, device=DEV)
    out = buf[pad:pad + M * N]
    old = torch.randn(M * N, device=DEV)
    out.copy_(old)
    db = torch.randn(M, device=DEV) if with_bias else None
    db_old = db.clone() if with_bias else None
    _ext_loaded.wgrad(dy, x, out, True, db, True)
    torch.cuda.synchronize()
    assert _ext_loaded.read_error_flag(True) == 0
    assert torch.all(buf[:pad] == 12345.0) and torch.all(buf[pad + M * N:] == 12345.0)
    assert rel(out.view(M, N) - old.view(M, N), ref) < 3e-3
    if with_bias:
        assert rel(db - db_old, ref_b) < 3e-3
    # written (not accumulated), twice: bit-identical
    d1 = _ext_loaded.wgrad(dy, x)
    d2 = _ext_loaded.wgrad(dy, x)
    assert rel(d1, ref) < 3e-3
    assert torch.equal(d1, d2)
    assert _ext_loaded.read_error_flag(True) == 0


def test_wgrad_segments_balanced_schedule(_ext_loaded):
    """Three equal row segments (a fused q/k/v projection) written to separate buffers in one launch,
    on shapes whose plan is the balanced schedule (tiles < CTA pairs) and the uniform split."""
    torch.manual_seed(12)
    for T, seg, N in ((64800, 1024, 1024), (20000, 512, 768)):
        dy = torch.randn(T, 3 * seg, device=DEV).bfloat16()
        x = torch.randn(T, N, device=DEV).bfloat16()
        ref = dy.float().t() @ x.float()
        ref_b = dy.float().sum(0)
        outs = [torch.randn(seg * N, device=DEV) for _ in range(3)]
        olds = [o.clone() for o in outs]
        dbs = [torch.randn(seg, device=DEV) for _ in range(3)]
        db_olds = [d.clone() for d in dbs]
        _ext_loaded.wgrad_segments(dy, x, outs, True, dbs, True)
        torch.cuda.synchronize()
        for i in range(3):
            assert rel((outs[i] - olds[i]).view(seg, N), ref[i * seg:(i + 1) * seg]) < 3e-3, (T, i)
            assert rel(dbs[i] - db_olds[i], ref_b[i * seg:(i + 1) * seg]) < 3e-3, (T, i)
        print(T, seg, N, _ext_loaded.wgrad_plan(3 * seg, N, T))
    assert _ext_loaded.read_error_flag(True) == 0


# --------------------------------------------------------------------------- SHT / AMSE on the device
def test_legendre_table_matches_recurrence_oracle(_ext_loaded):
    import numpy as np

    from neural_scaling_weather_b200.utils.sht import _clenshaw_curtis_fast, legendre_orthonormal

    nlat, m0, mc = 48, 3, 20
    x, w = _clenshaw_curtis_fast(nlat)
    P, row_off = _ext_loaded.legendre_table(torch.from_numpy(x).to(DEV), torch.from_numpy(w).to(DEV), m0, mc, nlat,
                                            True)
    ref = legendre_orthonormal(m0 + mc, nlat, x) * w[None, None, :]
    P, row_off = P.cpu().double(), row_off.cpu()
    for i in range(mc):
        m = m0 + i
        rows = P[row_off[i]:row_off[i] + (nlat - m)]
        assert torch.allclose(rows, torch.from_numpy(ref[m, m:]), rtol=1e-5, atol=1e-7), m


@pytest.mark.parametrize("H,W", [(64, 128), (45, 90)])
def test_amse_cuda_fp32_matches_fp64_oracle(H, W, _ext_loaded):
    """AMSE through the device SHT (fp32 Legendre kernels, fp64 sums over m) against the float64 CPU
    oracle: loss within 1e-5 and gradient within 1e-4 relative (the fp32 mode's tested bound)."""
    import numpy as np

    from neural_scaling_weather_b200.losses import AMSELoss

    lat = np.linspace(90, -90, H + 1)[:-1]
    lon = np.arange(W) * 360.0 / W
    torch.manual_seed(3)
    x = torch.randn(2, 1, 4, H, W, dtype=torch.float64)
    y = x + 0.3 * torch.randn_like(x)
    xc = x.clone().requires_grad_()
    ref = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[H], [W]])(xc, y)
    ref.backward()
    xg = x.float().to(DEV).requires_grad_()
    out = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[H], [W]])(xg, y.float().to(DEV))
    out.backward()
    assert abs(out.item() - ref.item()) <= 1e-5 * abs(ref.item()), (out.item(), ref.item())
    assert rel(xg.grad.cpu().double(), xc.grad) < 1e-4
    assert _ext_loaded.read_error_flag(True) == 0
