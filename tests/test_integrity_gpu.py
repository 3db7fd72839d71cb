"""Out-of-bounds writes and run-to-run determinism of the CUDA kernels.

Guard regions: a kernel's output is placed inside a larger buffer filled with a sentinel, and
the sentinel must survive the call (tile edges and TMA stores clipped at ragged M / N are
where an overrun would show).  Determinism: the same inputs give bit-identical results on a
second run (no atomics in the reductions; per-CTA partials are summed in a fixed order).
"""

import pytest
import torch

from neural_scaling_weather_b200.ops import _ext

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

DEV = "cuda"
GUARD = 256  # elements on each side (keeps the output 16-byte aligned)


def _guarded(M, N, dtype, sentinel):
    buf = torch.full((GUARD + M * N + GUARD,), sentinel, device=DEV, dtype=dtype)
    return buf, buf[GUARD:GUARD + M * N].view(M, N)


def _guards_intact(buf, sentinel):
    return bool((buf[:GUARD] == sentinel).all()) and bool((buf[-GUARD:] == sentinel).all())


@pytest.mark.parametrize("M,N,K", [(777, 1000, 256), (129, 40, 96), (4096, 1024, 512), (300, 1120, 1168)])
@pytest.mark.parametrize("impl", [1, 2])
def test_gemm_writes_stay_inside_out(M, N, K, impl):
    ext = _ext.require()
    torch.manual_seed(3)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.1
    bias = torch.randn(N, device=DEV)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    ref = a.float() @ b.float().t()
    sentinel = 1234.5
    buf, out = _guarded(M, N, torch.bfloat16, sentinel)
    ext.gemm(a, b, bias, res, out=out, impl=impl)
    assert _guards_intact(buf, sentinel)
    assert ((out.float() - (ref + bias + res.float())).norm() / ref.norm()).item() < 1e-2
    # fp32 accumulation into a caller's buffer
    buf32, out32 = _guarded(M, N, torch.float32, sentinel)
    out32.zero_()
    ext.gemm(a, b, None, None, 0, 0, None, True, 1.0, out32, True, impl=impl)
    assert _guards_intact(buf32, sentinel)
    assert ((out32 - ref).norm() / ref.norm()).item() < 1e-3
    assert ext.read_error_flag(True) == 0


def test_gemm_rejects_a_wrong_output_tensor():
    ext = _ext.require()
    a = torch.randn(256, 64, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(128, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="out"):
        ext.gemm(a, b, out=torch.empty(256, 64, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="out"):
        ext.gemm(a, b, out=torch.empty(256, 128, device=DEV, dtype=torch.float32))
    with pytest.raises(RuntimeError, match="out"):
        ext.gemm(a, b, out=torch.empty(128, 256, device=DEV, dtype=torch.bfloat16).t())


def test_attention_is_deterministic():
    ext = _ext.require()
    torch.manual_seed(4)
    B, T, H, W, nh, hd = 1, 1, 90, 360, 4, 64
    C = nh * hd
    qkv = torch.randn(B * T * H * W, 3 * C, device=DEV).bfloat16()
    qw = 1 + 0.1 * torch.randn(hd, device=DEV)
    kw = 1 + 0.1 * torch.randn(hd, device=DEV)
    gi = [B, T, H, W, nh, hd, 9, 18, 4, 9, 1, 4, 0, H]
    o1, l1 = ext.window_attn_fwd(qkv, qw, kw, gi, hd ** -0.5)
    o2, l2 = ext.window_attn_fwd(qkv, qw, kw, gi, hd ** -0.5)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    dout = torch.randn_like(o1)
    g1 = ext.window_attn_bwd(qkv, qw, kw, o1, dout, l1, gi, hd ** -0.5)
    g2 = ext.window_attn_bwd(qkv, qw, kw, o1, dout, l1, gi, hd ** -0.5)
    for x, y in zip(g1, g2):
        assert torch.equal(x, y)
    assert ext.read_error_flag(True) == 0


def test_model_step_is_deterministic():
    """Two forward + backward passes of the same model on the same batch give bit-identical
    gradients (the fused kernels and the column sums reduce in a fixed order)."""
    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.models.swin import get_model
    from neural_scaling_weather_b200.utils.misc import create_dummy_metadata

    torch.manual_seed(0)
    H, W, Cc = 72, 144, 5
    md = create_dummy_metadata(H, W, Cc)
    cfg = C.create(dict(
        model=dict(arch="swin", embed_dim=128, patch_size=4, depth=2, window_size=[9, 18], num_heads=2,
                   dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=["a", "b", "c"]),
        train=dict(temporal_context_window=1, num_rollout_steps=1),
        parallelism=dict(use_transformer_engine=False)))
    model = get_model(cfg, md).to(DEV)
    x = torch.randn(1, 1, Cc + 3, H, W, device=DEV)
    y = torch.randn(1, 1, Cc, H, W, device=DEV)

    def grads():
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(x)
        ((out.float() - y) ** 2).mean().backward()
        return [p.grad.clone() for p in model.parameters()]

    g1, g2 = grads(), grads()
    for (name, _), a, b in zip(model.named_parameters(), g1, g2):
        assert torch.equal(a, b), name
    assert _ext.require().read_error_flag(True) == 0


def test_bounded_wait_reports_a_peer_that_never_signals():
    """The fused tensor-parallel GEMM + all-reduce waits for every peer's per-tile flag with a
    time budget.  Driven on one GPU with a stand-in peer whose flags nothing ever sets, the
    kernel must give up, record the wait timeout in the device error word and return, leaving
    the context usable (no fault, trap or hang is involved)."""
    from neural_scaling_weather_b200.parallel.symm import FLAG_BASE

    ext = _ext.require()
    ext.read_error_flag(True)
    torch.manual_seed(5)
    M, N, K = 256, 256, 64
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    tiles = (M // 128) * (N // 256)
    parts = [torch.zeros(2 * M * N, device=DEV, dtype=torch.bfloat16) for _ in range(2)]  # a slot per rank
    flags = [torch.zeros(FLAG_BASE + 2 * tiles, device=DEV, dtype=torch.int32) for _ in range(2)]
    ext.gemm_allreduce(a, b, None, None, [p.data_ptr() for p in parts], [f.data_ptr() for f in flags], 0)
    torch.cuda.synchronize()
    assert ext.read_error_flag(True) == 1  # wait timeout
    # the context still works
    d = ext.gemm(a, b, impl=1)
    ref = a.float() @ b.float().t()
    assert ((d.float() - ref).norm() / ref.norm()).item() < 1e-2
    assert ext.read_error_flag(True) == 0


def test_bounded_wait_in_the_halo_roll():
    """The sharded roll's gather waits for the peer's ready flag with a time budget.  On one GPU with a
    stand-in peer (its band buffer and flag words are local tensors nothing else writes) the wait runs
    out: the timeout lands in the device error word, the kernels return and the context stays usable."""
    ext = _ext.require()
    ext.read_error_flag(True)
    H, W, C = 8, 16, 64  # the global grid: 8 x 16 patches split over sp2 = 2
    x = torch.randn(1, 1, H, W // 2, C, device=DEV, dtype=torch.bfloat16)
    out = torch.empty_like(x)
    geom, h_off, w_off, coord1, coord2 = [1, 2, 0, -3, 0], [0, H], [0, W // 2, W], [0, 0], [0, 1]
    nb = ext.halo_band_bytes(x, geom, h_off, w_off, coord1, coord2)
    bands = [torch.zeros(max(nb, 16), device=DEV, dtype=torch.uint8) for _ in range(2)]
    flags = [torch.zeros(48, device=DEV, dtype=torch.int32) for _ in range(2)]
    ext.halo_roll(x, out, geom, h_off, w_off, coord1, coord2, [b.data_ptr() for b in bands],
                  [f.data_ptr() for f in flags])
    torch.cuda.synchronize()
    assert ext.read_error_flag(True) == 1  # wait timeout
    # the locally sourced part of the roll is complete
    assert torch.equal(out[:, :, :, : W // 2 - 3], x[:, :, :, 3:])
    y = torch.randn(64, 64, device=DEV)
    assert torch.allclose(y.sum(0), y.t().sum(1))  # the context still works
    assert ext.read_error_flag(True) == 0


def test_bounded_wait_in_the_data_parallel_reduction():
    """The peer-memory data-parallel reduction announces a gradient bucket and waits for every rank's
    announcement with a time budget.  With a stand-in peer that never announces, the kernel gives up,
    records the timeout and returns; the context stays usable."""
    ext = _ext.require()
    ext.read_error_flag(True)
    n, slots = 1024, 2
    grads = [torch.randn(n, device=DEV) for _ in range(2)]
    datas = [torch.zeros(n, device=DEV) for _ in range(2)]
    flags = [torch.zeros(16 + 2 * slots, device=DEV, dtype=torch.int32) for _ in range(2)]
    keep = grads[0].clone()
    ext.dp_reduce([g.data_ptr() for g in grads], [d.data_ptr() for d in datas], [],
                  [f.data_ptr() for f in flags], 0, slots, 0, 1, 0, n, 0.5)
    torch.cuda.synchronize()
    assert ext.read_error_flag(True) == 1
    assert torch.equal(grads[0], keep)  # nothing was summed
    assert ext.read_error_flag(True) == 0
