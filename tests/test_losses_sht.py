"""Spherical harmonic transform, AMSE loss, metrics (CPU)."""

import math

import numpy as np
import pytest
import torch

from neural_scaling_weather_b200.losses import AMSELoss, WeightedLoss, anomaly_correlation
from neural_scaling_weather_b200.utils.sht import (
    RealSHT,
    _clenshaw_curtis_fast,
    clenshaw_curtis,
    legendre_orthonormal,
    power_spectrum,
)


def test_clenshaw_curtis_integrates_polynomials():
    for n in (5, 16, 33):
        x, w = clenshaw_curtis(n)
        x2, w2 = _clenshaw_curtis_fast(n)
        assert np.allclose(w, w2) and np.allclose(x, x2)
        assert w.sum() == pytest.approx(2.0)
        for k in range(0, n - 1):
            exact = 0.0 if k % 2 else 2.0 / (k + 1)
            assert (w * x ** k).sum() == pytest.approx(exact, abs=1e-12)


def test_legendre_orthonormality():
    n = 64
    x, w = _clenshaw_curtis_fast(n)
    P = legendre_orthonormal(8, 20, x)
    for m in range(8):
        G = 2 * math.pi * (P[m] * w) @ P[m].T  # (l, l')
        for l in range(m, 20):
            for l2 in range(m, 20):
                assert G[l, l2] == pytest.approx(1.0 if l == l2 else 0.0, abs=1e-10)


def test_sht_recovers_single_harmonic():
    nlat, nlon = 33, 64
    sht = RealSHT(nlat, nlon)
    x, _ = _clenshaw_curtis_fast(nlat)
    P = legendre_orthonormal(6, 10, x)
    phi = torch.arange(nlon, dtype=torch.float64) * 2 * math.pi / nlon
    l, m = 5, 3
    # real field = Y_lm + conj(Y_lm) = 2 Pbar_lm cos(m phi)
    f = 2 * torch.from_numpy(P[m, l])[:, None] * torch.cos(m * phi)[None, :]
    c = sht(f)
    assert abs(c[l, m].real.item() - 1.0) < 1e-10
    c[l, m] = 0
    # Clenshaw-Curtis on n nodes is exact to polynomial degree n-1: products with degrees
    # near lmax alias (as in any equiangular SHT), so check the well-resolved half.
    assert c[: nlat // 2].abs().max().item() < 1e-10


def test_amse_zero_for_identical_fields_and_positive_otherwise():
    lat = np.linspace(90, -90, 17)[:-1]
    lon = np.arange(32) * 360 / 32
    loss = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[16], [32]], loss_type="amse")
    torch.manual_seed(0)
    x = torch.randn(2, 1, 3, 16, 32)
    assert loss(x, x).item() == pytest.approx(0.0, abs=1e-10)
    y = x + 0.3 * torch.randn_like(x)
    v = loss(x, y)
    assert v.item() > 0
    xr = x.clone().requires_grad_()
    loss(xr, y).backward()
    assert torch.isfinite(xr.grad).all()


def test_power_spectrum_shapes():
    x = torch.randn(2, 3, 16, 32)
    p = power_spectrum(x)
    assert p.shape == (2, 3, 16) and (p >= 0).all()


def test_acc_perfect_and_anti():
    aw = torch.rand(8, 1)
    x = torch.randn(1, 1, 2, 8, 16)
    assert torch.allclose(anomaly_correlation(x, x, aw), torch.ones(1, 1, 2))
    assert torch.allclose(anomaly_correlation(x, -x, aw), -torch.ones(1, 1, 2))


def test_weighted_loss_manual():
    aw = torch.rand(4, 1)
    x, y = torch.randn(1, 1, 2, 4, 5), torch.randn(1, 1, 2, 4, 5)
    v = WeightedLoss(area_weighting=True, weights=aw)(x, y)
    assert v.item() == pytest.approx((((x - y) ** 2) * aw).mean().item(), rel=1e-6)


# --------------------------------------------------------------------------- distributed SHT / AMSE
def test_distributed_sht_on_one_rank_matches_realsht():
    from neural_scaling_weather_b200.utils.sht import DistributedRealSHT

    torch.manual_seed(1)
    x = torch.randn(2, 3, 17, 32, dtype=torch.float64)
    ref = RealSHT(17, 32)(x)
    c = DistributedRealSHT(17, 32)(x)
    assert c.shape == (2, 3, 17, 17, 2)
    assert torch.allclose(c[..., 0], ref.real, atol=1e-12) and torch.allclose(c[..., 1], ref.imag, atol=1e-12)


def test_amse_gradient_matches_finite_differences():
    lat = np.linspace(90, -90, 9)[:-1]
    lon = np.arange(16) * 360 / 16
    loss = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[8], [16]], loss_type="amse")
    torch.manual_seed(2)
    x = torch.randn(1, 1, 2, 8, 16, dtype=torch.float64, requires_grad=True)
    y = torch.randn(1, 1, 2, 8, 16, dtype=torch.float64)
    assert torch.autograd.gradcheck(lambda a: loss(a, y), (x,), eps=1e-6, atol=1e-6, rtol=1e-4)


def _amse_worker(rank, world, dp, sp1, sp2):
    import numpy as np
    import torch
    import torch.distributed as dist

    from neural_scaling_weather_b200.losses import AMSELoss
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes, offsets

    comm.init_model_parallel_info(tp=1, sp1=sp1, sp2=sp2, dp=dp)
    B, T, C, H, W = 4, 2, 3, 16, 32
    g = torch.Generator().manual_seed(0)
    pred = torch.randn(B, T, C, H, W, dtype=torch.float64, generator=g)
    targ = pred + 0.5 * torch.randn(B, T, C, H, W, dtype=torch.float64, generator=g)
    lat = np.linspace(90, -90, H + 1)[:-1]
    lon = np.arange(W) * 360.0 / W
    # single-rank oracle (no sharded shapes: no collectives)
    p = pred.clone().requires_grad_()
    ref = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[[H], [W]])(p, targ)
    ref.backward()
    # sharded: batch over dp, latitudes over sp1, longitudes over sp2
    hs, ws = compute_split_shapes(H, sp1), compute_split_shapes(W, sp2)
    r1, r2, rd = comm.get_rank("sp1"), comm.get_rank("sp2"), comm.get_rank("dp")
    h0, w0, b0 = offsets(hs)[r1], offsets(ws)[r2], rd * (B // dp)
    sl = (slice(b0, b0 + B // dp), slice(None), slice(None), slice(h0, h0 + hs[r1]), slice(w0, w0 + ws[r2]))
    pl = pred[sl].clone().requires_grad_()
    loss = AMSELoss(latitudes=lat, longitudes=lon, sp_shapes=[hs, ws])(pl, targ[sl])
    loss.backward()
    v = loss.detach().clone()
    if dp > 1:
        dist.all_reduce(v, group=comm.get_group("dp"))
        v /= dp
    assert abs(v.item() - ref.item()) <= 1e-10 * abs(ref.item()), (v.item(), ref.item())
    # the local loss is a mean over the local batch: its gradient is dp times the global one
    assert torch.allclose(pl.grad / dp, p.grad[sl], rtol=1e-9, atol=1e-14)


@pytest.mark.parametrize("dp,sp1,sp2", [(1, 2, 1), (1, 1, 2), (2, 2, 1), (1, 2, 2)])
def test_amse_sharded_matches_single_rank(dp, sp1, sp2):
    """As the reference's tests/test_losses.py: AMSE value and gradient with the batch split over dp
    and the grid over sp1 x sp2 equal the single-rank result (here without any full-globe gather)."""
    from tests.dist_utils import run

    run(_amse_worker, dp * sp1 * sp2, dp, sp1, sp2)


def _spectrum_worker(rank, world, sp1, sp2):
    import numpy as np
    import torch

    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes, offsets
    from neural_scaling_weather_b200.utils.sht import DistributedRealSHT, power_spectrum, power_spectrum_distributed

    comm.init_model_parallel_info(tp=1, sp1=sp1, sp2=sp2, dp=1)
    H, W = 12, 24
    x = torch.randn(2, 3, H, W, dtype=torch.float64, generator=torch.Generator().manual_seed(5))
    ref = power_spectrum(x)
    hs, ws = compute_split_shapes(H, sp1), compute_split_shapes(W, sp2)
    r1, r2 = comm.get_rank("sp1"), comm.get_rank("sp2")
    xl = x[..., offsets(hs)[r1]:offsets(hs)[r1] + hs[r1], offsets(ws)[r2]:offsets(ws)[r2] + ws[r2]]
    p = power_spectrum_distributed(xl, DistributedRealSHT(H, W, hs, ws))
    assert torch.allclose(p, ref, rtol=1e-10, atol=1e-14)


def test_power_spectrum_sharded_matches_single_rank():
    from tests.dist_utils import run

    run(_spectrum_worker, 4, 2, 2)


def test_sht_table_first_built_in_inference_mode_serves_training():
    """The Legendre table is built on first use; when that use is a validation pass under
    torch.inference_mode, a later training step must still be able to save it for its backward."""
    from neural_scaling_weather_b200.utils.sht import DistributedRealSHT

    sht = DistributedRealSHT(8, 16)
    x = torch.randn(2, 8, 16, dtype=torch.float64)
    with torch.inference_mode():
        sht(x)
    xg = x.clone().requires_grad_()
    sht(xg).square().sum().backward()
    assert xg.grad is not None and torch.isfinite(xg.grad).all()
