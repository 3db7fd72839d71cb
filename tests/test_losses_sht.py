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
