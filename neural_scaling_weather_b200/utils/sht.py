"""Real spherical harmonic transform on an equiangular (pole-to-pole) lat-lon grid.

This is the transform the reference obtains from ``torch_harmonics.RealSHT(nlat, nlon,
grid="equiangular")`` (``utils/losses.py:171``, ``utils/misc_utils.py:103-123``),
re-derived here from its mathematical definition because that package is unavailable:

* grid: ``nlat`` colatitudes ``theta_k = pi k / (nlat - 1)`` (north pole first) and
  ``nlon`` longitudes ``phi_j = 2 pi j / nlon``;
* longitude integral: ``int f e^{-i m phi} dphi ~= 2 pi * rfft(f, norm="forward")[m]``;
* latitude integral: Clenshaw-Curtis quadrature on ``x = cos(theta)`` (Trefethen 2008,
  "Is Gauss quadrature better than Clenshaw-Curtis?", eq. 2.1 closed form);
* basis: orthonormal associated Legendre functions ``Pbar_l^m`` (``2 pi int Pbar^2 dx = 1``)
  with the Condon-Shortley phase, from the standard stable recurrences (sectoral seed
  ``Pbar_mm = -sqrt((2m+1)/(2m)) sin(theta) Pbar_{m-1,m-1}``, then the three-term
  recurrence in ``l`` with coefficients ``a_lm = sqrt((4l^2-1)/(l^2-m^2))``,
  ``b_lm = sqrt(((l-1)^2-m^2)/(4(l-1)^2-1))``; Holmes & Featherstone 2002).

Coefficients ``c[l, m] = sum_k w_k Pbar_lm(x_k) 2 pi F_m(theta_k)`` for ``l < lmax = nlat``,
``m < mmax = nlon // 2 + 1``.  Everything is float64 by default, as in the reference.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch


def clenshaw_curtis(n: int):
    """Nodes ``x_k = cos(theta_k)`` (theta ascending from 0) and weights on [-1, 1]."""
    if n == 1:
        return np.array([1.0]), np.array([2.0])
    N = n - 1
    theta = np.pi * np.arange(n) / N
    w = np.zeros(n)
    jmax = N // 2
    for k in range(n):
        s = 0.0
        for j in range(1, jmax + 1):
            b = 1.0 if (2 * j == N) else 2.0
            s += b / (4.0 * j * j - 1.0) * math.cos(2.0 * j * theta[k])
        c = 1.0 if k in (0, N) else 2.0
        w[k] = c / N * (1.0 - s)
    return np.cos(theta), w


def _clenshaw_curtis_fast(n: int):
    """Vectorised form of :func:`clenshaw_curtis` (identical values)."""
    if n <= 2:
        return clenshaw_curtis(n)
    N = n - 1
    theta = np.pi * np.arange(n) / N
    j = np.arange(1, N // 2 + 1)
    b = np.where(2 * j == N, 1.0, 2.0)
    s = (b / (4.0 * j * j - 1.0))[None, :] * np.cos(2.0 * np.outer(theta, j))
    c = np.full(n, 2.0)
    c[0] = c[-1] = 1.0
    w = c / N * (1.0 - s.sum(axis=1))
    return np.cos(theta), w


def legendre_orthonormal(mmax: int, lmax: int, x: np.ndarray, csphase: bool = True) -> np.ndarray:
    """``P[m, l, k] = Pbar_l^m(x_k)`` for ``m < mmax``, ``l < lmax`` (zero for m > l)."""
    nk = x.shape[0]
    P = np.zeros((mmax, lmax, nk))
    sint = np.sqrt(np.clip(1.0 - x * x, 0.0, None))
    pmm = np.full(nk, 1.0 / math.sqrt(4.0 * math.pi))
    for m in range(0, min(mmax, lmax)):
        if m > 0:
            pmm = math.sqrt((2.0 * m + 1.0) / (2.0 * m)) * sint * pmm
            if csphase:
                pmm = -pmm
        P[m, m] = pmm
        if m + 1 < lmax:
            p_lm1 = pmm
            p_l = math.sqrt(2.0 * m + 3.0) * x * pmm
            P[m, m + 1] = p_l
            for l in range(m + 2, lmax):
                a = math.sqrt((4.0 * l * l - 1.0) / (l * l - m * m))
                b = math.sqrt(((l - 1.0) ** 2 - m * m) / (4.0 * (l - 1.0) ** 2 - 1.0))
                p_new = a * (x * p_l - b * p_lm1)
                p_lm1, p_l = p_l, p_new
                P[m, l] = p_l
    return P


@lru_cache(maxsize=8)
def _sht_weights_np(nlat: int, nlon: int, lmax: int, mmax: int) -> np.ndarray:
    x, w = _clenshaw_curtis_fast(nlat)
    P = legendre_orthonormal(mmax, lmax, x)
    return P * w[None, None, :]  # (mmax, lmax, nlat)


class RealSHT(torch.nn.Module):
    """Forward real SHT: (..., nlat, nlon) real -> (..., lmax, mmax) complex."""

    def __init__(self, nlat: int, nlon: int, lmax: int | None = None, mmax: int | None = None,
                 grid: str = "equiangular", dtype=torch.float64):
        super().__init__()
        if grid != "equiangular":
            raise NotImplementedError("only the equiangular grid is implemented")
        self.nlat, self.nlon = nlat, nlon
        self.lmax = lmax or nlat
        self.mmax = mmax or nlon // 2 + 1
        wt = torch.from_numpy(_sht_weights_np(nlat, nlon, self.lmax, self.mmax)).to(dtype)
        self.register_buffer("weights", wt, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.to(self.weights.dtype)
        f = 2.0 * math.pi * torch.fft.rfft(x, dim=-1, norm="forward")[..., : self.mmax]
        # (..., k, m) x (m, l, k) -> (..., l, m)
        re = torch.einsum("...km,mlk->...lm", f.real, self.weights)
        im = torch.einsum("...km,mlk->...lm", f.imag, self.weights)
        return torch.complex(re, im)


def power_spectrum(x: torch.Tensor, sht: RealSHT | None = None) -> torch.Tensor:
    """Angular power per degree ``sum_m |c_lm|^2 / (2l+1)`` (``utils/misc_utils.py:103-123``).

    x: (b, c, lat, lon) or (b, t, c, lat, lon) (the first time step is used).
    """
    if x.dim() > 4:
        x = x[:, 0]
    nlat, nlon = x.shape[-2:]
    if sht is None:
        sht = RealSHT(nlat, nlon).to(x.device)
    c = sht(x.to(torch.float64))
    p = c.real ** 2 + c.imag ** 2
    return p.sum(dim=-1) / (2 * torch.arange(sht.lmax, device=x.device, dtype=torch.float64) + 1)
