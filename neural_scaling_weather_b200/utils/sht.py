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
``m < mmax = nlon // 2 + 1``.  Normalisation as torch_harmonics' ``RealSHT(norm="ortho")``: a
field ``2 Pbar_lm(cos theta) cos(m phi)`` has ``c[l, m] = 1``; orders ``m >= lmax`` (torch_harmonics
stops at ``min(lmax, nlon // 2 + 1)``) have ``Pbar = 0`` and contribute nothing.

:class:`RealSHT` is the float64 single-field transform (the CPU oracle).  :class:`DistributedRealSHT`
transforms a field sharded over the ``sp1`` (latitude) x ``sp2`` (longitude) groups without
gathering the globe: the longitudes are gathered within ``sp2`` only, each ``sp2`` rank keeps its
own slice of the orders m after the rFFT, the Legendre sum runs over the rank's own latitudes, and
the partial sums are added over ``sp1``.  On CUDA the Legendre table (packed for l >= m) is built
once on the device and the contraction and its adjoint run in the extension's fp32 kernels
(``ops/csrc/sht.cu``); on CPU they are float64 einsums.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch

from ..parallel import comm
from ..parallel.helpers import compute_split_shapes
from ..parallel.mappings import allgather_forward_reducescatter_backward, allreduce_forward_identity_backward


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


class _LegendreCUDA(torch.autograd.Function):
    """C[m, l, :] = sum_k P[m, l, k] F[m, k, :] on the extension's kernels; backward is the adjoint."""

    @staticmethod
    def forward(ctx, F, P, row_off, m0, L):
        from ..ops._ext import require

        ext = require()
        ctx.save_for_backward(P, row_off)
        ctx.m0, ctx.K = m0, F.shape[1]
        return ext.legendre_fwd(P, row_off, F.contiguous(), m0, L)

    @staticmethod
    def backward(ctx, dC):
        from ..ops._ext import require

        P, row_off = ctx.saved_tensors
        return require().legendre_bwd(P, row_off, dC.contiguous(), ctx.m0, ctx.K), None, None, None, None


class DistributedRealSHT(torch.nn.Module):
    """Real SHT of a field sharded over ``sp1`` (latitudes, ``lat_shapes``) x ``sp2`` (longitudes,
    ``lon_shapes``).  ``forward(x)`` maps the local shard ``(..., H_loc, W_loc)`` to this rank's orders
    ``[m_lo, m_hi)`` of the full coefficients as real pairs ``(..., lmax, m_hi - m_lo, 2)``, identical on
    the ``sp1`` ranks of a ``sp2`` rank.  Gradients flow back to the local shard."""

    def __init__(self, nlat: int, nlon: int, lat_shapes=None, lon_shapes=None, lmax: int | None = None,
                 mmax: int | None = None):
        super().__init__()
        self.nlat, self.nlon = nlat, nlon
        self.lmax = lmax or nlat
        self.mmax = mmax or nlon // 2 + 1
        self.lat_shapes = list(lat_shapes) if lat_shapes is not None else [nlat]
        self.lon_shapes = list(lon_shapes) if lon_shapes is not None else [nlon]
        self.sp1 = comm.get_size("sp1") if len(self.lat_shapes) > 1 else 1
        self.sp2 = comm.get_size("sp2") if len(self.lon_shapes) > 1 else 1
        r1 = comm.get_rank("sp1") if self.sp1 > 1 else 0
        r2 = comm.get_rank("sp2") if self.sp2 > 1 else 0
        self.k_lo = sum(self.lat_shapes[:r1])
        self.k_hi = self.k_lo + self.lat_shapes[r1]
        m_shapes = compute_split_shapes(self.mmax, self.sp2)
        self.m_lo = sum(m_shapes[:r2])
        self.m_hi = self.m_lo + m_shapes[r2]
        x, w = _clenshaw_curtis_fast(nlat)
        self._x, self._w = x[self.k_lo:self.k_hi].copy(), w[self.k_lo:self.k_hi].copy()
        self._cpu_w = None  # float64 (m, l, k) table of the CPU path, built on first use
        self._cuda = {}     # device -> (P packed float32, row offsets)

    # The tables are built on first use, which may come inside torch.inference_mode (validation, a
    # rollout); they are built with inference mode off so that a later training step can save them
    # for its backward.
    def _cpu_table(self):
        if self._cpu_w is None:
            P = legendre_orthonormal(self.m_hi, self.lmax, self._x)[self.m_lo:self.m_hi]
            with torch.inference_mode(False):
                self._cpu_w = torch.from_numpy(P * self._w[None, None, :])
        return self._cpu_w

    def _cuda_table(self, device):
        key = (device.type, device.index)
        if key not in self._cuda:
            from ..ops._ext import require

            x = torch.from_numpy(self._x).to(device)
            w = torch.from_numpy(self._w).to(device)
            m_count = max(0, min(self.m_hi, self.lmax) - self.m_lo)
            with torch.inference_mode(False):
                self._cuda[key] = tuple(require().legendre_table(x.clone(), w.clone(), self.m_lo, m_count,
                                                                 self.lmax, True))
        return self._cuda[key]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sp2 > 1:
            x = allgather_forward_reducescatter_backward(x, -1, self.lon_shapes, "sp2")
        lead = x.shape[:-2]
        K = x.shape[-2]
        mc = self.m_hi - self.m_lo
        if x.is_cuda:
            with torch.autocast("cuda", enabled=False):
                f = 2.0 * math.pi * torch.fft.rfft(x.float(), dim=-1, norm="forward")[..., self.m_lo:self.m_hi]
                R = math.prod(lead)
                P, row_off = self._cuda_table(x.device)
                mt = row_off.numel()  # orders below lmax (higher ones have no coefficients)
                F = torch.view_as_real(f.reshape(R, K, mc)[..., :mt].contiguous())  # (R, K, mt, 2)
                F = F.permute(2, 1, 3, 0).reshape(mt, K, 2 * R)
                C = _LegendreCUDA.apply(F, P, row_off, self.m_lo, self.lmax)  # (mt, L, 2R)
                c = C.view(mt, self.lmax, 2, R).permute(3, 1, 0, 2)  # (R, L, mt, 2)
                if mt < mc:
                    c = torch.cat([c, c.new_zeros(R, self.lmax, mc - mt, 2)], dim=2)
                c = c.reshape(*lead, self.lmax, mc, 2)
        else:
            f = 2.0 * math.pi * torch.fft.rfft(x.to(torch.float64), dim=-1, norm="forward")[..., self.m_lo:self.m_hi]
            W = self._cpu_table()
            re = torch.einsum("...km,mlk->...lm", f.real, W)
            im = torch.einsum("...km,mlk->...lm", f.imag, W)
            c = torch.stack([re, im], dim=-1)
        if self.sp1 > 1:
            c = allreduce_forward_identity_backward(c, "sp1")
        return c

    def order_weights(self, device, dtype) -> torch.Tensor:
        """Weight of each local order in a sum over all m of a real field's spectrum: 1 for m = 0
        and 2 for m > 0 (the negative orders)."""
        w = torch.full((self.m_hi - self.m_lo,), 2.0, device=device, dtype=dtype)
        if self.m_lo == 0:
            w[0] = 1.0
        return w


def power_spectrum_distributed(x: torch.Tensor, sht: DistributedRealSHT) -> torch.Tensor:
    """:func:`power_spectrum` of a sharded field (the same values on every rank of the sp groups)."""
    if x.dim() > 4:
        x = x[:, 0]
    c = sht(x)
    p = (c[..., 0].double() ** 2 + c[..., 1].double() ** 2).sum(dim=-1)
    if sht.sp2 > 1:
        p = allreduce_forward_identity_backward(p, "sp2")
    return p / (2 * torch.arange(sht.lmax, device=x.device, dtype=torch.float64) + 1)


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
