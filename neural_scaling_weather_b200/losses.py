"""Training losses and evaluation metrics.

Reference behaviour (``utils/losses.py``):

* ``WeightedLoss`` (``:76-141``): squared error times optional latitude area weights
  ``[nlat_local, 1]`` and optional channel weights (GraphCast surface weights; pressure
  levels weighted ``0.001 * level``; normalised to mean 1), summed, all-reduced over
  ``sp1-sp2`` together with the pixel count, divided by ``pixels_global * B * T * C``;
* ``AMSELoss`` (``:143-228``): the same loss on a distributed SHT (no full-globe gather; see the class);
  and sums over degrees ``(|x|_l - |y|_l)^2 + 2 max(|x|_l^2, |y|_l^2) (1 - coh_l)`` with the
  m-sums weighting m >= 1 twice; mean over the leading dims;
* ``WeightedRMSE`` / ``WeightedMSE`` (``:230-305``) per (b, t, c), sp-reduced.

On CUDA the squared-error reductions are one fused kernel (forward sum, backward
gradient); the sp all-reduce is the autograd-aware reduce of
:mod:`neural_scaling_weather_b200.parallel.mappings`.
"""

from __future__ import annotations

import math
from typing import List, Optional

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .parallel import comm
from .parallel.mappings import allreduce_forward_identity_backward
from .utils.profiler import profile_range
from .utils.sht import DistributedRealSHT

GRAPHCAST_SFC = {"t2m": 1.0, "u10m": 0.1, "v10m": 0.1, "msl": 0.1, "tcwv": 0.1, "sp": 0.1}


def build_ch_weights(channel_list: List[str], sfc_weights, pressure_weights) -> torch.Tensor:
    wt = np.ones(len(channel_list))
    if sfc_weights:
        for i, var in enumerate(channel_list):
            if var in GRAPHCAST_SFC:
                wt[i] *= GRAPHCAST_SFC[var]
    if pressure_weights:
        for i, var in enumerate(channel_list):
            if var not in GRAPHCAST_SFC:
                wt[i] = 0.001 * int(var[1:])
    w = torch.from_numpy(wt)[:, None, None]
    return w / w.mean()


def get_loss(cfg, metadata):
    lf = cfg.loss.loss_func
    if lf in ("mse", "mse_weighted"):
        return WeightedLoss.instantiate_from_cfg(cfg, channels=metadata["channels"],
                                                 weights=metadata["area_weights"])
    if lf == "amse":
        return AMSELoss.instantiate_from_cfg(cfg, latitudes=metadata["global_latitudes"],
                                             longitudes=metadata["global_longitudes"],
                                             sp_shapes=metadata["sp_shapes"])
    raise NotImplementedError(f"loss {lf} is not implemented")


def get_metric(metric, metadata, temporal_average=True):
    if metric == "weighted_rmse":
        return WeightedRMSE(weights=metadata["area_weights"], temporal_average=temporal_average)
    raise NotImplementedError(f"metric {metric} is not implemented")


class WeightedLoss(nn.Module):
    @classmethod
    def instantiate_from_cfg(cls, cfg, channels, weights):
        return cls(sfc_weighting=cfg.loss.sfc_weights, pressure_weighting=cfg.loss.pressure_weights,
                   area_weighting=cfg.loss.area_weights, channels=channels, weights=weights)

    def __init__(self, sfc_weighting=False, pressure_weighting=False, area_weighting=False,
                 channels: Optional[List[str]] = None, weights: Optional[torch.Tensor] = None):
        super().__init__()
        self.area_weighting = bool(area_weighting)
        self.ch_weighting = bool(pressure_weighting or sfc_weighting)
        if self.area_weighting:
            if weights is None:
                raise AssertionError("area weighting needs weights")
            self.register_buffer("weights", torch.as_tensor(weights).float())
        if self.ch_weighting:
            if channels is None:
                raise AssertionError("channel weighting needs the channel list")
            self.register_buffer("channel_weights",
                                 build_ch_weights(channels, sfc_weighting, pressure_weighting).float())

    def forward(self, x, y):
        H, W = x.shape[-2], x.shape[-1]
        sse = ops.weighted_sse(x, y, self.weights if self.area_weighting else None,
                               self.channel_weights if self.ch_weighting else None)
        npix = global_pixel_count(H, W, x.device)
        sse = allreduce_forward_identity_backward(sse, "sp1-sp2")
        return sse / (npix * math.prod(x.shape[:-2]))


_PIXELS = {}


def global_pixel_count(h: int, w: int, device) -> float:
    """Grid points summed over the sp1 x sp2 shards (shards may be uneven).  A constant per
    local shape: computed once (one all-reduce when the spatial group is distributed) and kept
    as a Python number, so the loss adds no host-to-device copy to a step (a captured CUDA
    graph may not contain one)."""
    distributed = comm.get_size("sp1") * comm.get_size("sp2") > 1
    key = (h, w, comm.get_size("sp1"), comm.get_size("sp2"), comm.get_rank("sp1"), comm.get_rank("sp2"),
           id(comm.get_group("sp1-sp2")) if distributed else None)
    if key not in _PIXELS:
        if not distributed:
            _PIXELS[key] = float(h * w)
        else:
            t = torch.tensor(float(h * w), dtype=torch.float64, device=device)
            dist.all_reduce(t, group=comm.get_group("sp1-sp2"))
            _PIXELS[key] = float(t.item())
    return _PIXELS[key]


class AMSELoss(nn.Module):
    """Spectral AMSE (reference ``utils/losses.py:143-228``, eq. 6 of its paper): per degree l,
    ``(|x|_l - |y|_l)^2 + 2 max(|x|_l^2, |y|_l^2) (1 - coh_l)`` with ``|x|_l^2 = sum_m w_m |c_lm|^2``
    and the coherence ``coh_l = sum_m w_m Re(c^x_lm conj c^y_lm) / (|x|_l |y|_l)``, summed over l and
    averaged over the remaining dimensions.

    The reference gathers both fields to the full globe on every rank and runs a float64 SHT there.
    Here the transform is :class:`DistributedRealSHT`: no rank gathers the globe, each ``sp2`` rank
    computes its own orders m, and the per-degree sums over m are added over ``sp2``; the loss is the
    same on every rank.  CPU: float64 throughout; CUDA: the SHT in float32 (device kernels), the sums
    over m in float64.
    """

    @classmethod
    def instantiate_from_cfg(cls, cfg, latitudes, longitudes, sp_shapes):
        return cls(latitudes=latitudes, longitudes=longitudes, sp_shapes=sp_shapes,
                   loss_type=cfg.loss.loss_func)

    def __init__(self, latitudes=None, longitudes=None, sp_shapes=None, loss_type=None):
        super().__init__()
        self.latitudes, self.longitudes = latitudes, longitudes
        self.sp_shapes = sp_shapes
        self.loss_type = loss_type
        lat_shapes, lon_shapes = (sp_shapes if sp_shapes is not None else ([len(latitudes)], [len(longitudes)]))
        self.sht = DistributedRealSHT(len(latitudes), len(longitudes), lat_shapes, lon_shapes)

    def forward(self, x, y):
        with torch.autocast(x.device.type, enabled=False):
            cx = self.sht(x)
            cy = self.sht(y)
            wm = self.sht.order_weights(cx.device, torch.float64)
            xs = (cx[..., 0] ** 2 + cx[..., 1] ** 2).double()
            ys = (cy[..., 0] ** 2 + cy[..., 1] ** 2).double()
            xy = (cx[..., 0] * cy[..., 0] + cx[..., 1] * cy[..., 1]).double()
            sums = torch.stack([(xs * wm).sum(-1), (ys * wm).sum(-1), (xy * wm).sum(-1)])
            if self.sht.sp2 > 1:
                sums = allreduce_forward_identity_backward(sums, "sp2")
            xn2, yn2, coh = sums[0], sums[1], sums[2]
            xn, yn = torch.sqrt(xn2), torch.sqrt(yn2)
            coh = coh / (xn * yn)
            loss = (xn - yn) ** 2 + 2 * torch.maximum(xn2, yn2) * (1 - coh)
            return loss.sum(-1).mean()


class WeightedRMSE(nn.Module):
    def __init__(self, weights=None, temporal_average=True):
        super().__init__()
        if weights is None:
            raise AssertionError("weights needed")
        self.temporal_average = temporal_average
        self.register_buffer("weights", torch.as_tensor(weights).float())

    def forward(self, pred, target):
        with profile_range("weighted_rmse"):
            se_sum = ops.weighted_se_per_channel(pred, target, self.weights)
            count = global_pixel_count(pred.shape[-2], pred.shape[-1], pred.device)
            se_sum = allreduce_forward_identity_backward(se_sum, "sp1-sp2")
            rmse = torch.sqrt(se_sum / count)
            if self.temporal_average:
                while rmse.dim() > 1:
                    rmse = rmse.mean(dim=0)
            else:
                rmse = rmse.mean(dim=0)
            return rmse


class WeightedMSE(nn.Module):
    def __init__(self, weights=None, temporal_average=True):
        super().__init__()
        self.temporal_average = temporal_average
        self.weights = weights

    def forward(self, pred, target):
        w = self.weights if self.weights is not None else torch.ones(1, 1, device=pred.device)
        se_sum = ops.weighted_se_per_channel(pred, target, w)
        count = global_pixel_count(pred.shape[-2], pred.shape[-1], pred.device)
        se_sum = allreduce_forward_identity_backward(se_sum, "sp1-sp2")
        mse = se_sum / count
        if self.temporal_average:
            while mse.dim() > 1:
                mse = mse.mean(dim=0)
        else:
            mse = mse.mean(dim=0)
        return mse


def anomaly_correlation(pred, target, area_w, climatology=None):
    """Latitude-weighted anomaly correlation per (b, t, c) over the local grid, sp-reduced.

    ACC = sum w a_p a_t / sqrt(sum w a_p^2 * sum w a_t^2) with anomalies a = field - clim;
    for standardised synthetic data the climatology is 0.
    """
    p = pred.float()
    t = target.float()
    if climatology is not None:
        p = p - climatology
        t = t - climatology
    w = area_w.float()
    num = (w * p * t).sum(dim=(-1, -2))
    dp = (w * p * p).sum(dim=(-1, -2))
    dt = (w * t * t).sum(dim=(-1, -2))
    stacked = torch.stack([num, dp, dt])
    stacked = allreduce_forward_identity_backward(stacked, "sp1-sp2")
    return stacked[0] / torch.sqrt(stacked[1] * stacked[2]).clamp_min(1e-30)
