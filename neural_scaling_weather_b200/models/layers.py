"""Parameter-holding layers annotated with their distributed role.

Every parameter carries ``comm_metadata = {"sharded": [...], "shared": [...],
"reduce": [...]}`` as in ``models/layer_helpers.py:8-172`` of the reference:

* ``sharded``: per tensor dimension, the group it is split over (``None`` if whole);
* ``shared``: groups in which every rank holds the same copy (broadcast at start-up);
* ``reduce``: groups over which its gradient must be summed (besides the dp average).

Module and parameter names follow the reference (``proj.conv.weight``, ``norm.weight``,
``weight``, ``bias``) so checkpoints are interchangeable.  The compute is not done here:
the blocks call the fused operators in :mod:`neural_scaling_weather_b200.ops`.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..parallel import comm


def trunc_normal_(t: torch.Tensor, std: float = 0.02, mean: float = 0.0,
                  a: float = -2.0, b: float = 2.0) -> torch.Tensor:
    """Truncated normal init with absolute bounds ``[a, b]`` (as timm's helper)."""
    return nn.init.trunc_normal_(t, mean=mean, std=std, a=a, b=b)


def drop_path(x: torch.Tensor, drop_prob: float = 0.0, training: bool = False) -> torch.Tensor:
    """Stochastic depth per sample (timm's ``drop_path``; reference ``models/timm_helpers.py``,
    unused by the Swin blocks there as here): zero whole samples with probability ``drop_prob``
    and rescale the rest by ``1 / (1 - drop_prob)``."""
    if drop_prob == 0.0 or not training:
        return x
    keep = 1.0 - drop_prob
    mask = x.new_empty((x.shape[0],) + (1,) * (x.ndim - 1)).bernoulli_(keep)
    return x * mask / keep


class DropPath(nn.Module):
    """Module form of :func:`drop_path`."""

    def __init__(self, drop_prob: float = 0.0):
        super().__init__()
        self.drop_prob = drop_prob

    def forward(self, x):
        return drop_path(x, self.drop_prob, self.training)


def _meta(sharded, shared, reduce):
    return {"sharded": list(sharded), "shared": list(shared), "reduce": list(reduce)}


class LinearLayer(nn.Module):
    """Weight-only linear layer ``y = x W^T`` (bias lives in :class:`BiasLayer`)."""

    def __init__(self, in_features: int, out_features: int, comm_metadata=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.weight.comm_metadata = comm_metadata or _meta([None, None], [], [])
        trunc_normal_(self.weight, std=0.02)

    def forward(self, x):
        return torch.nn.functional.linear(x, self.weight)


class BiasLayer(nn.Module):
    """Separate bias, so a row-parallel bias is added once after the tp reduction."""

    def __init__(self, dim: int, comm_metadata=None):
        super().__init__()
        self.bias = nn.Parameter(torch.zeros(dim))
        self.bias.comm_metadata = comm_metadata or _meta([None], [], [])

    def forward(self, x):
        return x + self.bias


class NormLayer(nn.Module):
    """RMSNorm or LayerNorm holder (parameters under ``.norm``)."""

    def __init__(self, normalized_shape: int, elementwise_affine: bool = True,
                 norm_type: str = "layer_norm", comm_metadata=None):
        super().__init__()
        self.norm_type = norm_type
        if norm_type == "layer_norm":
            self.norm = nn.LayerNorm(normalized_shape, elementwise_affine=elementwise_affine)
            has_bias = True
        elif norm_type == "rms_norm":
            self.norm = nn.RMSNorm(normalized_shape, elementwise_affine=elementwise_affine)
            has_bias = False
        else:
            raise ValueError(f"invalid norm type {norm_type!r}")
        if elementwise_affine:
            meta = comm_metadata or _meta([None], [], [])
            self.norm.weight.comm_metadata = meta
            if has_bias:
                self.norm.bias.comm_metadata = meta

    @property
    def weight(self):
        return self.norm.weight

    def forward(self, x):
        from .. import ops

        if self.norm_type == "rms_norm":
            return ops.rms_norm(x, self.norm.weight)
        return self.norm(x)


class Conv2DLayer(nn.Module):
    def __init__(self, in_chans: int, out_chans: int, kernel_size: int, stride: int = 1,
                 bias: bool = True, comm_metadata=None):
        super().__init__()
        self.conv = nn.Conv2d(in_chans, out_chans, kernel_size=kernel_size, stride=stride, bias=bias)
        meta = comm_metadata or _meta([], ["tp-sp1-sp2"], ["sp1-sp2"])
        self.conv.weight.comm_metadata = meta
        if bias:
            self.conv.bias.comm_metadata = meta

    def forward(self, x):
        return self.conv(x)


class PatchEmbedLayer(nn.Module):
    """Non-overlapping ``p x p`` patch projection; records local patch-grid shape."""

    def __init__(self, patch_size: int = 16, in_chans: int = 3, embed_dim: int = 768,
                 sp1_shapes=None, sp2_shapes=None, comm_metadata=None):
        super().__init__()
        self.patch_size = patch_size
        self.in_chans, self.embed_dim = in_chans, embed_dim
        self.proj = Conv2DLayer(in_chans, embed_dim, kernel_size=patch_size, stride=patch_size,
                                comm_metadata=comm_metadata)
        self.sp1_patch_shapes = [s // patch_size for s in sp1_shapes]
        self.sp2_patch_shapes = [s // patch_size for s in sp2_shapes]
        self.h = self.sp1_patch_shapes[comm.get_rank("sp1")]
        self.w = self.sp2_patch_shapes[comm.get_rank("sp2")]
        self.num_patches = self.h * self.w

    def forward(self, x):
        """``x``: (N, C, H, W) -> tokens (N, h, w, E) through the fused patch-embed op."""
        from .. import ops

        return ops.patch_embed(x, self.proj.conv.weight, self.proj.conv.bias, self.patch_size)
