"""Fused operators of the weather transformer.

Each public function takes PyTorch tensors and returns PyTorch tensors with autograd.
CPU tensors run the plain-PyTorch oracle in :mod:`.reference`.  CUDA tensors run the
hand-written sm_100a kernels of the ``_C`` extension (tcgen05/TMEM GEMMs with fused
epilogues, windowed attention with fused QK-norm, shift and mask, fused norms, loss and
optimizer kernels); a CUDA call without the extension raises.

Compute precision on CUDA follows ``torch.autocast``: inside an autocast region (the
trainer uses one, as the reference does) activations are bf16 (or fp16); parameters stay
fp32 masters and are cast once per optimizer step into a cached low-precision copy.  The
kernels compute in 16 bits, so fp32 CUDA inputs outside autocast are also computed in bf16;
for fp32 arithmetic on the GPU (fp32 inference, as the reference runs it) wrap the call in
:func:`reference_ops`, which sends CUDA tensors through the plain-PyTorch oracle too.
"""

from __future__ import annotations

import contextlib
import threading
from typing import Optional, Sequence, Union

import torch

from . import reference
from ._ext import available as extension_available
from ._ext import require as require_extension
from .geometry import WindowGeometry

TensorOrParts = Union[torch.Tensor, Sequence[torch.Tensor]]


def compute_dtype(t: torch.Tensor) -> torch.dtype:
    """Activation dtype of a CUDA op: the autocast dtype if active, else the input dtype."""
    if t.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return t.dtype


_mode = threading.local()


@contextlib.contextmanager
def reference_ops():
    """Within this context every operator runs the plain-PyTorch oracle (:mod:`.reference`),
    on CUDA tensors too, in the tensors' own precision (fp32 math for fp32 inputs)."""
    prev = getattr(_mode, "reference", False)
    _mode.reference = True
    try:
        yield
    finally:
        _mode.reference = prev


def _use_cuda(t: torch.Tensor) -> bool:
    if not t.is_cuda or getattr(_mode, "reference", False):
        return False
    require_extension()
    return True


def _cat(parts):
    if isinstance(parts, torch.Tensor) or parts is None:
        return parts
    parts = list(parts)
    return parts[0] if len(parts) == 1 else torch.cat(parts, dim=0)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: Optional[float] = None) -> torch.Tensor:
    if not _use_cuda(x):
        return reference.rms_norm(x, w, eps)
    from .fused import rms_norm_cuda

    return rms_norm_cuda(x, w, eps)


def rms_norm_with_skip(x: torch.Tensor, w: torch.Tensor, eps: Optional[float] = None):
    """``(rms_norm(x, w), x)``: the pre-norm block input and its skip connection from one
    autograd node, so their gradients are summed inside the RMSNorm backward on CUDA."""
    if not _use_cuda(x):
        return reference.rms_norm(x, w, eps), x
    from .fused import rms_norm_skip_cuda

    return rms_norm_skip_cuda(x, w, eps)


def linear_allreduce(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     residual: Optional[torch.Tensor] = None, group: str = "tp") -> torch.Tensor:
    """Row-parallel linear: ``all_reduce_group(x W^T) + bias + residual``.  On CUDA with a
    symmetric-memory group of 2..8 GPUs the all-reduce runs inside the GEMM's epilogue over
    NVLink peer memory; otherwise GEMM, then the NCCL all-reduce mapping, then the adds."""
    from ..parallel import symm
    from ..parallel.mappings import allreduce_forward_identity_backward

    if _use_cuda(x) and symm.available(group):
        from .fused import linear_allreduce_cuda

        return linear_allreduce_cuda(x, weight, bias, residual, group)
    y = linear(x, weight)
    y = allreduce_forward_identity_backward(y, group)
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y if residual is None else y + residual


def linear_colparallel(x: torch.Tensor, weight: TensorOrParts, bias: Optional[TensorOrParts] = None,
                       activation: Optional[str] = None, group: str = "tp") -> torch.Tensor:
    """Column-parallel linear of a replicated input: ``act(x W_local^T + b_local)``, whose input
    gradient is all-reduced over ``group`` (the reference's ``copy_to_parallel_region`` followed by
    the linear).  On CUDA with a symmetric-memory group of 2..8 GPUs the all-reduce runs inside the
    data-gradient GEMM's epilogue over NVLink; otherwise the NCCL mapping wraps the linear."""
    from ..parallel import comm, symm
    from ..parallel.mappings import identity_forward_allreduce_backward

    if comm.get_size(group) > 1 and _use_cuda(x) and symm.available(group):
        from .fused import linear_cuda

        return linear_cuda(x, weight, bias, None, activation, allreduce_group=group)
    x = identity_forward_allreduce_backward(x, group)
    return linear(x, weight, bias, activation=activation)


def linear(x: torch.Tensor, weight: TensorOrParts, bias: Optional[TensorOrParts] = None,
           residual: Optional[torch.Tensor] = None, activation: Optional[str] = None):
    """``act(x W^T + b) + residual``; ``weight``/``bias`` may be lists concatenated on N."""
    if not _use_cuda(x):
        return reference.linear(x, _cat(weight), _cat(bias), residual, activation)
    from .fused import linear_cuda

    return linear_cuda(x, weight, bias, residual, activation)


def mlp(x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor,
        residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``fc2(GELU(fc1(x))) + residual`` with biases (fused backward on CUDA)."""
    if not _use_cuda(x):
        h = reference.linear(x, w1, b1, activation="gelu")
        return reference.linear(h, w2, b2, residual=residual)
    from .fused import mlp_cuda

    return mlp_cuda(x, w1, b1, w2, b2, residual)


def window_attention(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                     num_heads: int, head_dim: int, geom: WindowGeometry, scale: float):
    """Shifted-window attention over (B, T, H, W, 3*nh*hd) -> (B, T, H, W, nh*hd)."""
    if not _use_cuda(qkv):
        return reference.window_attention(qkv, q_norm_w, k_norm_w, num_heads, head_dim, geom, scale)
    from .fused import window_attention_cuda

    return window_attention_cuda(qkv, q_norm_w, k_norm_w, num_heads, head_dim, geom, scale)


def patch_embed(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                patch_size: int, add: Optional[torch.Tensor] = None):
    """(N, C, H, W) -> (N, h, w, E); ``add`` (P, h, w, E) is broadcast over N // P."""
    if not _use_cuda(x):
        return reference.patch_embed(x, weight, bias, patch_size, add)
    from .fused import patch_embed_cuda

    return patch_embed_cuda(x, weight, bias, patch_size, add)


def coord_pos_embed(coords: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                    patch_size: int) -> torch.Tensor:
    """Patch projection of a constant coordinate field (T, 4, H, W) -> (T, h, w, E): on CUDA computed
    once per weight version and reused by every forward until the next optimizer step."""
    if not _use_cuda(coords):
        return reference.patch_embed(coords, weight, bias, patch_size)
    from .fused import coord_pos_embed_cuda

    return coord_pos_embed_cuda(coords, weight, bias, patch_size)


def head_unpatchify(x: torch.Tensor, weight: torch.Tensor, patch_size: int, out_chans: int):
    """(B, T, h, w, E) -> (B, T, C, h*p, w*p)."""
    if not _use_cuda(x):
        return reference.head_unpatchify(x, weight, patch_size, out_chans)
    from .fused import head_unpatchify_cuda

    return head_unpatchify_cuda(x, weight, patch_size, out_chans)


def weighted_sse(x: torch.Tensor, y: torch.Tensor, area_w: Optional[torch.Tensor] = None,
                 ch_w: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Scalar sum of ``(x-y)^2 * area_w[h,1] * ch_w[c,1,1]`` (fp32)."""
    if not _use_cuda(x):
        return reference.weighted_sse(x, y, area_w, ch_w)
    from .fused import weighted_sse_cuda

    return weighted_sse_cuda(x, y, area_w, ch_w)


def weighted_se_per_channel(x: torch.Tensor, y: torch.Tensor, area_w: torch.Tensor):
    """``sum_{h,w} area_w * (x-y)^2`` keeping the leading dims (fp32)."""
    if not _use_cuda(x):
        return reference.weighted_se_per_channel(x, y, area_w)
    from .fused import weighted_se_per_channel_cuda

    return weighted_se_per_channel_cuda(x, y, area_w)


__all__ = [
    "WindowGeometry",
    "compute_dtype",
    "extension_available",
    "head_unpatchify",
    "linear",
    "mlp",
    "patch_embed",
    "reference",
    "rms_norm",
    "weighted_se_per_channel",
    "weighted_sse",
    "window_attention",
]
