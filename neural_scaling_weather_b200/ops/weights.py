"""Low-precision copies of fp32 master weights, made once per optimizer step.

The fused optimizer writes a bf16/fp16 shadow of every parameter in the same kernel as
the update and registers it here; the GEMM operators read the shadow instead of casting
the fp32 master on every micro-batch.  Parameters without a shadow are cast on demand
and the result is cached until the parameter's version counter changes.
"""

from __future__ import annotations

import weakref
from typing import Dict, Sequence, Tuple

import torch

_shadows: "weakref.WeakKeyDictionary[torch.Tensor, torch.Tensor]" = weakref.WeakKeyDictionary()
_cache: Dict[Tuple, Tuple[Tuple[int, ...], torch.Tensor]] = {}


def register_shadow(param: torch.Tensor, shadow: torch.Tensor) -> None:
    _shadows[param] = shadow


def clear() -> None:
    _shadows.clear()
    _cache.clear()


def get(param: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``param`` in ``dtype`` (a registered shadow, or a version-cached cast)."""
    if param.dtype == dtype:
        return param.detach()
    sh = _shadows.get(param)
    if sh is not None and sh.dtype == dtype:
        return sh
    key = (id(param), dtype)
    ver = (param._version,)
    hit = _cache.get(key)
    if hit is not None and hit[0] == ver and hit[1].data_ptr() != 0:
        return hit[1]
    t = param.detach().to(dtype)
    _cache[key] = (ver, t)
    return t


def get_cat(params: Sequence[torch.Tensor], dtype: torch.dtype) -> torch.Tensor:
    """Concatenation along dim 0 of several parameters, cached on their versions."""
    if len(params) == 1:
        return get(params[0], dtype)
    key = (tuple(id(p) for p in params), dtype)
    ver = tuple(p._version for p in params)
    sh = [_shadows.get(p) for p in params]
    hit = _cache.get(key)
    if hit is not None and hit[0] == ver:
        return hit[1]
    parts = [s if (s is not None and s.dtype == dtype) else p.detach().to(dtype)
             for p, s in zip(params, sh)]
    t = torch.cat(parts, dim=0)
    _cache[key] = (ver, t)
    return t
