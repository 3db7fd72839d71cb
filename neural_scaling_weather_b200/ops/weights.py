"""Low-precision copies of fp32 master weights, made once per optimizer step.

The fused optimizer writes a bf16/fp16 shadow of every parameter in the same kernel as
the update and registers it here; the GEMM operators read the shadow instead of casting
the fp32 master on every micro-batch.  Parameters without a shadow are cast on demand
and the result is cached until the parameter's version counter changes.
"""

from __future__ import annotations

import weakref
from typing import Callable, Dict, Sequence, Tuple

import torch

# id(param) -> (weak reference to param, shadow); tensors cannot be dict keys by value
_shadows: Dict[int, Tuple["weakref.ref", torch.Tensor]] = {}
_cache: Dict[Tuple, Tuple[Tuple[int, ...], torch.Tensor]] = {}
# derived tensors (concatenations, transposes) with the function that rebuilds them and the
# parameters they come from; refresh_derived() rewrites them in place after an optimizer step,
# so a CUDA graph that captured them keeps reading current weights
_derived: Dict[Tuple, Tuple[Tuple["weakref.ref", ...], torch.Tensor, Callable[[], torch.Tensor]]] = {}


def register_shadow(param: torch.Tensor, shadow: torch.Tensor) -> None:
    _shadows[id(param)] = (weakref.ref(param), shadow)


def _shadow_of(param: torch.Tensor):
    hit = _shadows.get(id(param))
    if hit is None or hit[0]() is not param:
        return None
    return hit[1]


def clear() -> None:
    _shadows.clear()
    _cache.clear()
    _derived.clear()


def register_derived(key: Tuple, params: Sequence[torch.Tensor], t: torch.Tensor,
                     rebuild: Callable[[], torch.Tensor]) -> None:
    _derived[key] = (tuple(weakref.ref(p) for p in params), t, rebuild)


def refresh_derived() -> None:
    """Recompute every cached concatenation / transpose in place (concatenations first: the
    transposes are built from them) and mark them current.  Called after each optimizer step
    when training runs from captured CUDA graphs."""
    dead = []
    for order in (0, 1):
        for key, (refs, t, rebuild) in list(_derived.items()):
            if (key[0] == "T") != bool(order):
                continue
            params = [r() for r in refs]
            if any(p is None for p in params):
                dead.append(key)
                continue
            with torch.no_grad():
                t.copy_(rebuild())
            ver = tuple(p._version for p in params)
            if key[0] == "T":
                from . import fused  # transposes live in the fused operators' cache

                fused._wt_cache[key[1]] = (ver, t)
            else:
                _cache[key] = (ver, t)
    for key in dead:
        _derived.pop(key, None)


def get(param: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``param`` in ``dtype`` (a registered shadow, or a version-cached cast)."""
    if param.dtype == dtype:
        return param.detach()
    if not isinstance(param, torch.nn.Parameter) or param.is_inference():
        return param.detach().to(dtype)  # temporaries are not cached
    sh = _shadow_of(param)
    if sh is not None and sh.dtype == dtype:
        return sh
    key = (id(param), dtype)
    ver = (param._version,)
    hit = _cache.get(key)
    if hit is not None and hit[0] == ver and hit[1].data_ptr() != 0:
        return hit[1]
    t = param.detach().to(dtype)
    _cache[key] = (ver, t)
    register_derived(key, [param], t, lambda: param.detach().to(dtype))
    return t


def get_cat(params: Sequence[torch.Tensor], dtype: torch.dtype) -> torch.Tensor:
    """Concatenation along dim 0 of several parameters, cached on their versions."""
    if len(params) == 1:
        return get(params[0], dtype)
    if not all(isinstance(p, torch.nn.Parameter) for p in params):
        return torch.cat([p.detach().to(dtype) for p in params], dim=0)
    key = (tuple(id(p) for p in params), dtype)
    ver = tuple(p._version for p in params)
    sh = [_shadow_of(p) for p in params]
    hit = _cache.get(key)
    if hit is not None and hit[0] == ver:
        return hit[1]
    parts = [s if (s is not None and s.dtype == dtype) else p.detach().to(dtype)
             for p, s in zip(params, sh)]
    t = torch.cat(parts, dim=0)
    _cache[key] = (ver, t)
    ps = list(params)
    register_derived(key, ps, t, lambda: torch.cat(
        [s if (s is not None and s.dtype == dtype) else p.detach().to(dtype)
         for p, s in zip(ps, [_shadow_of(q) for q in ps])], dim=0))
    return t
