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
# key -> (weak references to the source parameters, their versions, cached tensor).  A hit
# needs the SAME live parameter objects: ids are reused once a parameter is freed, so an id
# alone could hand a new model the cached copy of an old one.
_cache: Dict[Tuple, Tuple[Tuple["weakref.ref", ...], Tuple[int, ...], torch.Tensor]] = {}
# derived tensors (casts, concatenations, transposes) with the function that rebuilds them and
# the parameters they come from; refresh_derived() rewrites them in place after an optimizer
# step, so a CUDA graph that captured them keeps reading current weights
_derived: Dict[Tuple, Tuple[Tuple["weakref.ref", ...], torch.Tensor, Callable[[], torch.Tensor]]] = {}


def normal_tensor(fn: Callable[[], torch.Tensor]) -> torch.Tensor:
    """Run ``fn`` without autograd and with inference mode off.  A cached tensor outlives the context
    that built it: one first built during validation or a rollout (``torch.inference_mode``) would be
    an inference tensor, and a training forward that used it later would get an output without a
    gradient path (or an error where it is saved for backward)."""
    with torch.inference_mode(False), torch.no_grad():
        return fn()


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


def _versions(params: Sequence[torch.Tensor]) -> Tuple[int, ...]:
    return tuple(p._version for p in params)


def _lookup(key: Tuple, params: Sequence[torch.Tensor]):
    hit = _cache.get(key)
    if hit is None:
        return None
    refs, ver, t = hit
    if len(refs) != len(params) or any(r() is not p for r, p in zip(refs, params)):
        return None
    if ver != _versions(params) or t.data_ptr() == 0:
        return None
    return t


def _store(key: Tuple, params: Sequence[torch.Tensor], t: torch.Tensor,
           rebuild: Callable[[], torch.Tensor]) -> torch.Tensor:
    refs = tuple(weakref.ref(p) for p in params)
    _cache[key] = (refs, _versions(params), t)
    _derived[key] = (refs, t, rebuild)
    return t


def refresh_derived() -> None:
    """Recompute every cached cast / concatenation / transpose in place (casts and
    concatenations first: the transposes are built from them) and mark them current.  Called
    after each optimizer step when training runs from captured CUDA graphs."""
    dead = []
    for order in (0, 1):
        for key, (refs, t, rebuild) in list(_derived.items()):
            if (key[0] == "T") != bool(order):
                continue
            params = [r() for r in refs]
            if any(p is None for p in params):
                dead.append(key)
                continue
            with torch.inference_mode(False), torch.no_grad():
                t.copy_(rebuild())
            _cache[key] = (refs, _versions(params), t)
    for key in dead:
        _derived.pop(key, None)
        _cache.pop(key, None)


def get_derived(key: Tuple, params: Sequence[torch.Tensor], build: Callable[[], torch.Tensor]) -> torch.Tensor:
    """A tensor computed from ``params`` only (``build`` runs without autograd), cached on their
    versions and rebuilt in place by ``refresh_derived`` after each optimizer step."""
    ps = list(params)
    full = ("D",) + tuple(key) + tuple(id(p) for p in ps)
    t = _lookup(full, ps)
    if t is not None:
        return t

    def rebuild():
        return normal_tensor(build)

    return _store(full, ps, rebuild(), rebuild)


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
    t = _lookup(key, [param])
    if t is not None:
        return t

    def build():
        return normal_tensor(lambda: param.detach().to(dtype))

    return _store(key, [param], build(), build)


def get_cat(params: Sequence[torch.Tensor], dtype: torch.dtype) -> torch.Tensor:
    """Concatenation along dim 0 of several parameters, cached on their versions."""
    if len(params) == 1:
        return get(params[0], dtype)
    if not all(isinstance(p, torch.nn.Parameter) for p in params):
        return torch.cat([p.detach().to(dtype) for p in params], dim=0)
    ps = list(params)
    key = (tuple(id(p) for p in ps), dtype)
    t = _lookup(key, ps)
    if t is not None:
        return t

    def build():
        return normal_tensor(lambda: torch.cat([s if (s is not None and s.dtype == dtype) else p.detach().to(dtype)
                                                for p, s in zip(ps, [_shadow_of(q) for q in ps])], dim=0))

    return _store(key, ps, build(), build)


def get_t(params: Sequence[torch.Tensor], w: torch.Tensor) -> torch.Tensor:
    """Contiguous transpose of ``w``, the (concatenated, possibly reshaped) compute-dtype copy
    of ``params``, cached on the parameters' versions (data-gradient GEMM operand)."""
    if not all(isinstance(p, torch.nn.Parameter) for p in params):
        return w.t().contiguous()
    ps = list(params)
    key = ("T", tuple(id(p) for p in ps), w.dtype)
    t = _lookup(key, ps)
    if t is not None:
        return t
    t = normal_tensor(lambda: w.t().contiguous())
    dt, n, k = w.dtype, t.shape[1], t.shape[0]
    return _store(key, ps, t, lambda: get_cat(ps, dt).reshape(n, k).t())
