"""Weight gradients written straight into ``param.grad`` by the weight-gradient kernel.

The fused linear layers compute dW (and db) on the tensor cores with fp32 accumulation
(``ext.wgrad``).  When a parameter's ``.grad`` is an fp32 contiguous tensor (the optimizer's flat
gradient buffer keeps every ``.grad`` as such a view), the kernel adds into it directly and the
autograd function returns ``None`` for that input: no separate gradient tensor, no autograd
accumulation kernel.  Autograd's post-accumulate-grad hook of such a parameter still fires (with
no gradient), after all of its uses; the data-parallel reducer registers its hook here as well and
counts each parameter once per backward, whichever notice comes first.  A parameter used by several forward
calls before one backward (a multi-step rollout applies the model several times) is reported once,
after the last of its backward calls has written its share, as autograd would have done.
"""

from __future__ import annotations

import os
import weakref
from typing import Callable, List, Optional

import torch

# weak references: a reducer that is no longer used (its trainer gone) drops out by itself
_callbacks: List[weakref.WeakMethod] = []


def register(cb: Callable[[torch.nn.Parameter], None]) -> None:
    """Register a bound method to be called with each parameter whose gradient was written in place."""
    ref = weakref.WeakMethod(cb)
    if all(r() != cb for r in _callbacks):
        _callbacks.append(ref)


def unregister(cb: Callable[[torch.nn.Parameter], None]) -> None:
    _callbacks[:] = [r for r in _callbacks if r() is not None and r() != cb]


_IN_PLACE = os.environ.get("NSW_WGRAD_INPLACE", "1") != "0"


def target(p: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """``p.grad`` if the kernel may accumulate into it in place (fp32, contiguous, 16-byte aligned).
    ``NSW_WGRAD_INPLACE=0`` returns every gradient through autograd instead."""
    if not _IN_PLACE or p is None or not isinstance(p, torch.nn.Parameter) or not p.requires_grad:
        return None
    g = p.grad
    if g is None or g.dtype != torch.float32 or not g.is_contiguous() or g.data_ptr() % 16 != 0:
        return None
    return g


def use(params) -> None:
    """A forward call whose backward will write these parameters' gradients."""
    for p in params:
        if p is not None:
            p._nsw_pending = getattr(p, "_nsw_pending", 0) + 1


def done(p: torch.nn.Parameter, written: bool) -> None:
    """One backward call has produced its share of ``p``'s gradient (in place if ``written``);
    after the last one the registered hooks run for parameters written in place."""
    n = getattr(p, "_nsw_pending", 1) - 1
    p._nsw_pending = max(n, 0)
    if written:
        p._nsw_written = True
    if n <= 0 and getattr(p, "_nsw_written", False):
        p._nsw_written = False
        for ref in list(_callbacks):
            cb = ref()
            if cb is None:
                _callbacks.remove(ref)
            else:
                cb(p)
