"""Data-parallel gradient synchronisation that honours ``comm_metadata['reduce']``.

Semantics of the reference (``distributed/mappings.py:217-341``): DDP over the ``dp``
group plus a comm hook, so that after backward every gradient equals

    (1 / dp) * sum over dp  of  sum over the param's ``reduce`` groups  of  local grads.

Because the groups are orthogonal, that is ONE sum over the product group, divided by
``dp``: ``dp`` for params with no extra group, ``dp-sp1-sp2`` for ``["sp1-sp2"]`` and
``dp-tp-sp1-sp2`` (the world, pp = 1) for ``["tp-sp1-sp2"]``.  The reducer therefore
sorts the parameters by that product group, lays their gradients out contiguously in
the optimizer's flat fp32 gradient buffer (``.grad`` are views, like DDP's
``gradient_as_bucket_view``), cuts each group's range into buckets, and launches one
asynchronous all-reduce per bucket as soon as backward has produced every gradient in it
(post-accumulate-grad hooks, and ``ops.gradsink`` for gradients the weight-gradient kernel
writes in place), so communication overlaps the rest of backward.  The
``1/dp`` factor is applied to the bucket before the sum.  ``no_sync()`` skips the
reduction on gradient-accumulation micro-batches, as DDP's does.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from . import comm


def reduction_group_name(param) -> str:
    reduce = list(getattr(param, "comm_metadata", {}).get("reduce", []))
    if not reduce:
        return "dp"
    if all(g == "sp1-sp2" for g in reduce):
        return "dp-sp1-sp2"
    if all(g in ("tp-sp1-sp2", "sp1-sp2") for g in reduce):
        return "dp-tp-sp1-sp2"
    raise ValueError(f"unsupported reduce groups {reduce}")


def _group(name: str):
    if name == "dp-tp-sp1-sp2":
        return None  # the default (world) group when pp == 1
    return comm.get_group(name)


def _group_size(name: str) -> int:
    if name == "dp-tp-sp1-sp2":
        return comm.get_world_size()
    return comm.get_size(name)


def order_params(params: List[torch.nn.Parameter]) -> List[torch.nn.Parameter]:
    """Parameter order for the flat buffers: grouped by reduction group, and inside a
    group in reverse registration order (the order backward produces gradients)."""
    rank = {"dp": 0, "dp-sp1-sp2": 1, "dp-tp-sp1-sp2": 2}
    idx = {id(p): i for i, p in enumerate(params)}
    return sorted(params, key=lambda p: (rank[reduction_group_name(p)], -idx[id(p)]))


class _Bucket:
    def __init__(self, group_name: str, lo: int, hi: int, params: List[torch.nn.Parameter]):
        self.group_name = group_name
        self.lo, self.hi = lo, hi
        self.params = params
        self.pending = len(params)
        self.handle = None


class GradReducer:
    """Bucketed, overlapped gradient all-reduce over a :class:`FlatParamSpace`."""

    def __init__(self, space, bucket_cap_mb: float = 25.0, broadcast_from_root: bool = True):
        self.space = space
        self.enabled = dist.is_initialized() and any(
            _group_size(reduction_group_name(p)) > 1 for p in space.params)
        self.dp = comm.get_size("dp")
        self._sync = True
        self.buckets: List[_Bucket] = []
        self._param_bucket: Dict[int, _Bucket] = {}
        cap = int(bucket_cap_mb * 1024 * 1024 // 4)
        cur: Optional[_Bucket] = None
        for i, p in enumerate(space.params):
            gname = reduction_group_name(p)
            lo = space.offsets[i]
            hi = space.offsets[i + 1] if i + 1 < len(space.params) else space.numel
            if cur is None or cur.group_name != gname or (cur.hi - cur.lo) >= cap:
                cur = _Bucket(gname, lo, hi, [])
                self.buckets.append(cur)
            cur.hi = hi
            cur.params.append(p)
            self._param_bucket[id(p)] = cur
        for b in self.buckets:
            b.pending = len(b.params)
        self._seen = set()
        self._hooks = []
        if self.enabled:
            for p in space.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))
            # gradients that the weight-gradient kernel adds into .grad in place bypass autograd's
            # accumulation (and its hooks); the fused layers report them here instead
            from ..ops import gradsink

            gradsink.register(self._on_grad)
            if broadcast_from_root and comm.get_size("dp") > 1:
                dist.broadcast(space.data, src=comm.get_root("dp"), group=comm.get_group("dp"))

    @contextmanager
    def no_sync(self):
        old = self._sync
        self._sync = False
        try:
            yield
        finally:
            self._sync = old

    def _on_grad(self, p):
        if not self._sync:
            return
        b = self._param_bucket.get(id(p))
        if b is None or not any(q is p for q in b.params):  # another model's parameter
            return
        # a parameter is counted once per backward: autograd's post-accumulate hook also fires
        # (with no gradient) for a parameter whose gradient the kernel wrote in place and reported
        # through ops.gradsink
        if id(p) in self._seen:
            return
        self._seen.add(id(p))
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b: _Bucket):
        if _group_size(b.group_name) == 1:
            if self.dp != 1:
                self.space.grad[b.lo:b.hi].mul_(1.0 / self.dp)
            b.handle = None
            return
        buf = self.space.grad[b.lo:b.hi]
        if self.dp != 1:
            buf.mul_(1.0 / self.dp)
        b.handle = dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=_group(b.group_name),
                                   async_op=True)

    def finish(self):
        """Wait for every bucket (launching any whose hooks did not all fire)."""
        if not self.enabled or not self._sync:
            return
        for b in self.buckets:
            if b.pending > 0:
                self._launch(b)
        for b in self.buckets:
            if b.handle is not None:
                b.handle.wait()
                b.handle = None
            b.pending = len(b.params)
        self._seen.clear()

    def reset(self):
        for b in self.buckets:
            b.pending = len(b.params)
            b.handle = None
        self._seen.clear()
