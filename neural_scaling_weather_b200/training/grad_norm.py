"""Sharding-aware global gradient (or weight) norm without host synchronisation.

The reference (``utils/trainer.py:416-448``) sums ``p.grad**2`` per parameter, all-reduces
that scalar over every group the parameter is sharded on, adds the results and calls
``.item()`` (a host sync), twice per step.  Here parameters are grouped by their set of
sharding groups; one kernel computes the per-class sums of squares over the flat buffer,
each class's scalar is all-reduced over its groups (device tensors, no sync) and the
clip coefficient ``max_norm / (norm + 1e-6)`` (when ``norm > max_norm``) stays on device
for the fused optimizer to read.
"""

from __future__ import annotations

from typing import Dict, Tuple

import torch
import torch.distributed as dist

from ..ops import _ext
from ..parallel import comm


class ShardedNorm:
    """``owned``: with the data-parallel sharded step, the element ranges this rank owns; the gradient
    norm is then summed over those only and all-reduced over dp (every gradient is owned once)."""

    def __init__(self, space, owned=None):
        self.space = space
        self.owned = owned
        classes: Dict[Tuple[str, ...], int] = {}
        seg_lo, seg_hi, seg_cls = [], [], []
        for i, p in enumerate(space.params):
            key = tuple(g for g in getattr(p, "comm_metadata", {}).get("sharded", []) if g is not None)
            c = classes.setdefault(key, len(classes))
            lo = space.offsets[i]
            seg_lo.append(lo)
            seg_hi.append(lo + p.numel())
            seg_cls.append(c)
        self.classes = sorted(classes, key=classes.get)
        self._lo, self._hi, self._cls = seg_lo, seg_hi, seg_cls
        # fixed work split for the kernel: blocks of <= 64K elements inside one segment
        blo, bhi, bcls = [], [], []
        chunk = 1 << 16
        for lo, hi, c in zip(seg_lo, seg_hi, seg_cls):
            for a in range(lo, hi, chunk):
                blo.append(a)
                bhi.append(min(hi, a + chunk))
                bcls.append(c)
        dev = space.data.device
        self.block_lo = torch.tensor(blo, dtype=torch.int64, device=dev)
        self.block_hi = torch.tensor(bhi, dtype=torch.int64, device=dev)
        self.block_cls = torch.tensor(bcls, dtype=torch.int32, device=dev)
        if owned is not None:
            self._owned_blocks = self._blocks_over(owned)

    def _blocks_over(self, ranges):
        """Kernel blocks (lo, hi, class) of the parameter segments restricted to ``ranges``."""
        blo, bhi, bcls = [], [], []
        chunk = 1 << 16
        for lo, hi, c in zip(self._lo, self._hi, self._cls):
            for a, b in ranges:
                s, e = max(lo, a), min(hi, b)
                for x in range(s, e, chunk):
                    blo.append(x)
                    bhi.append(min(e, x + chunk))
                    bcls.append(c)
        dev = self.space.data.device
        if not blo:  # nothing owned: one empty block
            blo, bhi, bcls = [0], [0], [0]
        return (torch.tensor(blo, dtype=torch.int64, device=dev), torch.tensor(bhi, dtype=torch.int64, device=dev),
                torch.tensor(bcls, dtype=torch.int32, device=dev))

    def _class_sums(self, buf: torch.Tensor, owned: bool = False) -> torch.Tensor:
        if buf.is_cuda:
            lo, hi, cls = self._owned_blocks if owned else (self.block_lo, self.block_hi, self.block_cls)
            return _ext.require().segment_sumsq(buf, lo, hi, cls, len(self.classes))
        out = torch.zeros(len(self.classes), dtype=torch.float32)
        for lo, hi, c in zip(self._lo, self._hi, self._cls):
            out[c] += buf[lo:hi].float().square().sum()
        return out

    def norm(self, which: str = "grad") -> torch.Tensor:
        """Global L2 norm (device scalar tensor, shape [1])."""
        buf = self.space.grad if which == "grad" else self.space.data
        owned = which == "grad" and self.owned is not None and buf.is_cuda
        sums = self._class_sums(buf, owned)
        if owned:  # each gradient element is owned by one dp rank
            dist.all_reduce(sums, group=comm.get_group("dp"))
        total = torch.zeros(1, dtype=torch.float32, device=buf.device)
        for c, groups in enumerate(self.classes):
            s = sums[c:c + 1].clone()
            for g in groups:
                if comm.get_size(g) > 1:
                    dist.all_reduce(s, group=comm.get_group(g))
            total += s
        return total.sqrt()

    @staticmethod
    def clip_coef(norm: torch.Tensor, max_norm: float) -> torch.Tensor:
        return torch.where(norm > max_norm, max_norm / (norm + 1e-6), torch.ones_like(norm))
