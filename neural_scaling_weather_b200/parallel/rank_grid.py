"""Rank grid: the hyper-rectangle of ranks spanned by the parallel dimensions.

Behaviour matches ``utils/rank_generator.py:11-195`` of the reference (itself the
Megatron-LM scheme): the dimensions are listed in an ``order`` string such as
``"sp1-sp2-tp-pp-dp"`` whose FIRST entry varies fastest, so

    global_rank = sum_i coord[i] * stride[i],   stride[i] = prod(size[:i]).

A group token such as ``"tp"`` or ``"dp-sp1-sp2"`` selects a subset of the dimensions;
each group holds the ranks that share every coordinate outside that subset.  Groups are
listed with the unselected coordinates enumerated first-dimension-fastest, and ranks
inside a group with the selected coordinates enumerated first-dimension-fastest.  The
exact listing is part of the interface (process groups are created in this order on
every rank), so it is reproduced exactly; the implementation below is a direct
mixed-radix enumeration.
"""

from __future__ import annotations

import itertools
from typing import Dict, List, Sequence

DIMS = ("tp", "pp", "dp", "sp1", "sp2")


def _strides(sizes: Sequence[int]) -> List[int]:
    out, acc = [], 1
    for s in sizes:
        out.append(acc)
        acc *= s
    return out


def _mixed_radix(sizes: Sequence[int]):
    """All coordinate tuples over ``sizes`` with the first coordinate varying fastest."""
    for rev in itertools.product(*[range(s) for s in reversed(sizes)]):
        yield tuple(reversed(rev))


def orthogonal_groups(sizes: Sequence[int], selected: Sequence[bool]) -> List[List[int]]:
    """Rank groups spanning the ``selected`` dimensions of a grid of ``sizes``."""
    strides = _strides(sizes)
    sel = [i for i, m in enumerate(selected) if m]
    rest = [i for i, m in enumerate(selected) if not m]
    groups = []
    for outer in _mixed_radix([sizes[i] for i in rest]):
        base = sum(c * strides[i] for c, i in zip(outer, rest))
        group = [
            base + sum(c * strides[i] for c, i in zip(inner, sel))
            for inner in _mixed_radix([sizes[i] for i in sel])
        ]
        groups.append(group)
    return groups


class RankGrid:
    """Orthogonal process-group layout for tp x pp x dp x sp1 x sp2."""

    def __init__(self, tp: int = 1, dp: int = 1, pp: int = 1, sp1: int = 1, sp2: int = 1,
                 order: str = "sp1-sp2-tp-pp-dp", rank_offset: int = 0):
        self.sizes: Dict[str, int] = {"tp": tp, "pp": pp, "dp": dp, "sp1": sp1, "sp2": sp2}
        self.rank_offset = rank_offset
        self.world_size = tp * dp * pp * sp1 * sp2
        names = [t for t in order.lower().split("-") if t]
        for name in DIMS:
            if name not in names:
                if self.sizes[name] != 1:
                    raise RuntimeError(
                        f"dimension {name} has size {self.sizes[name]} but is missing "
                        f"from the order string {order!r}"
                    )
                names.append(name)
        self.order = "-".join(names)
        self.names = names
        self.ordered_sizes = [self.sizes[n] for n in names]

    def mask(self, token: str) -> List[bool]:
        wanted = token.lower().split("-")
        for w in wanted:
            if w not in self.names:
                raise ValueError(f"unknown parallel dimension {w!r} in {token!r}")
        return [n in wanted for n in self.names]

    def get_ranks(self, token: str) -> List[List[int]]:
        groups = orthogonal_groups(self.ordered_sizes, self.mask(token))
        if self.rank_offset:
            groups = [[r + self.rank_offset for r in g] for g in groups]
        return groups

    def coords(self, rank: int) -> Dict[str, int]:
        """Coordinate of ``rank`` along every dimension."""
        r = rank - self.rank_offset
        out = {}
        for name, size in zip(self.names, self.ordered_sizes):
            out[name] = r % size
            r //= size
        return out


# name used by the reference (utils/rank_generator.py:120)
RankGenerator = RankGrid
