"""Symmetric (peer-addressable) buffers for kernels that communicate over NVLink themselves.

The fused GEMM + all-reduce (``ops.linear_allreduce``, the tensor-parallel row-parallel
linears of reference ``models/swin_helpers.py`` (proj) and ``models/mlp.py`` (fc2), whose
output the reference reduces with ``reduce_from_parallel_region`` = NCCL all-reduce) needs, on
every rank of the group, a partial-result buffer and a few flag words whose addresses the
other ranks can load from and store to.  They come from ``torch.distributed._symmetric_memory``
(one allocation per (group, rows, columns, dtype), rendezvoused once and cached); the kernel
receives every rank's pointers.
"""

from __future__ import annotations

import importlib
import math
import os
from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch
import torch.distributed as dist

from . import comm

_BUFS: Dict[Tuple, "ARBuffers"] = {}
_DISABLED: Dict[str, str] = {}

FLAG_BASE = 16  # flag words before the per-tile ready flags (kernel layout)


@dataclass
class ARBuffers:
    part: torch.Tensor
    flags: torch.Tensor
    part_ptrs: List[int]
    flag_ptrs: List[int]
    rank: int
    world: int
    handles: tuple


def available(group_name: str) -> bool:
    """The fused path applies: a CUDA process group of 2..8 ranks (one node), symmetric memory
    usable, not switched off with NSW_FUSED_COLLECTIVES=0."""
    if os.environ.get("NSW_FUSED_COLLECTIVES", "1") == "0" or group_name in _DISABLED:
        return False
    if not torch.cuda.is_available() or not dist.is_initialized():
        return False
    world = comm.get_size(group_name)
    if world < 2 or world > 8 or dist.get_backend(comm.get_group(group_name)) != "nccl":
        return False
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False
    return True


def disable(group_name: str, why: str) -> None:
    _DISABLED[group_name] = why


def allreduce_buffers(group_name: str, m: int, n: int, dtype: torch.dtype, device: torch.device) -> ARBuffers:
    """Partial buffer (one [m, n] slot of ``dtype`` per rank: slot s receives rank s's partial) and
    zeroed flag words for a fused all-reduce of an [m, n] output over ``group_name``; a collective on first use of a shape (all ranks call it
    in the same order)."""
    key = (group_name, m, n, dtype, device.index)
    hit = _BUFS.get(key)
    if hit is not None:
        return hit
    import torch.distributed._symmetric_memory as symm

    group = comm.get_group(group_name)
    world = comm.get_size(group_name)
    tiles = math.ceil(m / 128) * math.ceil(n / 128)  # upper bound over the kernel's tile widths
    part = symm.empty(world * m * n, dtype=dtype, device=device)  # one [m, n] slot per rank
    flags = symm.empty(FLAG_BASE + world * tiles, dtype=torch.int32, device=device)
    flags.zero_()
    hp = symm.rendezvous(part, group)
    hf = symm.rendezvous(flags, group)
    torch.cuda.synchronize(device)
    dist.barrier(group=group)  # every rank's flags are zero before any launch uses them
    bufs = ARBuffers(part, flags, [int(p) for p in hp.buffer_ptrs], [int(p) for p in hf.buffer_ptrs],
                     int(hp.rank), int(hp.world_size), (hp, hf))
    _BUFS[key] = bufs
    return bufs


def reset() -> None:
    _BUFS.clear()
    _DISABLED.clear()
