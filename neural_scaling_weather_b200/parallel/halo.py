"""Shifted-window roll of spatially sharded activations over NVLink peer memory.

The reference rolls a tensor sharded over sp1 (latitude) and sp2 (longitude) one dimension at a
time with NCCL point-to-point sends plus copies (``distributed/helpers.py:192-277``), once before
and once after every shifted-window attention (``models/swin_helpers.py:399-433``), and the same
in reverse in the backward pass.  Here one call rolls both dimensions: ``halo_roll.cu`` packs this
rank's edge bands (|shift| rows / columns) into a symmetric buffer and signals the peers, copies
the locally sourced bulk of the output, then pulls the remaining rows from the neighbours' band
buffers with peer loads (epoch-tagged flags, bounded waits; see the kernel file).

Applies to a (B, T, H_l, W_l, C) CUDA tensor rolled along (H, W) over the ``sp1-sp2`` group of 2..8
GPUs of one node under NCCL, with every |shift| smaller than every split shard and C times the
element size a multiple of 16 bytes; otherwise ``parallel.helpers`` does the NCCL roll.
``NSW_FUSED_HALO=0`` (or ``NSW_FUSED_COLLECTIVES=0``) selects the NCCL roll.
"""

from __future__ import annotations

import importlib
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import comm
from .helpers import offsets

GROUP = "sp1-sp2"
FLAG_WORDS = 48  # kHaloFlagWords of ops/csrc/kernels.h
_GROUP_INFO: Optional["_Group"] = None
_BUFS: Dict[int, "_Bands"] = {}


@dataclass
class _Group:
    rank: int
    world: int
    coord1: List[int]
    coord2: List[int]


@dataclass
class _Bands:
    band: torch.Tensor
    flags: torch.Tensor
    band_ptrs: List[int]
    flag_ptrs: List[int]
    handles: tuple


def _enabled() -> bool:
    return os.environ.get("NSW_FUSED_HALO", "1") != "0" and os.environ.get("NSW_FUSED_COLLECTIVES", "1") != "0"


def available(x: torch.Tensor, shifts: Sequence[int], dims: Sequence[int], comm_names: Sequence[str],
              shapes) -> bool:
    """The fused roll applies to this call (see the module docstring)."""
    if not _enabled() or not x.is_cuda or not dist.is_initialized() or shapes is None:
        return False
    if tuple(comm_names) != ("sp1", "sp2") or x.dim() != 5:
        return False
    if tuple(d % 5 for d in dims) != (2, 3) or len(shifts) != 2:
        return False
    world = comm.get_size(GROUP)
    if world < 2 or world > 8 or dist.get_backend(comm.get_group(GROUP)) != "nccl":
        return False
    n1, n2 = comm.get_size("sp1"), comm.get_size("sp2")
    if n1 * n2 != world or len(shapes[0]) != n1 or len(shapes[1]) != n2:
        return False
    sh, sw = _norm(shifts[0], sum(shapes[0])), _norm(shifts[1], sum(shapes[1]))
    if (n1 > 1 and abs(sh) >= min(shapes[0])) or (n2 > 1 and abs(sw) >= min(shapes[1])):
        return False
    if (x.shape[-1] * x.element_size()) % 16 or x.data_ptr() % 16:
        return False
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False
    return True


def _norm(s: int, n: int) -> int:
    """The shift in (-n/2, n/2] equivalent to ``s`` modulo ``n`` (the thinner band)."""
    s = int(s) % n
    return s - n if s > n // 2 else s


def _group() -> _Group:
    """This rank's place in the sp1-sp2 group and every member's (sp1, sp2) shard (collective, once)."""
    global _GROUP_INFO
    if _GROUP_INFO is None:
        g = comm.get_group(GROUP)
        world = comm.get_size(GROUP)
        mine = torch.tensor([comm.get_rank("sp1"), comm.get_rank("sp2")], dtype=torch.int64, device="cuda")
        allc = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allc, mine, group=g)
        c = torch.stack(allc).cpu()
        _GROUP_INFO = _Group(rank=dist.get_rank(g), world=world, coord1=c[:, 0].tolist(), coord2=c[:, 1].tolist())
    return _GROUP_INFO


def _bands(nbytes: int, device: torch.device) -> _Bands:
    """Symmetric band buffer of at least ``nbytes`` and the flag words (a collective on first use of a size
    class; every rank of the group asks for the same sizes in the same order)."""
    size = 1 << max(20, (max(nbytes, 16) - 1).bit_length())  # power-of-two classes from 1 MiB
    hit = _BUFS.get(size)
    if hit is not None:
        return hit
    import torch.distributed._symmetric_memory as symm

    g = comm.get_group(GROUP)
    band = symm.empty(size, dtype=torch.uint8, device=device)
    flags = symm.empty(FLAG_WORDS, dtype=torch.int32, device=device)
    flags.zero_()
    hb = symm.rendezvous(band, g)
    hf = symm.rendezvous(flags, g)
    torch.cuda.synchronize(device)
    dist.barrier(group=g)  # every rank's flags are zero before any roll uses them
    b = _Bands(band, flags, [int(p) for p in hb.buffer_ptrs], [int(p) for p in hf.buffer_ptrs], (hb, hf))
    _BUFS[size] = b
    return b


def _ext():
    from ..ops import _ext as E

    return E.require()


def roll(x: torch.Tensor, shifts: Tuple[int, int], shapes) -> torch.Tensor:
    """``torch.roll(x_global, shifts, dims=(2, 3))`` restricted to this rank's shard."""
    ext = _ext()
    gi = _group()
    n1, n2 = comm.get_size("sp1"), comm.get_size("sp2")
    h_off, w_off = offsets(list(shapes[0])), offsets(list(shapes[1]))
    h_off = list(h_off) + [sum(shapes[0])]
    w_off = list(w_off) + [sum(shapes[1])]
    sh, sw = _norm(shifts[0], h_off[-1]), _norm(shifts[1], w_off[-1])
    x = x.contiguous()
    out = torch.empty_like(x)
    geom = [n1, n2, sh, sw, gi.rank]
    need = ext.halo_band_bytes(x, geom, h_off, w_off, gi.coord1, gi.coord2)
    b = _bands(need, x.device)
    ext.halo_roll(x, out, geom, h_off, w_off, gi.coord1, gi.coord2, b.band_ptrs, b.flag_ptrs)
    return out


def reset() -> None:
    global _GROUP_INFO
    _GROUP_INFO = None
    _BUFS.clear()
