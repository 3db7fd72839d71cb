"""Process-group registry for the DP x TP x SP1 x SP2 layout.

Same contract as ``utils/comm.py`` in the reference: a module-level registry of named
groups (``dp, tp, sp1, sp2, sp1-sp2, pp, tp-sp1-sp2, dp-sp1-sp2``); getters return size 1
and rank 0 for a group that was never created, which is how single-process code and the
single-rank oracle in the tests run the distributed layers unchanged
(``utils/comm.py:11-79``).  ``init`` reads ``WORLD_SIZE``/``RANK`` (falling back to
``SLURM_NTASKS``/``SLURM_PROCID``), derives ``dp = world / (tp*sp1*sp2*pp)`` and builds
every group (``utils/comm.py:82-148``).

Beyond the reference, the registry records each group's member list, so the fused
peer-memory kernels (which address peers by global rank) can map a group-local index to
a device.
"""

from __future__ import annotations

import datetime
import logging
import os
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .rank_grid import RankGrid

_COMM_GROUPS: Dict[str, "dist.ProcessGroup"] = {}
_GROUP_RANKS: Dict[str, List[int]] = {}
_GRID: Optional[RankGrid] = None

GROUP_NAMES = ("dp", "tp", "sp1", "sp2", "sp1-sp2", "pp", "tp-sp1-sp2", "dp-sp1-sp2")


def get_names():
    return _COMM_GROUPS.keys()


def is_initialized(comm_name: str) -> bool:
    return comm_name in _COMM_GROUPS


def get_group(comm_name: str):
    if not is_initialized(comm_name):
        raise IndexError(f"communicator {comm_name!r} is not initialized")
    return _COMM_GROUPS[comm_name]


def get_size(comm_name: str) -> int:
    if not dist.is_initialized() or not is_initialized(comm_name):
        return 1
    return dist.get_world_size(group=get_group(comm_name))


def get_rank(comm_name: str) -> int:
    if not dist.is_initialized() or not is_initialized(comm_name):
        return 0
    return dist.get_rank(group=get_group(comm_name))


def get_root(comm_name: str) -> int:
    if not dist.is_initialized() or not is_initialized(comm_name):
        return 0
    return min(dist.get_process_group_ranks(get_group(comm_name)))


def get_group_ranks(comm_name: str) -> List[int]:
    """Global ranks of this rank's group ``comm_name`` (``[0]`` when not distributed)."""
    if not dist.is_initialized() or not is_initialized(comm_name):
        return [get_world_rank()]
    return list(_GROUP_RANKS[comm_name])


def get_world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def get_world_rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def get_local_rank() -> int:
    if not dist.is_initialized():
        return 0
    if os.getenv("LOCAL_RANK") is not None:
        return int(os.environ["LOCAL_RANK"])
    n = torch.cuda.device_count() if torch.cuda.is_available() else 1
    return get_world_rank() % max(n, 1)


def get_grid() -> Optional[RankGrid]:
    return _GRID


def init_process_group(backend: str, timeout_s: Optional[float] = None) -> None:
    if dist.is_initialized():
        return
    if os.getenv("WORLD_SIZE") is not None and os.getenv("RANK") is not None:
        world_size = int(os.environ["WORLD_SIZE"])
        world_rank = int(os.environ["RANK"])
    else:
        world_size = int(os.getenv("SLURM_NTASKS", 1))
        world_rank = int(os.getenv("SLURM_PROCID", 0))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    kwargs = {}
    if timeout_s is not None:
        kwargs["timeout"] = datetime.timedelta(seconds=timeout_s)
    if backend == "nccl" and torch.cuda.is_available():
        local = int(os.getenv("LOCAL_RANK", world_rank % max(torch.cuda.device_count(), 1)))
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend=backend, rank=world_rank, world_size=world_size, **kwargs)


def init(cfg, timeout_s: Optional[float] = None) -> None:
    """Initialise torch.distributed and every named group from ``cfg.parallelism``."""
    par = cfg.parallelism
    backend = par.backend
    if backend == "nccl" and not torch.cuda.is_available():
        backend = "gloo"
    init_process_group(backend, timeout_s=timeout_s)
    tp, sp1, sp2, pp = int(par.tp), int(par.sp1), int(par.sp2), int(par.pp)
    if pp != 1:
        raise AssertionError("pipeline parallelism is not supported (pp must be 1)")
    mp = tp * sp1 * sp2 * pp
    world = get_world_size()
    if world % mp != 0:
        raise AssertionError(
            f"world size {world} must be divisible by model parallel size {mp} "
            f"(TP={tp}, SP=({sp1}, {sp2}), PP={pp})"
        )
    dp = world // mp
    if get_world_rank() == 0:
        logging.info(f"Using backend {backend}")
        logging.info(f"Setting DP = {dp}, TP = {tp}, SP = ({sp1}, {sp2}), PP = {pp}")
    init_model_parallel_info(tp=tp, sp1=sp1, sp2=sp2, dp=dp, pp=pp, order=par.order)


def init_model_parallel_info(tp=1, pp=1, dp=1, sp1=1, sp2=1, order="sp1-sp2-tp-pp-dp"):
    """Create every named group; each rank keeps the group that contains it."""
    global _GRID
    _GRID = RankGrid(tp=tp, dp=dp, pp=pp, sp1=sp1, sp2=sp2, order=order)
    me = get_world_rank()
    for name in GROUP_NAMES:
        for ranks in _GRID.get_ranks(name):
            group = dist.new_group(ranks)
            if me in ranks:
                _COMM_GROUPS[name] = group
                _GROUP_RANKS[name] = list(ranks)


def reset() -> None:
    """Forget every group (used by tests and at shutdown)."""
    global _GRID
    _COMM_GROUPS.clear()
    _GROUP_RANKS.clear()
    _GRID = None


def all_model_groups_exist(model):
    """Assert that every group named in a parameter's ``comm_metadata`` exists."""
    for name, param in model.named_parameters():
        meta = getattr(param, "comm_metadata", None)
        if meta is None:
            continue
        for key in ("shared", "reduce", "sharded"):
            for comm_name in meta.get(key, []):
                if comm_name is not None and not is_initialized(comm_name) and dist.is_initialized():
                    raise AssertionError(
                        f"comm group {comm_name!r} not initialized for parameter {name!r}"
                    )
    return model
