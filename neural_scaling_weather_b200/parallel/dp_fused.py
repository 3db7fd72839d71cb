"""Data-parallel gradient reduction fused with the optimizer over NVLink peer memory.

Pure data parallelism on one node (``dp`` = world, 2..8 GPUs).  The reference reduces gradients with
DDP's bucketed all-reduce plus a comm hook that divides by dp (``distributed/mappings.py:217-341``)
and then every rank clips (``utils/trainer.py:416-448``) and steps the full optimizer
(``utils/optimizer_utils.py:56-72``).  Here:

* the optimizer's flat fp32 gradients, fp32 parameters and their 16-bit shadow live in symmetric
  memory (``torch.distributed._symmetric_memory``), so the extension's kernels get every rank's
  pointer;
* each rank owns one slice of every gradient bucket; when backward has produced a bucket (the same
  post-accumulate hooks as :class:`~.grad_sync.GradReducer`, plus ``ops.gradsink`` for in-place
  weight gradients), ``dp_reduce`` runs on a side stream: it announces the bucket with an
  epoch-tagged flag in every peer's flag array, waits (bounded) for every rank's announcement, pulls
  the owned slice from every rank with peer loads and writes ``sum / dp`` (rank order: the same
  bits on every launch) into the rank's own buffer, overlapped with the rest of backward;
* the clip norm's sums of squares run over the owned slices only and are all-reduced over dp;
* ``dp_adamw`` updates the owned slices and stores the new fp32 values and their 16-bit shadow into
  EVERY rank's buffers (the parameter all-gather rides on the update), and ``dp_barrier`` makes every
  rank wait until all owners have stored before its next forward;
* the AdamW moments are valid only on the owned slices (zero elsewhere); a checkpoint sums them over
  dp, so the saved optimizer state is the full ``torch.optim.AdamW`` layout as before.

Every wait in the kernels is bounded (the device error word records a timeout).  No TMA and no
multicast touches peer memory.  ``NSW_FUSED_DP=1`` selects this path (default: the NCCL reducer).
"""

from __future__ import annotations

import importlib
import os
from typing import Dict, List, Tuple

import torch
import torch.distributed as dist

from . import comm

FLAG_BASE = 16  # kDpFlagBase of the kernels


def available(space, optimizer_name: str, fp16_scaler: bool) -> Tuple[bool, str]:
    """Whether the fused path applies to this run (and why not)."""
    if os.environ.get("NSW_FUSED_DP", "0") != "1" or os.environ.get("NSW_FUSED_COLLECTIVES", "1") == "0":
        return False, "switched off (NSW_FUSED_DP=1 selects it)"
    if not (dist.is_initialized() and torch.cuda.is_available() and space.data.is_cuda):
        return False, "needs CUDA and a process group"
    if optimizer_name not in ("adam", "adamw") or fp16_scaler:
        return False, "needs the fused Adam/AdamW without fp16 loss scaling"
    dp, world = comm.get_size("dp"), comm.get_world_size()
    if dp < 2 or dp > 8 or world != dp:
        return False, "needs pure data parallelism over 2..8 ranks"
    if int(os.environ.get("LOCAL_WORLD_SIZE", world)) != world:
        return False, "needs all ranks on one node"
    if dist.get_backend(comm.get_group("dp")) != "nccl":
        return False, "needs the NCCL backend"
    # with tp = sp1 = sp2 = 1 every product reduction group of a parameter is the dp group
    if any(comm.get_size(g) != 1 for g in ("tp", "sp1", "sp2")):
        return False, "parameters reduced over other groups"
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False, "symmetric memory unavailable"
    return True, ""


class _Bucket:
    def __init__(self, slot: int, lo: int, hi: int, params):
        self.slot, self.lo, self.hi = slot, lo, hi
        self.params = params
        self.pending = len(params)
        self.own = (0, 0)


class FusedDPReducer:
    """Drop-in for :class:`~.grad_sync.GradReducer` (``no_sync``, ``finish``, ``reset``) whose
    buckets are reduced by ``dp_reduce`` and whose optimizer step is ``dp_adamw`` (see the module)."""

    sharded = True

    def __init__(self, space, bucket_cap_mb: float = 25.0):
        import torch.distributed._symmetric_memory as symm

        from ..ops import _ext, gradsink

        self.ext = _ext.require()
        self.space = space
        self.enabled = True
        self.dp = comm.get_size("dp")
        self.rank = comm.get_rank("dp")
        group = comm.get_group("dp")
        dev = space.data.device
        # flat buffers into symmetric memory (contents kept; .data / .grad views re-pointed)
        data = symm.empty(space.numel, dtype=torch.float32, device=dev)
        grad = symm.empty(space.numel, dtype=torch.float32, device=dev)
        data.copy_(space.data)
        grad.zero_()
        shadow = None
        if space.shadow is not None:
            shadow = symm.empty(space.numel, dtype=space.shadow.dtype, device=dev)
            shadow.copy_(space.shadow)
        space.rebind(data, grad, shadow)
        # buckets over the parameter order (the order backward produces gradients)
        cap = int(bucket_cap_mb * 1024 * 1024 // 4)
        self.buckets: List[_Bucket] = []
        self._param_bucket: Dict[int, _Bucket] = {}
        cur = None
        for i, p in enumerate(space.params):
            lo = space.offsets[i]
            hi = space.offsets[i + 1] if i + 1 < len(space.params) else space.numel
            if cur is None or (cur.hi - cur.lo) >= cap:
                cur = _Bucket(len(self.buckets), lo, hi, [])
                self.buckets.append(cur)
            cur.hi = hi
            cur.params.append(p)
            self._param_bucket[id(p)] = cur
        for b in self.buckets:
            n = b.hi - b.lo
            chunk = ((n + self.dp - 1) // self.dp + 3) // 4 * 4
            lo = min(b.lo + self.rank * chunk, b.hi)
            b.own = (lo, min(lo + chunk, b.hi))
            b.pending = len(b.params)
        self.slots = len(self.buckets) + 1  # the last slot is the optimizer's barrier
        flags = symm.empty(FLAG_BASE + self.dp * self.slots, dtype=torch.int32, device=dev)
        flags.zero_()
        handles = [symm.rendezvous(t, group) for t in (data, grad, flags) + ((shadow,) if shadow is not None else ())]
        self._handles = handles  # keep the rendezvous alive
        self.data_ptrs = [int(p) for p in handles[0].buffer_ptrs]
        self.grad_ptrs = [int(p) for p in handles[1].buffer_ptrs]
        self.flag_ptrs = [int(p) for p in handles[2].buffer_ptrs]
        self.shadow_ptrs = [int(p) for p in handles[3].buffer_ptrs] if shadow is not None else []
        self._flags = flags
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every rank's flags are zero before any kernel uses them
        # replicas start equal (as DDP's broadcast from the root)
        dist.broadcast(space.data, src=comm.get_root("dp"), group=group)
        if space.shadow is not None:
            space.refresh_shadow()
        self.stream = torch.cuda.Stream(device=dev)
        self._seen = set()
        self.epoch = 0
        self._open = False
        self._sync = True
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in space.params]
        gradsink.register(self._on_grad)
        # owned ranges of the whole buffer (for the norm and the optimizer), in buffer order
        self.owned = [b.own for b in sorted(self.buckets, key=lambda b: b.lo) if b.own[1] > b.own[0]]

    # ------------------------------------------------------------------ reducer interface
    def no_sync(self):
        from contextlib import contextmanager

        @contextmanager
        def ctx():
            old = self._sync
            self._sync = False
            try:
                yield
            finally:
                self._sync = old

        return ctx()

    def peers(self):
        return (self.grad_ptrs, self.data_ptrs, self.shadow_ptrs, self.flag_ptrs, self.rank, self.slots)

    def _open_epoch(self):
        if not self._open:
            self.epoch += 1
            self._open = True

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
        self._open_epoch()
        cur = torch.cuda.current_stream(self.space.data.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self.ext.dp_reduce(*self.peers(), b.slot, self.epoch, b.own[0], b.own[1], 1.0 / self.dp)
        b.pending = -1  # launched this step

    def finish(self):
        """Launch the buckets whose hooks did not all fire and make the compute stream wait for all
        reductions (the owned slices of .grad then hold the dp average)."""
        if not self._sync:
            return
        for b in self.buckets:
            if b.pending != -1:
                self._launch(b)
        torch.cuda.current_stream(self.space.data.device).wait_stream(self.stream)
        for b in self.buckets:
            b.pending = len(b.params)
        self._seen.clear()

    def reset(self):
        for b in self.buckets:
            b.pending = len(b.params)
        self._seen.clear()

    # ------------------------------------------------------------------ optimizer side
    def barrier_after_step(self):
        """Every rank waits until all owners have stored their updated parameters."""
        self.ext.dp_barrier(*self.peers(), self.slots - 1, self.epoch)
        self._open = False
