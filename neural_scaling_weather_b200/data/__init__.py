"""Datasets, loaders and the pre-processor (``utils/data_utils.py`` of the reference).

``get_dataset(cfg, mode)`` returns the synthetic ERA5-shaped dataset for
``data.loader == 'synthetic'`` and the HDF5 readers for ``'pytorch'``/``'dali'`` (those need
``h5py``; DALI itself is not used: its HDF5 windows are read by the same stateful reader).
``get_data_loader(cfg, dataset, mode)`` returns ``(loader, sampler)`` like the reference.
"""

from __future__ import annotations

from collections import deque
from typing import Deque, Iterable, Iterator, Optional, Tuple, Union

import torch
import torch.nn as nn

from .synthetic import SyntheticERA5, SyntheticLoader


def get_dataset(cfg, mode: str = "train"):
    loader = cfg.data.loader
    if loader == "synthetic":
        return SyntheticERA5.instantiate_from_cfg(cfg, mode=mode, seed=42)
    if loader in ("pytorch", "dali"):
        from .era5hdf5 import Era5HDF5Dataset

        return Era5HDF5Dataset.instantiate_from_cfg(cfg, mode)
    raise ValueError(f"unknown data loader {loader!r}")


def _device_for_loader():
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


def get_data_loader(cfg, dataset, mode: str = "train"):
    d = cfg.data
    if mode == "train" and d.limit_nsamples > 0 and d.limit_nsamples < d.batch_size:
        raise ValueError(f"not enough training samples ({d.limit_nsamples}) for batch size {d.batch_size}")
    if mode in ("valid", "test") and d.limit_nsamples_val > 0 and d.limit_nsamples_val < d.batch_size:
        raise ValueError(f"not enough validation samples ({d.limit_nsamples_val}) for batch size {d.batch_size}")
    mbs = int(cfg.parallelism.micro_batch_size)
    if isinstance(dataset, SyntheticERA5):
        return SyntheticLoader(dataset, micro_batch_size=mbs, device=_device_for_loader(), mode=mode), None
    from .era5hdf5 import make_hdf5_loader

    return make_hdf5_loader(cfg, dataset, mode)


def device_prefetch(batches: Iterable[torch.Tensor], device, depth: int = 1) -> Iterator[torch.Tensor]:
    """Yield ``batches`` on ``device``, copying the next ``depth`` host batches on a side stream
    while the current one is consumed (the role of the DALI pipeline's device prefetch queue,
    ``utils/dataloaders/era5hdf5_dali.py:70-100`` of the reference).

    The copies land in a ring of ``depth + 1`` device buffers allocated once (per batch shape),
    so the steady state allocates nothing and no block waits on another stream's work: a yielded
    batch is valid until the next one is requested, after which its buffer is refilled.  Copies
    are ordered with events: the compute stream waits for a batch's copy before using it, and a
    buffer is refilled only after the work that used it has been enqueued and, on the device,
    finished.  Host batches should be pinned for the copies to be asynchronous; batches already
    on the device, and every batch when ``device`` is not CUDA, pass through unchanged."""
    device = torch.device(device)
    if device.type != "cuda":
        yield from batches
        return
    it = iter(batches)
    stream = torch.cuda.Stream(device=device)
    nbuf = depth + 1
    ring: list = [None] * nbuf       # device buffers, filled round-robin
    released: list = [None] * nbuf   # per buffer: compute-stream event after its last use
    pending: Deque = deque()
    slot = 0

    def issue() -> bool:
        nonlocal slot
        try:
            b = next(it)
        except StopIteration:
            return False
        if b.is_cuda:
            pending.append((b, None, None))
            return True
        k = slot % nbuf
        slot += 1
        cur = torch.cuda.current_stream(device)
        buf = ring[k]
        if buf is None or buf.shape != b.shape or buf.dtype != b.dtype:
            buf = ring[k] = torch.empty(b.shape, dtype=b.dtype, device=device)
            released[k] = None
        if released[k] is not None:
            stream.wait_event(released[k])  # the batch that last used this buffer is done
        else:
            stream.wait_stream(cur)  # fresh buffer, allocated on the compute stream
        with torch.cuda.stream(stream):
            buf.copy_(b, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
        pending.append((buf, ev, k))
        return True

    try:
        for _ in range(depth):
            if not issue():
                break
        while pending:
            d, ev, k = pending.popleft()
            cur = torch.cuda.current_stream(device)
            if ev is not None:
                cur.wait_event(ev)
            issue()
            yield d
            if k is not None:  # the consumer's work on this batch is enqueued on `cur`
                done = torch.cuda.Event()
                done.record(cur)
                released[k] = done
    finally:
        # copies still in flight (the consumer stopped early) complete before the ring's memory
        # can be handed out again on the compute stream
        torch.cuda.current_stream(device).wait_stream(stream)


def get_preprocessor(cfg, dataset):
    return PreProcessor.instantiate_from_cfg(cfg, dataset)


class PreProcessor(nn.Module):
    """Appends invariants on the channel axis and splits inputs / targets by rollout steps."""

    @classmethod
    def instantiate_from_cfg(cls, cfg, dataset):
        return cls(dataset, invariants=cfg.data.invariants, send_to_device=True,
                   num_rollout_steps=cfg.train.num_rollout_steps)

    def __init__(self, dataset, invariants=None, send_to_device=True, num_rollout_steps=1):
        super().__init__()
        self.add_invariants = bool(invariants)
        if self.add_invariants:
            inv = torch.from_numpy(dataset.invar).unsqueeze(0).unsqueeze(0)
            self.register_buffer("invariants", inv)
        self.send_to_device = send_to_device
        self.num_rollout_steps = int(num_rollout_steps)

    def forward(self, batch: torch.Tensor, device: torch.device, mode: str = "train"
                ) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
        B, T, C, H, W = batch.shape
        if self.send_to_device:
            batch = batch.to(device, non_blocking=True)
        if self.add_invariants:
            batch = torch.cat([batch, self.invariants.to(batch.dtype).expand(B, T, -1, H, W)], dim=2)
        if mode == "train":
            nrs = self.num_rollout_steps
            return batch[:, :-nrs], batch[:, -nrs:, :C]
        if mode == "inference":
            return batch
        raise ValueError(f"invalid preprocessor mode {mode!r}")
