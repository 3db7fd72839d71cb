"""ERA5 HDF5 reader with the stateful sampling semantics of the synthetic dataset.

File layout (as consumed by ``utils/dataloaders/era5hdf5.py`` / ``era5hdf5_dali.py`` of the
reference): ``<root>/<name>/<year>.h5`` with datasets ``data[time, channel, lat, lon]``,
``time`` (hours since 1900-01-01), ``channel`` (names), ``latitude`` (721 values; the
south-pole row is dropped), ``longitude``; statistics in ``stats/stats_<tag>.h5``
(``global_mean``, ``global_std``) and invariants in ``invar/invariants.h5``
(``channel``, ``data[channel, lat, lon]``; ``orog`` is min-max normalised, ``coslat`` is
computed).  Years in ``valid_years``/``test_years`` are held out of training.

Samples, epochs, dp sharding and resume follow :class:`SyntheticERA5` (which documents
the reference's DALI semantics); windows are read with one strided read per year file
(local spatial slab when ``read_local``), normalised on the host and moved to the GPU
through pinned memory by :class:`HDF5Loader`.  Requires ``h5py``.
"""

from __future__ import annotations

import glob
import os
from typing import List

import numpy as np
import torch

from ..parallel import comm
from .synthetic import EPOCH0, SyntheticERA5


def _h5py():
    try:
        import h5py

        return h5py
    except Exception as e:  # pragma: no cover - depends on the environment
        raise RuntimeError("the HDF5 ERA5 reader needs h5py, which is not installed") from e


class Era5HDF5Dataset(SyntheticERA5):
    """Reads ERA5 windows from yearly HDF5 files."""

    @classmethod
    def instantiate_from_cfg(cls, cfg, mode):
        d = cfg.data
        return cls(
            root=d.get("root", "/data"), name=d.name, tag=d.tag, mode=mode, dt_scale=int(d.dt_scale),
            temporal_context_window=int(cfg.train.temporal_context_window),
            num_rollout_steps=int(cfg.train.num_rollout_steps), model_patch_size=int(cfg.model.patch_size),
            limit_nsamples=int(d.limit_nsamples_val if mode == "valid" else d.limit_nsamples),
            valid_years=list(d.valid_years), test_years=list(d.test_years),
            invariants=list(d.invariants) if d.invariants else [], read_local=bool(d.read_local),
            micro_batch_size=int(cfg.parallelism.micro_batch_size))

    def __init__(self, root="/data", name="latlon_025deg_hdf5_1h", tag="v1.0", mode="train", dt_scale=1,
                 temporal_context_window=1, num_rollout_steps=1, model_patch_size=1, limit_nsamples=-1,
                 valid_years=(), test_years=(), invariants=(), read_local=False, micro_batch_size=1,
                 seed=42):
        h5py = _h5py()
        self.location = os.path.join(root, name)
        self.tag, self.mode = tag, mode
        self.dt_scale = dt_scale
        self.temporal_context_window = temporal_context_window
        self.num_rollout_steps = num_rollout_steps
        self.model_patch_size = model_patch_size
        self.invariants = list(invariants)
        self.micro_batch_size = micro_batch_size
        self.read_local = read_local
        self.seed = seed
        self.shuffle = mode == "train"
        self.return_timestamp = False
        paths = sorted(glob.glob(os.path.join(self.location, "*.h5")),
                       key=lambda x: int(os.path.basename(x)[:-3]))
        if not paths:
            raise FileNotFoundError(f"no HDF5 files in {self.location}")
        years = [int(os.path.basename(p)[:-3]) for p in paths]
        hold = set(valid_years) | set(test_years)
        if mode == "train":
            keep = [y not in hold for y in years]
        elif mode == "valid":
            keep = [y in set(valid_years) for y in years]
        else:
            keep = [y in set(test_years) for y in years]
        self.paths = [p for p, k in zip(paths, keep) if k]
        self.years = [y for y, k in zip(years, keep) if k]
        with h5py.File(self.paths[0], "r") as f:
            self.era5_channels = [n.decode() if isinstance(n, bytes) else str(n) for n in f["channel"][:]]
            t = f["time"][:]
            self.dt_hours = np.timedelta64(int(t[1] - t[0]), "h")
            self.latitudes = f["latitude"][:-1]
            self.longitudes = f["longitude"][:]
        per_year = []
        for p in self.paths:
            with h5py.File(p, "r") as f:
                per_year.append(EPOCH0 + f["time"][:].astype("timedelta64[h]"))
        self.n_per_year = np.array([len(t) for t in per_year], dtype=np.int64)
        self.year_offsets = np.concatenate(([0], np.cumsum(self.n_per_year)[:-1]))
        self.all_times = np.concatenate(per_year)
        self.n_samples_total = len(self.all_times) - (temporal_context_window + num_rollout_steps - 1) * dt_scale
        if limit_nsamples > 0:
            self.n_samples_total = min(self.n_samples_total, limit_nsamples)
        self.n_samples_shard = self.n_samples_total // comm.get_size("dp")
        self.shard_id = comm.get_rank("dp")
        self.num_steps_per_epoch = self.n_samples_shard // micro_batch_size
        self.nlat, self.nlon = len(self.latitudes), len(self.longitudes)
        self._set_shapes_and_metadata()
        with h5py.File(os.path.join(self.location, "stats", f"stats_{tag}.h5"), "r") as f:
            self.means = f["global_mean"][:].reshape(1, -1, 1, 1).astype(np.float32)
            self.stds = f["global_std"][:].reshape(1, -1, 1, 1).astype(np.float32)
        self.invar = self.get_invariants() if self.invariants else None
        self._files = {}
        self.resume_skip_batches = 0
        self.iterations_to_skip = 0
        self.ckpt_epoch = 0

    def get_invariants(self):
        h5py = _h5py()
        wanted = [v for v in self.invariants if v != "coslat"]
        arrs: List[np.ndarray] = []
        if wanted:
            with h5py.File(os.path.join(self.location, "invar", "invariants.h5"), "r") as f:
                names = [n.decode() if isinstance(n, bytes) else str(n) for n in f["channel"][:]]
                idx = [i for i, n in enumerate(names) if n in wanted]
                data = f["data"][idx, :-1, :]
                names = [names[i] for i in idx]
            if "orog" in names:
                o = data[names.index("orog")]
                data[names.index("orog")] = (o - o.min()) / o.max()
            arrs.append(data)
        if "coslat" in self.invariants:
            c = np.cos(np.deg2rad(self.latitudes))[None, :, None] * np.ones((1, 1, len(self.longitudes)))
            arrs.append(c)
        arr = np.concatenate(arrs)
        lat_sl, lon_sl = self.metadata["sp_slices"]
        return arr[:, lat_sl, lon_sl].astype(np.float32)

    def _file(self, yi):
        if yi not in self._files:
            self._files[yi] = _h5py().File(self.paths[yi], "r")
        return self._files[yi]

    def _read_hours(self, hours: np.ndarray) -> np.ndarray:
        lat_sl, lon_sl = self.metadata["sp_slices"]
        out = np.empty((len(hours), len(self.era5_channels), lat_sl.stop - lat_sl.start,
                        lon_sl.stop - lon_sl.start), dtype=np.float32)
        ts = EPOCH0 + np.asarray(hours).astype("timedelta64[h]")
        gidx = np.searchsorted(self.all_times, ts)
        for j, g in enumerate(gidx):
            yi = int(np.searchsorted(self.year_offsets, g, side="right") - 1)
            li = int(g - self.year_offsets[yi])
            ds = self._file(yi)["data"]
            out[j] = ds[li, :, lat_sl, lon_sl] if self.read_local else ds[li][:, lat_sl, lon_sl]
        return out

    def generate(self, hours, device="cpu", dtype=torch.float32):
        x = (self._read_hours(np.asarray(hours)) - self.means[0]) / self.stds[0]
        t = torch.from_numpy(x.astype(np.float32))
        if torch.device(device).type == "cuda":
            t = t.pin_memory().to(device, non_blocking=True)
        return t.to(dtype)


def make_hdf5_loader(cfg, dataset, mode):
    from .synthetic import SyntheticLoader

    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    return SyntheticLoader(dataset, micro_batch_size=int(cfg.parallelism.micro_batch_size), device=dev,
                           mode=mode), None
