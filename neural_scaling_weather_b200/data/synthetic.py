"""Seeded synthetic ERA5-shaped dataset with the reference loader's stateful semantics.

Fields.  Channel ``c`` at absolute hour ``tau`` (hours since 1900-01-01) is

    f_c(tau, lat, lon) = sum_i a_ci * sin(m_ci * (lon - 2 pi v_c tau / (nlon * dt_scale))
                                        + n_ci * colat + p_ci) / s_c + noise,

a sum of ``n_modes`` low-order sinusoids advected eastward by ``v_c`` grid cells per model
step (``v_c`` in ``[advect_min, advect_max]``), scaled to unit variance, plus
``N(0, noise)`` white noise.  Consecutive model steps are therefore the same pattern
shifted east by whole cells, plus fresh noise: the target is the advected input.  All
random numbers come from a counter-based hash of ``(seed, channel, mode)`` and
``(seed, tau, channel, pixel)``, so a sample is a pure function of its timestamp and is
identical on CPU and GPU.  Values are already standardised; the dataset still exposes
per-channel physical ``means``/``stds`` (seeded) for un-normalising, as the ERA5 statistics
files do.

Sampling semantics follow ``utils/dataloaders/era5hdf5_dali.py`` of the reference:

* a sample is the window ``[k, k + dt_scale, ..., k + (T + nrs - 1) dt_scale]`` hours;
  ``n_samples_total = n_times - (T + nrs - 1) dt_scale`` (``:406-420``);
* each epoch permutes ``range(n_samples_total)`` with
  ``numpy.random.default_rng(seed + ckpt_epoch + epoch_idx)`` and keeps the contiguous dp
  shard ``[n_shard * dp_rank, n_shard * (dp_rank + 1))`` (``:533-556``);
* after a restore, the first epoch skips ``n_mbs_in_epoch`` micro-batches (``:536-566``);
* the local spatial shard is the patch-aware split of lat over sp1 and lon over sp2.
"""

from __future__ import annotations

import math
from typing import Iterator, List

import numpy as np
import torch

from ..parallel import comm
from ..parallel.helpers import compute_split_shapes_for_patching
from ..utils.misc import build_spherical_area_weights, get_local_slice, get_spatial_coords

EPOCH0 = np.datetime64("1900-01-01T00", "h")

_M1 = 0x7FEB352D
_M2 = 0x846CA68B
_MASK32 = 0xFFFFFFFF


def _hash32(x: torch.Tensor) -> torch.Tensor:
    """lowbias32 integer hash (Wellons) on int64 tensors holding uint32 values."""
    x = x & _MASK32
    x = x ^ (x >> 16)
    x = (x * _M1) & _MASK32
    x = x ^ (x >> 15)
    x = (x * _M2) & _MASK32
    x = x ^ (x >> 16)
    return x


def _uniform(key: torch.Tensor) -> torch.Tensor:
    """Uniform in (0, 1) from a hashed key (float64)."""
    return (_hash32(key).double() + 0.5) / 4294967296.0


def _normal(key: torch.Tensor) -> torch.Tensor:
    """Standard normal from a key via Box-Muller on two decorrelated hashes."""
    u1 = _uniform(key * 2 + 1)
    u2 = _uniform(_hash32(key * 2 + 0x9E3779B9))
    return torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)


def channel_names(sfc_vars: List[str], pl_vars: List[str], levels: List[int]) -> List[str]:
    names = list(sfc_vars)
    for v in pl_vars:
        names.extend(f"{v}{lev}" for lev in levels)
    return names


class SyntheticERA5:
    """Synthetic stand-in for the ERA5 HDF5 datasets (same metadata and state API)."""

    @classmethod
    def instantiate_from_cfg(cls, cfg, mode: str, seed: int = 42):
        d = cfg.data
        syn = d.get("synthetic", None) or {}
        return cls(
            mode=mode,
            nlat=int(syn.get("nlat", 720)),
            nlon=int(syn.get("nlon", 1440)),
            sfc_vars=list(syn.get("sfc_vars", ["u10m", "v10m", "t2m", "tcwv", "msl"])),
            pl_vars=list(syn.get("pl_vars", ["u", "v", "z", "t", "q"])),
            levels=list(d.levels),
            n_modes=int(syn.get("n_modes", 16)),
            noise=float(syn.get("noise", 0.1)),
            advect_min=int(syn.get("advect_min", 1)),
            advect_max=int(syn.get("advect_max", 3)),
            n_times=int(syn.get("n_samples", 1460)),
            data_seed=int(syn.get("seed", 42)),
            dt_scale=int(d.dt_scale),
            temporal_context_window=int(cfg.train.temporal_context_window),
            num_rollout_steps=int(cfg.train.num_rollout_steps),
            model_patch_size=int(cfg.model.patch_size),
            limit_nsamples=int(d.limit_nsamples_val if mode == "valid" else d.limit_nsamples),
            invariants=list(d.invariants) if d.invariants else [],
            micro_batch_size=int(cfg.parallelism.micro_batch_size),
            seed=seed,
        )

    def __init__(self, mode="train", nlat=720, nlon=1440, sfc_vars=None, pl_vars=None,
                 levels=None, n_modes=16, noise=0.1, advect_min=1, advect_max=3, n_times=1460,
                 data_seed=42, dt_scale=6, temporal_context_window=1, num_rollout_steps=1,
                 model_patch_size=1, limit_nsamples=-1, invariants=None, micro_batch_size=1,
                 seed=42, return_timestamp=False):
        self.mode = mode
        self.nlat, self.nlon = nlat, nlon
        levels = levels if levels is not None else []
        self.era5_channels = channel_names(sfc_vars or [], pl_vars or [], levels)
        self.n_modes, self.noise = n_modes, noise
        self.data_seed = data_seed
        self.dt_scale = dt_scale
        self.temporal_context_window = temporal_context_window
        self.num_rollout_steps = num_rollout_steps
        self.model_patch_size = model_patch_size
        self.invariants = invariants or []
        self.micro_batch_size = micro_batch_size
        self.seed = seed
        self.shuffle = mode == "train"
        self.return_timestamp = return_timestamp
        self.dt_hours = np.timedelta64(1, "h")

        # time axis (hourly); splits live in different years
        start = {"train": "1980-01-01T00", "valid": "2017-01-01T00"}.get(mode, "2018-01-01T00")
        self.all_times = np.datetime64(start, "h") + np.arange(n_times).astype("timedelta64[h]")
        self.n_samples_total = n_times - (temporal_context_window + num_rollout_steps - 1) * dt_scale
        if limit_nsamples > 0:
            self.n_samples_total = min(self.n_samples_total, limit_nsamples)
        if self.n_samples_total <= 0:
            raise ValueError("synthetic dataset too short for the temporal window")
        self.n_samples_shard = self.n_samples_total // comm.get_size("dp")
        self.shard_id = comm.get_rank("dp")
        self.num_steps_per_epoch = self.n_samples_shard // micro_batch_size

        # grid, split and metadata
        self.latitudes = np.linspace(90.0, -90.0, nlat + 1)[:-1]  # south pole row dropped
        self.longitudes = np.arange(nlon) * (360.0 / nlon)
        self._set_shapes_and_metadata()

        # per-channel field parameters
        C = len(self.era5_channels)
        g = torch.Generator().manual_seed(data_seed)
        self.m = torch.randint(1, 7, (C, n_modes), generator=g).double()
        self.n = torch.randint(0, 6, (C, n_modes), generator=g).double()
        self.p = torch.rand(C, n_modes, generator=g, dtype=torch.float64) * 2 * math.pi
        self.a = torch.rand(C, n_modes, generator=g, dtype=torch.float64) + 0.25
        self.v = torch.randint(advect_min, advect_max + 1, (C,), generator=g).double()
        self.scale = torch.sqrt((self.a ** 2).sum(1) / 2.0 + noise ** 2)
        phys_std = torch.rand(C, generator=g, dtype=torch.float64) * 20 + 0.5
        phys_mean = torch.rand(C, generator=g, dtype=torch.float64) * 300 - 10
        self.means = phys_mean.numpy().reshape(1, C, 1, 1).astype(np.float32)
        self.stds = phys_std.numpy().reshape(1, C, 1, 1).astype(np.float32)
        self.invar = self.get_invariants() if self.invariants else None

        # checkpoint / resume state
        self.resume_skip_batches = 0
        self.iterations_to_skip = 0
        self.ckpt_epoch = 0
        self.last_epoch = None
        self.index_permutation = None

    # ------------------------------------------------------------------ metadata
    def _set_shapes_and_metadata(self):
        area = build_spherical_area_weights(self.latitudes)
        sp1 = compute_split_shapes_for_patching(self.nlat, comm.get_size("sp1"), self.model_patch_size)
        sp2 = compute_split_shapes_for_patching(self.nlon, comm.get_size("sp2"), self.model_patch_size)
        lat_sl = get_local_slice(sp1, comm.get_rank("sp1"))
        lon_sl = get_local_slice(sp2, comm.get_rank("sp2"))
        lat_loc, lon_loc = self.latitudes[lat_sl], self.longitudes[lon_sl]
        self.metadata = {
            "sp_shapes": [sp1, sp2],
            "sp_slices": [lat_sl, lon_sl],
            "spatial_dims": [len(lat_loc), len(lon_loc)],
            "channels": self.era5_channels,
            "n_channels": len(self.era5_channels),
            "coords": get_spatial_coords((lat_loc, lon_loc)).float(),
            "area_weights": area[lat_sl, None].float(),
            "temporal_context_window": self.temporal_context_window,
            "num_rollout_steps": self.num_rollout_steps,
            "dt_hours": self.dt_hours,
            "dt_scale": self.dt_scale,
            "global_latitudes": self.latitudes,
            "global_longitudes": self.longitudes,
        }

    def get_metadata(self):
        md = dict(self.metadata)
        md.update(n_samples_total=self.n_samples_total, n_samples_shard=self.n_samples_shard,
                  num_steps_per_epoch=self.num_steps_per_epoch)
        return md

    def get_invariants(self) -> np.ndarray:
        """lsm (smooth 0/1 pattern), orog (min-max normalised), coslat; local slice."""
        lat = torch.from_numpy(np.deg2rad(self.latitudes))
        lon = torch.from_numpy(np.deg2rad(self.longitudes))
        LAT, LON = torch.meshgrid(lat, lon, indexing="ij")
        out = []
        for name in self.invariants:
            if name == "lsm":
                out.append((torch.sin(3 * LON) * torch.cos(2 * LAT) > 0.2).double())
            elif name == "orog":
                o = torch.relu(torch.sin(5 * LON + 1.0) * torch.cos(3 * LAT)) * 3000.0
                low, high = o.min(), o.max()
                out.append((o - low) / high)
            elif name == "coslat":
                out.append(torch.cos(LAT))
            else:
                raise ValueError(f"unknown invariant {name!r}")
        arr = torch.stack(out).numpy()
        lat_sl, lon_sl = self.metadata["sp_slices"]
        return arr[:, lat_sl, lon_sl].astype(np.float32)

    # ------------------------------------------------------------------ fields
    def hours_since_1900(self, timestamps) -> np.ndarray:
        ts = np.asarray(timestamps).astype("datetime64[h]")
        return (ts - EPOCH0).astype(np.int64)

    def generate(self, hours: np.ndarray, device="cpu", dtype=torch.float32) -> torch.Tensor:
        """Standardised fields at the given absolute hours: (len, C, H_loc, W_loc)."""
        lat_sl, lon_sl = self.metadata["sp_slices"]
        dev = torch.device(device)
        colat = torch.from_numpy(np.deg2rad(90.0 - self.latitudes[lat_sl])).to(dev)
        lon = torch.from_numpy(np.deg2rad(self.longitudes[lon_sl])).to(dev)
        lat_idx = torch.arange(lat_sl.start, lat_sl.stop, device=dev, dtype=torch.int64)
        lon_idx = torch.arange(lon_sl.start, lon_sl.stop, device=dev, dtype=torch.int64)
        pix = (lat_idx[:, None] * self.nlon + lon_idx[None, :])  # global pixel id
        m, n, p, a = (t.to(dev) for t in (self.m, self.n, self.p, self.a))
        v, scale = self.v.to(dev), self.scale.to(dev)
        C = m.shape[0]
        out = torch.empty(len(hours), C, colat.numel(), lon.numel(), dtype=dtype, device=dev)
        for i, tau in enumerate(np.asarray(hours, dtype=np.int64)):
            shift = 2 * math.pi * v * float(tau) / (self.nlon * self.dt_scale)  # (C,)
            # separable form: sin(m(lon - s) + n colat + p) = sin(mL) cos(nT + p) + cos(mL) sin(nT + p)
            ml = m[:, :, None] * (lon[None, None, :] - shift[:, None, None])  # C, K, W
            nt = n[:, :, None] * colat[None, None, :] + p[:, :, None]  # C, K, H
            A = torch.cat([torch.cos(nt), torch.sin(nt)], dim=1) * torch.cat([a, a], dim=1)[:, :, None]
            B = torch.cat([torch.sin(ml), torch.cos(ml)], dim=1)
            f = torch.einsum("ckh,ckw->chw", A, B) / scale[:, None, None]
            key = ((int(tau) * 1000003 + self.data_seed * 7919) & _MASK32)
            ck = (torch.arange(C, device=dev, dtype=torch.int64)[:, None, None] * 2654435761) & _MASK32
            noise = _normal((_hash32(pix[None] + ck) ^ key) & _MASK32)
            f = f + self.noise / scale[:, None, None] * noise
            out[i] = f.to(dtype)
        return out

    def get_samples(self, timestamps, device="cpu") -> torch.Tensor:
        return self.generate(self.hours_since_1900(timestamps), device=device)

    def window_hours(self, global_idx: int) -> np.ndarray:
        steps = self.temporal_context_window + self.num_rollout_steps
        ts = self.all_times[global_idx + np.arange(steps) * self.dt_scale]
        return self.hours_since_1900(ts)

    def unnormalize_era5(self, img):
        return img * self.stds + self.means

    # ------------------------------------------------------------------ state
    def set_dataset_state(self, checkpoint):
        self.resume_skip_batches = int(checkpoint["n_mbs_in_epoch"])
        self.ckpt_epoch = int(checkpoint["epoch"])

    def epoch_indices(self, epoch_idx: int) -> np.ndarray:
        """This dp shard's sample order for loader epoch ``epoch_idx``."""
        if self.shuffle:
            rng = np.random.default_rng(seed=self.seed + self.ckpt_epoch + epoch_idx)
            perm = rng.permutation(self.n_samples_total)
        else:
            perm = np.arange(self.n_samples_total)
        start = self.n_samples_shard * self.shard_id
        return perm[start:start + self.n_samples_shard]

    def __len__(self):
        return self.n_samples_shard


class SyntheticLoader:
    """Iterates micro-batches ``(mbs, T + nrs, C, H_loc, W_loc)`` of one dataset.

    ``device='cuda'`` generates on the GPU (no host traffic); ``pin_host=True`` generates
    on the GPU once per sample and serves it from pinned host memory, so each step pays a
    real host-to-device copy (used for end-to-end timing).
    """

    def __init__(self, dataset: SyntheticERA5, micro_batch_size: int = 1, device="cpu",
                 mode: str = "train"):
        self.dataset = dataset
        self.mbs = micro_batch_size
        self.device = torch.device(device)
        self.mode = mode
        self._epoch_idx = 0

    def __len__(self):
        return self.dataset.num_steps_per_epoch

    def __iter__(self) -> Iterator[torch.Tensor]:
        ds = self.dataset
        epoch_idx = self._epoch_idx
        self._epoch_idx += 1
        if ds.resume_skip_batches > 0:
            ds.iterations_to_skip = ds.resume_skip_batches
            ds.resume_skip_batches = 0
        else:
            ds.iterations_to_skip = 0
        order = ds.epoch_indices(epoch_idx)
        skip = ds.iterations_to_skip
        for it in range(ds.num_steps_per_epoch - skip):
            idx = order[(it + skip) * self.mbs:(it + skip + 1) * self.mbs]
            batch = torch.stack([ds.generate(ds.window_hours(int(k)), device=self.device)
                                 for k in idx])
            if ds.return_timestamp:
                yield batch, torch.stack([torch.from_numpy(ds.window_hours(int(k))) for k in idx])
            else:
                yield batch
