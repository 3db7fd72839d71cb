"""Autoregressive inference and scoring.

Follows ``utils/inferencer.py`` of the reference: the trained model's ``model``/``train``
config is loaded from ``inference.checkpoint_hyperparams`` with one rollout step
(``:74-102``); initial conditions every 12 h in ``[start_date, end_date]`` are sharded
round-robin over dp (``:157-166``); each IC is rolled out to ``time_horizon_in_hours`` in
model steps, each prediction un-normalised and scored with the latitude-weighted RMSE per
channel, power spectra are taken at ``spectra_times_in_hours`` from the sp-gathered
field (``:337-464``); at the end unstable ICs (channel-0 RMSE > 10) are dropped, sums are
all-reduced over dp and averaged, and ``rmse_{ch}.npy`` / ``spectra_{ch}_{lt}h.npy`` are
written (``:466-560``).

``inference.run_benchmark`` (``graphcast`` / ``hres``) scores a WeatherBench2 forecast in place of
the model (``inference/benchmarks.py``); ``inference.random_init`` runs without a checkpoint
(random-init weights, for benchmarks of the rollout itself).

Additions: a latitude-weighted anomaly correlation (ACC) per channel and lead, the choice
of compute precision (``inference.precision``: ``fp32`` as in the reference, computed with
the plain-PyTorch operators on the GPU, or ``bf16`` / ``fp16`` for the fused kernels) and
device-timed milliseconds per rollout step.
"""

from __future__ import annotations

import logging
import os
import time

import numpy as np
import torch
import torch.distributed as dist

from .. import config as C
from .. import ops
from ..data import get_dataset, get_preprocessor
from ..losses import anomaly_correlation, get_metric
from ..models.swin import get_model, strip_module_prefix
from ..parallel import comm
from ..parallel.mappings import allgather_forward_split_backward
from ..training.trainer import experiment_dir
from ..utils.checkpoint_io import verified_load
from ..utils.sht import DistributedRealSHT, power_spectrum_distributed
from . import benchmarks


class Inferencer:
    def __init__(self, cfg, bench_source=None):
        """``bench_source``: a :class:`~.benchmarks.ForecastSource` to score instead of the one
        ``inference.run_benchmark`` names (for stores already opened, or other providers)."""
        self.cfg = cfg
        self.bench_source = bench_source
        self.exp_dir = experiment_dir(cfg)
        comm.init(cfg, timeout_s=float(os.environ.get("NSW_PG_TIMEOUT_S", 600)))
        self.world_size = comm.get_world_size()
        self.local_rank = comm.get_local_rank()
        self.world_rank = comm.get_world_rank()
        if torch.cuda.is_available():
            torch.cuda.set_device(self.local_rank)
            self.device = torch.device("cuda", self.local_rank)
        else:
            self.device = torch.device("cpu")
        self.log_to_screen = bool(cfg.logging.log_to_screen) and self.world_rank == 0
        self.log_to_wandb = False
        prec = str(cfg.inference.get("precision", "fp32"))
        self.dtype = {"fp32": None, "bf16": torch.bfloat16, "fp16": torch.float16}[prec]

    def init_exp_dir(self, exp_dir):
        self.checkpoint_file = self.cfg.inference.checkpoint
        hp = self.cfg.inference.checkpoint_hyperparams
        if hp and os.path.exists(hp):
            trained = C.load(hp)
            self.cfg.model = trained.model
            self.cfg.train = trained.train
            self.cfg.train.num_rollout_steps = 1
            if self.log_to_screen:
                logging.info(f"Loaded trained model's config from {hp}")
        if self.world_rank == 0:
            random_ok = bool(self.cfg.inference.get("random_init", False))
            if not os.path.isfile(self.checkpoint_file) and not self.cfg.inference.run_benchmark and not random_ok:
                raise FileNotFoundError(f"Checkpoint file not found at {self.checkpoint_file}")
            os.makedirs(exp_dir, exist_ok=True)

    def launch(self):
        self.init_exp_dir(self.exp_dir)
        self.build()
        self.inference()
        return self.compute_final_metrics()

    def build(self):
        cfg = self.cfg
        if self.world_rank == 0:
            C.save(cfg, os.path.join(self.exp_dir, "hyperparameters.yaml"))
        self.test_dataset = get_dataset(cfg, "test")
        md = self.test_dataset.metadata
        self.metadata = md
        self.n_channels = md["n_channels"]
        self.n_lat = len(md["global_latitudes"])
        self.n_lon = len(md["global_longitudes"])
        self.context_window = md["temporal_context_window"]
        self.dt_hours = int(md["dt_hours"] * md["dt_scale"] / np.timedelta64(1, "h"))
        self.lead_times = list(range(self.dt_hours, int(cfg.inference.time_horizon_in_hours) + 1,
                                     self.dt_hours))
        start = np.datetime64(cfg.inference.start_date)
        end = np.datetime64(cfg.inference.end_date)
        ics = np.arange(start, end + np.timedelta64(12, "h"), np.timedelta64(12, "h"))
        self.total_ic_count = len(ics)
        self.ics = ics[comm.get_rank("dp")::comm.get_size("dp")]
        self.set_log_channels()
        self.ic_count = 0
        self.weighted_rmse = get_metric("weighted_rmse", md, temporal_average=False).to(self.device)
        self.area_w = md["area_weights"].to(self.device)
        self.mean = torch.as_tensor(self.test_dataset.means).to(self.device)
        self.std = torch.as_tensor(self.test_dataset.stds).to(self.device)
        nl = len(self.lead_times)
        self.rmse = torch.zeros(len(self.ics), self.n_channels, nl, device=self.device)
        self.acc = torch.zeros(len(self.ics), self.n_channels, nl, device=self.device)
        self.spectra = {lt: torch.zeros(len(self.ics), 2, self.n_channels, self.n_lat, device=self.device)
                        for lt in self.spectra_times_in_hours}
        # spectra from the distributed SHT: no rank gathers the globe
        self.sht = (DistributedRealSHT(self.n_lat, self.n_lon, md["sp_shapes"][0], md["sp_shapes"][1])
                    if self.spectra_times_in_hours else None)
        self.step_ms = []
        self.run_benchmark = cfg.inference.get("run_benchmark", None)
        if self.run_benchmark:
            # a third-party forecast is scored in place of the model (reference
            # utils/inferencer.py:201-233): no model, no checkpoint
            if self.bench_source is None:
                self.bench_source = benchmarks.make_source(cfg.inference)
            self.model = None
            return
        self.model = get_model(cfg, domain_metadata=md).to(self.device)
        comm.all_model_groups_exist(self.model)
        self.preprocessor = get_preprocessor(cfg, self.test_dataset).to(self.device)
        if self.checkpoint_file and os.path.isfile(self.checkpoint_file):
            self.restore_checkpoint(self.checkpoint_file)
        self.model.eval()

    def set_log_channels(self):
        inf = self.cfg.inference
        chans = list(inf.log_sfc) + [f"{v}{lev}" for v in inf.log_var for lev in inf.log_levels]
        self.log_channels = [c for c in chans if c in self.metadata["channels"]]
        self.spectra_times_in_hours = list(inf.spectra_times_in_hours)

    def all_gather_helper(self, x):
        with torch.no_grad():
            x = allgather_forward_split_backward(x, -1, self.metadata["sp_shapes"][1], "sp2")
            return allgather_forward_split_backward(x, -2, self.metadata["sp_shapes"][0], "sp1")

    def _forward(self, inputs):
        if self.device.type != "cuda":
            return self.model(inputs)
        if self.dtype is not None:
            with torch.autocast("cuda", dtype=self.dtype):
                return self.model(inputs).float()
        # fp32: the fused kernels compute in 16 bits, so fp32 rollouts use the plain-PyTorch
        # operators (fp32 arithmetic, as the reference runs inference)
        with ops.reference_ops():
            return self.model(inputs)

    def inference(self):
        timed = self.device.type == "cuda"
        with torch.inference_mode():
            for ic in self.ics:
                past = self.context_window - 1
                ts = ic - np.timedelta64(past * self.dt_hours, "h") + \
                    np.timedelta64(self.dt_hours, "h") * np.arange(self.context_window)
                if self.run_benchmark:
                    lat_sl, lon_sl = self.metadata["sp_slices"]
                    fc, _ = benchmarks.assemble(self.bench_source, ic, self.lead_times, self.metadata["channels"],
                                                lat_sl, lon_sl, self.n_lat)
                    fc = fc.to(self.device)
                else:
                    window = self.test_dataset.get_samples(ts, device=self.device).unsqueeze(0).to(self.device)
                for i, lead in enumerate(self.lead_times):
                    tgt = self.test_dataset.get_samples([ic + np.timedelta64(lead, "h")], device=self.device)
                    tgt = tgt.unsqueeze(0).to(self.device)
                    if self.run_benchmark:  # physical units already; normalised for the ACC
                        pred = fc[i].unsqueeze(0).unsqueeze(0)
                        gen = (pred - self.mean) / self.std
                    else:
                        inputs = self.preprocessor(window, device=self.device, mode="inference")
                        if timed:
                            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            e0.record()
                        gen = self._forward(inputs)
                        if timed:
                            e1.record()
                            self.step_ms.append((e0, e1))
                        pred = gen * self.std + self.mean
                    targ = tgt * self.std + self.mean
                    self.rmse[self.ic_count, :, i] = self.weighted_rmse(pred, targ)[0]
                    self.acc[self.ic_count, :, i] = anomaly_correlation(gen, tgt, self.area_w)[0, 0]
                    if lead in self.spectra_times_in_hours:
                        self.spectra[lead][self.ic_count, 0] = power_spectrum_distributed(pred, self.sht)[0].float()
                        self.spectra[lead][self.ic_count, 1] = power_spectrum_distributed(targ, self.sht)[0].float()
                    if not self.run_benchmark:
                        window = torch.roll(window, shifts=-1, dims=1)
                        window[:, -1].copy_(gen[:, 0])
                if self.device.type == "cuda":
                    # a kernel whose bounded wait ran out leaves its outputs incomplete: stop
                    # before this initial condition's scores are counted
                    ops._ext.check_device_errors()
                self.ic_count += 1

    def compute_final_metrics(self):
        if self.ic_count <= 0:
            raise AssertionError("no initial conditions processed")
        unstable = 0
        # the reference drops ICs whose channel-0 RMSE exceeds 10 at any lead
        limit = float(self.cfg.inference.get("unstable_rmse_threshold", 10.0))
        for ic in range(self.ic_count):
            if (self.rmse[ic, 0] > limit).any():
                unstable += 1
                self.rmse[ic] = 0
                self.acc[ic] = 0
                for lt in self.spectra:
                    self.spectra[lt][ic] = 0
        n_ok = self.ic_count - unstable
        rmse = self.rmse.sum(0)
        acc = self.acc.sum(0)
        spectra = {lt: s.sum(0) for lt, s in self.spectra.items()}
        counts = torch.tensor([n_ok, unstable], dtype=torch.float64, device=self.device)
        if dist.is_initialized() and comm.get_size("dp") > 1:
            g = comm.get_group("dp")
            dist.all_reduce(rmse, group=g)
            dist.all_reduce(acc, group=g)
            for lt in spectra:
                dist.all_reduce(spectra[lt], group=g)
            dist.all_reduce(counts, group=g)
        total_ok, total_unstable = int(counts[0].item()), int(counts[1].item())
        if total_ok != self.total_ic_count - total_unstable:
            raise AssertionError(f"IC count mismatch: {total_ok} != {self.total_ic_count} - {total_unstable}")
        denom = max(total_ok, 1)
        rmse /= denom
        acc /= denom
        for lt in spectra:
            spectra[lt] /= denom
        step_ms = None
        if self.step_ms:
            torch.cuda.synchronize()
            ms = [a.elapsed_time(b) for a, b in self.step_ms]
            step_ms = float(np.median(ms))
        if self.world_rank == 0:
            chans = self.metadata["channels"]
            for ch in self.log_channels:
                ci = chans.index(ch)
                np.save(os.path.join(self.exp_dir, f"rmse_{ch}.npy"), rmse[ci].cpu().numpy())
                np.save(os.path.join(self.exp_dir, f"acc_{ch}.npy"), acc[ci].cpu().numpy())
                for lt in self.spectra_times_in_hours:
                    np.save(os.path.join(self.exp_dir, f"spectra_{ch}_{lt}h.npy"),
                            spectra[lt][:, ci].cpu().numpy())
            if self.log_to_screen:
                logging.info(f"Number of unstable ICs (RMSE > {limit:g}): {total_unstable} out of "
                             f"{self.total_ic_count}")
        return {"rmse": rmse, "acc": acc, "spectra": spectra, "unstable": total_unstable,
                "ms_per_step": step_ms}

    def restore_checkpoint(self, path):
        ckpt = verified_load(path, map_location=self.device, weights_only=False)
        state = strip_module_prefix(ckpt["model_state"])
        self.model.load_state_dict(state)
