"""Training driver.

Structure and semantics follow ``utils/trainer.py`` of the reference: communicator
set-up and gradient accumulation ``batch_size / (micro_batch_size * dp)`` (``:56-98``),
experiment directory and optional wandb (``:100-129``), the resume / branch / finetune
checkpoint strategy (``:131-182``), the build order (datasets, FLOP model, model,
shared-weight broadcast, pre-processor, data-parallel wrapper, optimizer, scheduler,
AMP + GradScaler, loss and metric, checkpoint restore, then loaders) (``:184-350``), the
hot loop with ``no_sync`` on accumulation micro-batches, clipping, the step, the
scheduler and the post-step gradient norm (``:545-657``), validation (``:659-717``), the
CSV ``logs.txt`` (``:719-734``) and the ``ckpt_*.tar`` format and naming (``:736-851``).

B200-specific changes, none of which alter the math:

* the model is wrapped by :class:`DataParallel` (state-dict prefix ``module.`` as DDP's)
  whose reducer all-reduces fp32 gradient buckets that are views of the optimizer's
  flat buffer, overlapped with backward;
* the clip coefficient and the logged gradient norm are device tensors: no ``.item()``
  host sync inside the loop (the reference has two per step);
* the NaN check reads the previous micro-batch's loss from a pinned host copy made
  asynchronously, instead of synchronising on the current one; the device error word of
  the extension (set by a kernel whose bounded wait ran out) is copied with it, and a
  nonzero word stops training with :class:`~..ops._ext.DeviceError`; the word is also read
  synchronously before every validation/checkpoint and at the end of training, so no
  checkpoint is written from a step whose kernels gave up;
* checkpoints are written atomically (temporary file + rename) with a SHA-256 record that is
  checked on load (``utils/checkpoint_io.py``), and the throughput (samples/s) and model FLOP
  rate (TFLOP/s, whole job) are logged next to the reference's keys.
"""

from __future__ import annotations

import logging
import math
import os
import random
import time
from contextlib import nullcontext
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn

from .. import config as C
from ..data import device_prefetch, get_data_loader, get_dataset, get_preprocessor
from ..losses import get_loss, get_metric
from ..models.swin import get_model, strip_module_prefix
from ..parallel import comm
from ..parallel.grad_sync import GradReducer, order_params
from ..parallel.helpers import init_params_for_shared_weights
from ..utils.checkpoint_io import atomic_save, verified_load  # noqa: F401 (atomic_save re-exported)
from ..utils.flops import FlopsCalculator
from ..utils.profiler import init_profiler, profile_range
from .grad_norm import ShardedNorm
from .loss_scale import DeviceLossScaler
from .optimizer import FlatParamSpace, FusedAdamW, set_optimizer, set_scheduler

AMP_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16}


def set_seed(cfg, world_size):
    seed = np.random.randint(10000) if cfg.train.seed is None else int(cfg.train.seed)
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    return seed


def count_parameters(model) -> float:
    return sum(p.numel() for p in model.parameters() if p.requires_grad) / 1e6


class DataParallel(nn.Module):
    """Holds the model under ``.module`` and exposes the reducer's ``no_sync``."""

    def __init__(self, module: nn.Module, reducer: Optional[GradReducer] = None):
        super().__init__()
        self.module = module
        self.reducer = reducer

    def forward(self, *a, **k):
        return self.module(*a, **k)

    def no_sync(self):
        return self.reducer.no_sync() if self.reducer is not None else nullcontext()


def experiment_dir(cfg) -> str:
    run = cfg.get("hydra", {}).get("run", {}) if isinstance(cfg.get("hydra", None), dict) else {}
    d = run.get("dir") if run else None
    return d or os.path.join("/expts", str(cfg.run_name), str(cfg.run_tag))


class Trainer:
    def __init__(self, cfg):
        self.cfg = cfg
        self.exp_dir = experiment_dir(cfg)
        self.run_name, self.run_tag = cfg.run_name, cfg.run_tag
        self.auto_resume = not cfg.disable_auto_resume
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
        self.log_to_wandb = bool(cfg.logging.log_to_wandb) and self.world_rank == 0
        if self.log_to_wandb:
            try:
                import wandb  # noqa: F401
            except Exception:
                self.log_to_wandb = False
                if self.log_to_screen:
                    logging.info("wandb is not importable; wandb logging disabled")
        global_mbs = int(cfg.parallelism.micro_batch_size) * comm.get_size("dp")
        self.gradient_accum_steps = int(cfg.data.batch_size) // global_mbs
        if self.gradient_accum_steps <= 0:
            raise ValueError("gradient_accum_steps must be positive")
        if int(cfg.data.batch_size) % global_mbs != 0:
            raise ValueError(
                "cfg.data.batch_size must be divisible by micro_batch_size * data_parallel_size "
                f"({cfg.data.batch_size} % {global_mbs} != 0)")

    # ------------------------------------------------------------------ setup
    def init_exp_dir(self, exp_dir):
        if self.world_rank == 0:
            os.makedirs(os.path.join(exp_dir, "checkpoints"), exist_ok=True)
            os.makedirs(os.path.join(exp_dir, "wandb"), exist_ok=True)
        if dist.is_initialized():
            dist.barrier()

    def launch(self):
        self.init_exp_dir(self.exp_dir)
        if self.log_to_wandb:
            try:
                import wandb

                wandb.init(dir=os.path.join(self.exp_dir, "wandb"), name=f"{self.run_name}_{self.run_tag}",
                           config=C.to_container(self.cfg), group=self.run_name,
                           project=self.cfg.logging.project, entity=self.cfg.logging.entity,
                           resume=self.auto_resume)
            except Exception as e:  # offline box / no credentials
                logging.info(f"wandb.init failed ({type(e).__name__}); wandb logging disabled")
                self.log_to_wandb = False
        self.build_and_run()

    def setup_checkpoint_strategy(self):
        self.checkpoint_path = os.path.join(self.exp_dir, "checkpoints", "ckpt.tar")
        self.resuming = os.path.isfile(self.modify_checkpoint_path(self.checkpoint_path)) and self.auto_resume
        tc = self.cfg.train
        if self.resuming:
            prev = os.path.join(self.exp_dir, "hyperparameters.yaml")
            if os.path.isfile(prev):
                if C.to_container(C.load(prev)) != C.to_container(self.cfg):
                    raise AssertionError(
                        f"Resuming run_name={self.run_name}, run_tag={self.run_tag} failed: config "
                        "saved to hyperparameters.yaml does not match current config")
            logging.info(f"Resuming checkpoint {self.checkpoint_path}")
            self.restore_checkpoint(self.checkpoint_path, True, True, True)
        elif tc.branch_from is not None:
            logging.info(f"Branching from checkpoint {tc.branch_from}")
            self.restore_checkpoint(tc.branch_from, True, False, True)
            if self.iters != self.cfg.optimizer.cooldown_from_iter:
                raise AssertionError("must branch from an iteration where cooldown starts")
        elif tc.finetune_from is not None:
            logging.info(f"Finetuning from checkpoint {tc.finetune_from}")
            self.restore_checkpoint(tc.finetune_from, False, False, False)

    def build_and_run(self):
        self.build()
        self.train()

    def build(self):
        cfg = self.cfg
        self.profiler = init_profiler(cfg)
        if self.world_rank == 0:
            logging.info("------------------ Config ------------------")
            for line in C.to_yaml(cfg).split("\n"):
                logging.info(line)
        set_seed(cfg, self.world_size)
        self.train_dataset = get_dataset(cfg, "train")
        self.val_dataset = get_dataset(cfg, "valid")
        self.metadata = self.train_dataset.metadata
        n_inv = len(cfg.data.invariants) if cfg.data.invariants else 0
        self.flops_calculator = FlopsCalculator(
            cfg, h=len(self.metadata["global_latitudes"]), w=len(self.metadata["global_longitudes"]),
            c_in=len(self.metadata["channels"]) + n_inv, c_out=len(self.metadata["channels"]))

        model = get_model(cfg, domain_metadata=self.metadata).to(self.device)
        comm.all_model_groups_exist(model)
        if comm.get_size("tp-sp1-sp2") > 1:
            init_params_for_shared_weights(model)
        self.preprocessor = get_preprocessor(cfg, self.train_dataset).to(self.device)

        try:
            self.amp_dtype = AMP_DTYPES[cfg.train.amp_dtype]
        except KeyError as exc:
            raise ValueError(f"Unsupported AMP dtype {cfg.train.amp_dtype!r}; expected one of "
                             f"{tuple(AMP_DTYPES)}") from exc
        self.amp_enabled = bool(cfg.train.enable_amp) and self.device.type == "cuda"
        shadow = self.amp_dtype if self.amp_enabled else None

        params = [p for p in model.parameters() if p.requires_grad]
        self.space = FlatParamSpace(order_params(params), shadow_dtype=shadow)
        reducer = None
        if dist.is_initialized():
            from ..parallel import dp_fused

            fp16_scaler = self.amp_enabled and self.amp_dtype == torch.float16
            ok, why = dp_fused.available(self.space, cfg.optimizer.optimizer, fp16_scaler)
            if ok:
                reducer = dp_fused.FusedDPReducer(self.space)
            else:
                reducer = GradReducer(self.space)
                if self.log_to_screen and comm.get_size("dp") > 1:
                    logging.info(f"data-parallel reduction over NCCL ({why})")
        self.model = DataParallel(model, reducer)
        self.optimizer = set_optimizer(cfg, model, shadow_dtype=shadow, space=self.space)
        owned = None
        if getattr(reducer, "sharded", False) and isinstance(self.optimizer, FusedAdamW):
            self.optimizer.enable_dp_sharding(reducer)
            owned = reducer.owned
        self.scheduler = set_scheduler(cfg, self.optimizer)
        self.norms = ShardedNorm(self.space, owned=owned)
        self.use_cuda_graphs = bool(cfg.train.get("cuda_graphs", False))
        self._graph, self._graph_calls, self._static, self._static_loss = None, 0, None, None
        self._graph_pool, self._graph_stream = None, None
        fp16 = self.amp_enabled and self.amp_dtype == torch.float16
        if isinstance(self.optimizer, FusedAdamW):
            # the unscale and inf check ride on the fused step (training/loss_scale.py)
            self.gscaler = DeviceLossScaler(self.device, enabled=fp16)
        else:
            self.gscaler = torch.amp.GradScaler("cuda", enabled=fp16)
        self.loss_func = get_loss(cfg, self.metadata).to(self.device)
        self.weighted_rmse = get_metric("weighted_rmse", self.metadata).to(self.device)

        self.iters_per_epoch = self.train_dataset.n_samples_total // int(cfg.data.batch_size)
        self.max_iters = (cfg.optimizer.cooldown_to_iter if cfg.optimizer.scheduler == "cooldown"
                          else cfg.optimizer.max_iterations)
        self.iters = 0
        self.n_mbs = 0
        self.n_mbs_in_epoch = 0
        self.start_epoch = 0
        self.end_epoch = math.ceil(self.max_iters / max(self.iters_per_epoch, 1))
        self.setup_checkpoint_strategy()

        self.train_data_loader, self.train_sampler = get_data_loader(cfg, self.train_dataset, "train")
        self.val_data_loader, self.val_sampler = get_data_loader(cfg, self.val_dataset, "valid")
        if self.world_rank == 0:
            C.save(cfg, os.path.join(self.exp_dir, "hyperparameters.yaml"))

        self.epoch = self.start_epoch
        self.logs = {}
        self.train_loss = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.train_time = 0.0
        self.flops_consumed = 0.0
        self.iters_last_log = self.iters
        self.n_mbs_last_log = self.n_mbs
        self.log_every = (cfg.train.log_every if cfg.train.log_every is not None
                          else max(1, int(cfg.train.log_frequency * self.max_iters)))
        self._loss_host = torch.zeros(1, dtype=torch.float32, pin_memory=self.device.type == "cuda")
        self._loss_evt = None
        self._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=self.device.type == "cuda")
        self._err_word = None
        if self.device.type == "cuda":
            from ..ops import _ext

            self._err_word = _ext.require().error_word()
        if self.log_to_screen:
            logging.info(f"number of model parameters (M): {count_parameters(self.model)}")
            logging.info(f"number of training steps per epoch: {self.iters_per_epoch}")
            logging.info(f"max iterations: {self.max_iters}")
            logging.info(f"number of training samples: {self.train_dataset.n_samples_total}")
        self.sync_devices()

    # ------------------------------------------------------------------ loop
    def train(self):
        if self.log_to_screen:
            logging.info("starting training loop...")
        self.best_loss = getattr(self, "best_loss", np.inf)
        self.best_iter = getattr(self, "best_iter", 0)
        self.logs["best_iter"] = self.best_iter
        self.train_time = time.time()
        self.train_loss.zero_()
        self.grad.zero_()
        app = time.time()
        for epoch in range(self.start_epoch, self.end_epoch):
            self.epoch = epoch
            self.profiler.set_epoch(epoch)
            if self.train_sampler is not None and hasattr(self.train_sampler, "set_epoch"):
                self.train_sampler.set_epoch(epoch)
            t0 = time.time()
            nsteps = self.train_one_epoch()
            if self.log_to_screen:
                logging.info(f"Epoch {epoch} completed; Training Steps: {nsteps}; Time: {time.time() - t0:.2f}s")
            if self.iters >= self.max_iters or self._stop:
                break
        if self.log_to_wandb:
            import wandb

            wandb.finish()
        if self.log_to_screen:
            logging.info(f"Application time: {time.time() - app:.2f}s")
        self.sync_devices()
        self.check_device_errors()

    _stop = False

    def _nan_seen(self) -> bool:
        """NaN check on the previous micro-batch's accumulated loss (no sync on this one).
        Raises :class:`DeviceError` if the device error word copied with that loss is set."""
        if self.device.type != "cuda":
            return bool(torch.isnan(self.train_loss).item())
        if self._loss_evt is not None and self._loss_evt.query():
            if int(self._err_host[0]) != 0:
                self._device_error(int(self._err_host[0]))
            return bool(math.isnan(float(self._loss_host[0])))
        return False

    def _snapshot_loss(self):
        if self.device.type == "cuda":
            self._loss_host.copy_(self.train_loss, non_blocking=True)
            self._err_host.copy_(self._err_word, non_blocking=True)
            self._loss_evt = torch.cuda.Event()
            self._loss_evt.record()

    def check_device_errors(self):
        """Synchronous read (and clear) of the device error word; raises if it is set."""
        if self.device.type == "cuda":
            from ..ops import _ext

            code = _ext.require().read_error_flag(True)
            if code != 0:
                self._device_error(code)

    def _device_error(self, code: int):
        from ..ops._ext import DeviceError

        self._stop = True
        logging.error(f"device error word {code} set by a kernel; stopping without a checkpoint")
        raise DeviceError(code)

    def optimizer_step(self):
        """Reduce, clip, step, schedule, log the post-step norm and zero the grads."""
        if self.model.reducer is not None:
            self.model.reducer.finish()
        opt = self.optimizer
        device_scale = isinstance(self.gscaler, DeviceLossScaler) and self.gscaler.is_enabled()
        if self.gscaler.is_enabled() and not device_scale:
            self.gscaler.unscale_(opt)
        clip = self.cfg.train.clip_grad_norm
        norm = self.norms.norm("grad")
        if device_scale:  # norm of the scaled gradients: non-finite <=> some gradient is inf / nan
            found_inf = (~torch.isfinite(norm)).to(torch.int32)
            inv = self.gscaler.inv_scale()
            norm = norm * inv
        coef = ShardedNorm.clip_coef(norm, float(clip)) if clip else torch.ones_like(norm)
        if isinstance(opt, FusedAdamW):
            if device_scale:  # unscale and clip in the kernel's one multiply; skip the step on inf / nan
                opt.grad_scale, opt.found_inf = coef * inv, found_inf
                opt.step()
                opt.found_inf = None
                self.gscaler.update(found_inf)
            else:
                opt.grad_scale = coef
                opt.step()
        else:
            for p in self.model.parameters():
                if p.grad is not None:
                    p.grad.mul_(coef)
            self.gscaler.step(opt)
            self.gscaler.update()
        self.iters += 1
        if self.scheduler is not None:
            self.scheduler.step()
        with profile_range("grad norm"):
            if device_scale:  # a skipped (inf / nan) step adds nothing to the logged norm
                self.grad += torch.where(found_inf != 0, torch.zeros_like(norm), norm * coef)
            else:
                self.grad += norm * coef
        opt.zero_grad(set_to_none=False)

    def _micro_batch(self, inputs, targets):
        """Forward, loss and backward of one micro-batch (gradients accumulate in place)."""
        with profile_range("forward pass"):
            with torch.autocast(self.device.type, dtype=self.amp_dtype, enabled=self.amp_enabled):
                gen = self.model(inputs)
                loss = self.loss_func(gen, targets)
            self.train_loss += loss.detach()
            loss = loss / self.gradient_accum_steps
        with profile_range("backward pass"):
            self.gscaler.scale(loss).backward()
        return loss

    def _graphable(self, is_optimizer_step: bool) -> bool:
        """Micro-batches that can replay a captured CUDA graph: CUDA, no fp16 loss scaling, and
        not the one whose backward launches the data-parallel gradient reduction."""
        if not self.use_cuda_graphs or self.device.type != "cuda" or self.gscaler.is_enabled():
            return False
        return self.model.reducer is None or not is_optimizer_step

    def _graph_step(self, inputs, targets):
        """Replay the captured micro-batch graph on this batch (capturing it on the third call;
        the first two run eagerly so every cache and workspace exists before capture)."""
        if self._graph is None:
            # warm-up and capture run on one side stream, so the autograd accumulation nodes the
            # captured backward uses live on the capture stream
            self._graph_calls += 1
            if self._graph_stream is None:
                self._graph_stream = torch.cuda.Stream(device=self.device)
            s = self._graph_stream
            s.wait_stream(torch.cuda.current_stream(self.device))
            if self._graph_calls <= 2:
                with torch.cuda.stream(s):
                    loss = self._micro_batch(inputs, targets).detach()
                torch.cuda.current_stream(self.device).wait_stream(s)
                return loss
            try:
                with torch.cuda.stream(s):
                    self._static = (inputs.clone(), targets.clone())
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=self._graph_pool, stream=s):
                    self._static_loss = self._micro_batch(*self._static).detach()
                torch.cuda.current_stream(self.device).wait_stream(s)
                self._graph = g
            except Exception as e:  # capture unsupported here: stay eager
                logging.warning(f"CUDA graph capture failed ({type(e).__name__}: {e}); running eagerly")
                self.use_cuda_graphs = False
                self._graph, self._static = None, None
                torch.cuda.synchronize()
                self.optimizer.zero_grad(set_to_none=False)
                self.train_loss.zero_()
                return self._micro_batch(inputs, targets)
        self._static[0].copy_(inputs, non_blocking=True)
        self._static[1].copy_(targets, non_blocking=True)
        self._graph.replay()
        return self._static_loss

    def train_step(self, batch, is_optimizer_step: bool):
        """One micro-batch forward/backward (and the optimizer step on the last one).  With
        ``train.cuda_graphs`` the micro-batch replays one captured CUDA graph (host launch
        overhead removed); derived weight copies are refreshed in place after each step."""
        graphed = self._graphable(is_optimizer_step)
        sync_ctx = self.model.no_sync() if (self.model.reducer is not None and not is_optimizer_step) else nullcontext()
        with profile_range(f"iter {self.iters}"):
            with sync_ctx:
                with profile_range("data preproc"):
                    inputs, targets = self.preprocessor(batch, device=self.device)
                loss = self._graph_step(inputs, targets) if graphed else self._micro_batch(inputs, targets).detach()
            with profile_range("optimizer"):
                if is_optimizer_step:
                    self.optimizer_step()
                    if self.use_cuda_graphs:
                        from ..ops import weights as wcache

                        wcache.refresh_derived()
        return loss

    def train_one_epoch(self):
        self.model.train()
        nsteps = 0
        n_batches = len(self.train_data_loader)
        ds = self.train_dataset
        if self.epoch == getattr(ds, "ckpt_epoch", -1):
            n_batches = max(0, n_batches - max(ds.resume_skip_batches, ds.iterations_to_skip))
        n_accum = n_batches - (n_batches % self.gradient_accum_steps)
        # host batches are copied to the device one batch ahead, on a side stream
        for batch_idx, batch in enumerate(device_prefetch(self.train_data_loader, self.device)):
            if self._nan_seen():
                logging.warning("NaN detected; stopping")
                self._stop = True
                break
            if self.iters >= self.max_iters:
                if self.iters % self.log_every != 0:
                    self.validate_and_checkpoint()
                break
            is_opt = (batch_idx + 1) % self.gradient_accum_steps == 0
            if batch_idx + 1 > n_accum:
                break
            nsteps += 1
            self.n_mbs += 1
            self.n_mbs_in_epoch += 1
            self.train_step(batch, is_opt)
            self._snapshot_loss()
            if is_opt:
                if self.iters % self.log_every == 0:
                    self.validate_and_checkpoint()
                    self.train_loss.zero_()
                    self.grad.zero_()
                    self.train_time = time.time()
                o = self.cfg.optimizer
                if o.scheduler == "cooldown":
                    cds = int(o.cooldown_to_iter * o.cooldown_fraction)
                    if self.iters == o.cooldown_to_iter - cds:
                        self.save_checkpoint(self.checkpoint_path.replace(".tar", "_base.tar"))
                if self.iters >= self.max_iters:
                    if self.iters % self.log_every != 0:
                        self.validate_and_checkpoint()
                    break
        self.n_mbs_in_epoch = 0
        return nsteps

    # ------------------------------------------------------------------ eval / logs
    def sync_devices(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()

    @torch.no_grad()
    def val_one_epoch(self):
        self.model.eval()
        t0 = time.time()
        nc = self.metadata["n_channels"]
        mult = torch.as_tensor(self.train_dataset.stds[0, :, 0, 0]).to(self.device)
        vloss = torch.zeros(1, dtype=torch.float32, device=self.device)
        vrmse = torch.zeros(nc, dtype=torch.float32, device=self.device)
        nsteps = 0
        limit = self.cfg.train.get("limit_validation", None)
        with torch.inference_mode():
            for batch in self.val_data_loader:
                nsteps += 1
                inputs, targets = self.preprocessor(batch, device=self.device)
                with torch.autocast(self.device.type, dtype=self.amp_dtype, enabled=self.amp_enabled):
                    gen = self.model(inputs)
                vloss += self.loss_func(gen, targets)
                vrmse += self.weighted_rmse(gen, targets)
                if limit is not None and nsteps >= int(limit):
                    break
        nsteps = max(nsteps, 1)
        vloss /= nsteps
        vrmse /= nsteps
        vrmse *= mult
        if dist.is_initialized() and comm.get_size("dp") > 1:
            dist.all_reduce(vloss, op=dist.ReduceOp.AVG, group=comm.get_group("dp"))
            dist.all_reduce(vrmse, op=dist.ReduceOp.AVG, group=comm.get_group("dp"))
        self.logs["val_loss"] = float(vloss.item())
        for var in self.cfg.data.track_channels:
            if var in self.val_dataset.era5_channels:
                idx = self.val_dataset.era5_channels.index(var)
                self.logs[f"val_rmse_{var}"] = float(vrmse[idx].item())
        self.sync_devices()
        return time.time() - t0, nsteps, []

    def validate_and_checkpoint(self):
        self.sync_devices()
        self.check_device_errors()
        self.logs["train_time"] = time.time() - self.train_time
        self.logs["val_time"], self.logs["val_nsteps"], _ = self.val_one_epoch()
        t0 = time.time()
        fwd = self.flops_calculator.flops()
        self.flops_consumed = fwd * 3 * int(self.cfg.train.num_rollout_steps) * self.n_mbs * comm.get_size("dp")
        self.logs["flops_consumed"] = self.flops_consumed
        self.logs["learning_rate"] = self.optimizer.param_groups[0]["lr"]
        self.logs["wt_norm"] = float(self.norms.norm("weights").item())
        is_best = self.logs["val_loss"] <= self.best_loss
        if is_best:
            self.best_loss, self.best_iter = self.logs["val_loss"], self.iters
        self.logs["best_val_loss"] = self.best_loss
        self.logs["best_iter"] = self.best_iter
        n_mbs = max(1, self.n_mbs - self.n_mbs_last_log)
        n_it = max(1, self.iters - self.iters_last_log)
        train_loss = self.train_loss / n_mbs
        grad = self.grad / n_it
        if dist.is_initialized() and comm.get_size("dp") > 1:
            dist.all_reduce(train_loss, op=dist.ReduceOp.AVG, group=comm.get_group("dp"))
            dist.all_reduce(grad, op=dist.ReduceOp.AVG, group=comm.get_group("dp"))
        self.logs["train_loss"] = float(train_loss.item())
        self.logs["grad"] = float(grad.item())
        samples = n_mbs * int(self.cfg.parallelism.micro_batch_size) * comm.get_size("dp")
        self.logs["samples_per_sec"] = samples / max(self.logs["train_time"], 1e-9)
        # model FLOP rate of the whole job over the interval (forward x 3 for the backward)
        interval_flops = fwd * 3 * int(self.cfg.train.num_rollout_steps) * n_mbs * comm.get_size("dp")
        self.logs["tflops_per_sec"] = interval_flops / max(self.logs["train_time"], 1e-9) / 1e12
        peak = float(self.cfg.train.get("peak_tflops_per_gpu", 2250.0)) * self.world_size
        self.logs["mfu"] = self.logs["tflops_per_sec"] / peak if peak > 0 else 0.0
        if self.log_to_wandb:
            import wandb

            wandb.log(self.logs, step=self.iters, commit=True)
        if self.world_rank == 0:
            self.write_logs()
        if self.cfg.train.save_checkpoint:
            with profile_range("save checkpoint"):
                self.save_checkpoint(self.checkpoint_path, is_best=is_best)
        if self.log_to_screen:
            logging.info(f"Iteration {self.iters}: train loss {self.logs['train_loss']:.6f}, "
                         f"val loss {self.logs['val_loss']:.6f}, grad {self.logs['grad']:.4f}, "
                         f"{self.logs['samples_per_sec']:.2f} samples/s, log time {time.time() - t0:.2f}s")
        self.sync_devices()
        self.iters_last_log = self.iters
        self.n_mbs_last_log = self.n_mbs
        self.model.train()

    def write_logs(self):
        path = os.path.join(self.exp_dir, "logs.txt")
        exists = os.path.exists(path)
        row = {"iter": self.iters}
        for k, v in self.logs.items():
            row[k] = v.item() if hasattr(v, "item") else v
        with open(path, "a") as f:
            if not exists:
                f.write(",".join(row.keys()) + "\n")
            f.write(",".join(str(row[k]) for k in row) + "\n")

    # ------------------------------------------------------------------ checkpoints
    def modify_checkpoint_path(self, path):
        if comm.get_size("tp") > 1:
            path = path.replace("ckpt", f"ckpt_tp{comm.get_rank('tp')}")
        if not getattr(self.cfg.model, "coord_pos_embed", False) and comm.get_size("sp1") * comm.get_size("sp2") > 1:
            path = path.replace("ckpt", f"ckpt_sp1{comm.get_rank('sp1')}_sp2{comm.get_rank('sp2')}")
        return path

    def _should_save(self) -> bool:
        """dp-rank 0 saves; every tp rank saves its own shard file when tp > 1, every sp
        rank when the positional embedding is sp-sharded, else only sp-rank 0."""
        if comm.get_rank("dp") != 0:
            return False
        pos_sharded = not getattr(self.cfg.model, "coord_pos_embed", False)
        if not pos_sharded and (comm.get_rank("sp1") != 0 or comm.get_rank("sp2") != 0):
            return False
        return True

    def checkpoint_dict(self):
        return {
            "iters": self.iters,
            "n_mbs": self.n_mbs,
            "n_mbs_in_epoch": self.n_mbs_in_epoch,
            "epoch": self.epoch,
            "model_state": self.model.state_dict(),
            "optimizer_state_dict": self.optimizer.state_dict(),
            "scheduler_state_dict": self.scheduler.state_dict() if self.scheduler is not None else None,
            "grad_scaler_state_dict": self.gscaler.state_dict(),
            "best_loss": self.best_loss,
            "best_iter": self.best_iter,
            "micro_batch_size": int(self.cfg.parallelism.micro_batch_size),
        }

    def save_checkpoint(self, checkpoint_path, is_best=False):
        path = self.modify_checkpoint_path(checkpoint_path)
        ckpt = self.checkpoint_dict()
        if self._should_save():
            logging.info(f"Rank {comm.get_world_rank()} saving checkpoint to {path}")
            atomic_save(ckpt, path)
            if is_best:
                atomic_save(ckpt, path.replace(".tar", "_best.tar"))
            atomic_save(ckpt, path.replace(".tar", f"_iter{self.iters}.tar"))

    def restore_checkpoint(self, checkpoint_path, restore_optimizer=True, restore_scheduler=True,
                           restore_dataset=False):
        path = self.modify_checkpoint_path(checkpoint_path)
        ckpt = verified_load(path, map_location=self.device, weights_only=False)
        state = ckpt["model_state"]
        try:
            self.model.load_state_dict(state)
        except RuntimeError:
            if any(k.startswith("module.") for k in state):
                self.model.module.load_state_dict(strip_module_prefix(state))
            else:
                self.model.module.load_state_dict(state)
        if restore_optimizer:
            self.iters = ckpt["iters"]
            self.n_mbs = ckpt["n_mbs"]
            self.n_mbs_in_epoch = ckpt["n_mbs_in_epoch"]
            self.start_epoch = ckpt["epoch"]
            self.optimizer.load_state_dict(ckpt["optimizer_state_dict"])
            self.gscaler.load_state_dict(ckpt["grad_scaler_state_dict"])
            self.best_loss = ckpt["best_loss"]
            self.best_iter = ckpt["best_iter"]
        if restore_scheduler and self.scheduler is not None and ckpt.get("scheduler_state_dict"):
            self.scheduler.load_state_dict(ckpt["scheduler_state_dict"])
        if restore_dataset:
            self.iters = ckpt["iters"]
            self.n_mbs = ckpt["n_mbs"]
            self.n_mbs_in_epoch = ckpt["n_mbs_in_epoch"]
            self.start_epoch = ckpt["epoch"]
            self.train_dataset.set_dataset_state({
                "n_mbs_in_epoch": self.n_mbs_in_epoch,
                "epoch": self.start_epoch,
                "micro_batch_size": int(ckpt.get("micro_batch_size", 1)),
            })
        self.space.refresh_shadow()
        if self.log_to_screen:
            logging.info(f"Restored checkpoint iteration = {self.iters}, epoch = {self.start_epoch}, "
                         f"micro-batches in epoch = {self.n_mbs_in_epoch}")
