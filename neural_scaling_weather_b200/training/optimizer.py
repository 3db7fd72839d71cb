"""Optimizers and learning-rate schedules.

Reference behaviour (``utils/optimizer_utils.py:10-72``): Adam / AdamW with
``betas = (0.9, 0.95)`` (AdamW takes ``optimizer.weight_decay``), SGD with momentum 0.9;
schedules ``cosine``, ``cosine_warmup``, ``cooldown`` (constant, then ``1 - sqrt(step /
cooldown_steps)``), ``fixed_warmup`` (linear warm-up, then 1) or none.

:class:`FusedAdamW` keeps parameters, gradients and both moments in flat fp32 buffers
(parameters and ``.grad`` become views into them), so the whole update is ONE kernel:
gradient-norm clipping scale (read from device memory, no host sync), the Adam/AdamW
update, and a bf16 shadow copy of the weights that the GEMM kernels read directly.  Its
``state_dict`` has exactly the layout of ``torch.optim.AdamW`` so checkpoints load either
way.
"""

from __future__ import annotations

import math
from typing import Iterable, List, Optional

import numpy as np
import torch
from torch.optim import lr_scheduler

from ..ops import _ext


class FlatParamSpace:
    """Packs a list of parameters into contiguous fp32 (and bf16 shadow) buffers."""

    def __init__(self, params: List[torch.nn.Parameter], shadow_dtype: Optional[torch.dtype] = None,
                 align: int = 64):
        self.params = params
        self.offsets: List[int] = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += (p.numel() + align - 1) // align * align
        self.numel = off
        dev = params[0].device
        self.data = torch.zeros(off, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(off, dtype=torch.float32, device=dev)
        for p, o in zip(params, self.offsets):
            self.data[o:o + p.numel()].copy_(p.detach().reshape(-1).float())
            p.data = self.data[o:o + p.numel()].view(p.shape)
            p.grad = self.grad[o:o + p.numel()].view(p.shape)
        self.shadow = None
        if shadow_dtype is not None:
            self.shadow = self.data.to(shadow_dtype)
        # segment table for the norm kernel: one class id per element range
        self.class_ids: Optional[torch.Tensor] = None

    def rebind(self, data: torch.Tensor, grad: torch.Tensor, shadow: Optional[torch.Tensor]):
        """Use these flat buffers (same size; contents already copied) and re-point every
        parameter's ``.data`` / ``.grad`` at them (e.g. buffers in symmetric memory)."""
        self.data, self.grad = data, grad
        if shadow is not None:
            self.shadow = shadow
        for p, o in zip(self.params, self.offsets):
            p.data = self.data[o:o + p.numel()].view(p.shape)
            p.grad = self.grad[o:o + p.numel()].view(p.shape)

    def view(self, buf: torch.Tensor, i: int) -> torch.Tensor:
        p = self.params[i]
        o = self.offsets[i]
        return buf[o:o + p.numel()].view(p.shape)

    def zero_grad(self):
        self.grad.zero_()
        for i, p in enumerate(self.params):
            if p.grad is None or p.grad.data_ptr() != self.view(self.grad, i).data_ptr():
                p.grad = self.view(self.grad, i)

    def refresh_shadow(self):
        if self.shadow is not None:
            self.shadow.copy_(self.data)


class FusedAdamW(torch.optim.Optimizer):
    """Adam/AdamW over flat buffers; one fused kernel per step on CUDA."""

    def __init__(self, params: Iterable[torch.nn.Parameter], lr=1e-3, betas=(0.9, 0.999),
                 eps=1e-8, weight_decay=0.0, decoupled_weight_decay=True,
                 shadow_dtype: Optional[torch.dtype] = None, space: Optional[FlatParamSpace] = None):
        params = [p for p in params if p.requires_grad]
        # checkpoint indices follow the caller's parameter order (as torch.optim does)
        self._given = list(params)
        if space is not None:
            params = list(space.params)
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay,
                        amsgrad=False, maximize=False, foreach=None, capturable=False,
                        differentiable=False, fused=True,
                        decoupled_weight_decay=decoupled_weight_decay)
        super().__init__(params, defaults)
        self.space = space if space is not None else FlatParamSpace(params, shadow_dtype=shadow_dtype)
        self.exp_avg = torch.zeros_like(self.space.data)
        self.exp_avg_sq = torch.zeros_like(self.space.data)
        self.step_count = 0
        self.grad_scale: Optional[torch.Tensor] = None  # device scalar multiplying grads
        self.found_inf: Optional[torch.Tensor] = None  # device flag (skip step if nonzero)
        self.dp = None  # FusedDPReducer when the data-parallel step is sharded (enable_dp_sharding)
        self._space_index = {id(p): j for j, p in enumerate(self.space.params)}
        self._publish_shadow()

    # --------------------------------------------------------------- helpers
    def _publish_shadow(self):
        if self.space.shadow is None:
            return
        from ..ops import weights as wcache

        for i, p in enumerate(self.space.params):
            wcache.register_shadow(p, self.space.view(self.space.shadow, i))

    def enable_dp_sharding(self, reducer):
        """Step only this rank's owned slices (``dp_adamw``: the update stores the new parameters into
        every rank's buffers) and keep the moments zero outside them."""
        self.dp = reducer
        dev = self.space.data.device
        lo = [a for a, _ in reducer.owned]
        hi = [b for _, b in reducer.owned]
        starts, acc = [], 0
        for a, b in reducer.owned:
            starts.append(acc)
            acc += (b - a) // 4
        self._rlo = torch.tensor(lo, dtype=torch.int64, device=dev)
        self._rhi = torch.tensor(hi, dtype=torch.int64, device=dev)
        self._rstart = torch.tensor(starts, dtype=torch.int64, device=dev)
        self._total4 = acc
        self._zero_unowned()
        self._publish_shadow()

    def _zero_unowned(self):
        keep = torch.zeros(self.space.numel, dtype=torch.bool, device=self.space.data.device)
        for a, b in self.dp.owned:
            keep[a:b] = True
        self.exp_avg.masked_fill_(~keep, 0.0)
        self.exp_avg_sq.masked_fill_(~keep, 0.0)

    def zero_grad(self, set_to_none: bool = False):
        self.space.zero_grad()

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        decoupled = g.get("decoupled_weight_decay", True)
        self.step_count += 1
        t = self.step_count
        bc1 = 1.0 - b1 ** t
        bc2 = 1.0 - b2 ** t
        sp = self.space
        if sp.data.is_cuda and self.dp is not None:
            ext = _ext.require()
            scale = self.grad_scale if self.grad_scale is not None else torch.ones(1, device=sp.data.device)
            skip = self.found_inf if self.found_inf is not None else torch.zeros(1, device=sp.data.device, dtype=torch.int32)
            shadow_code = 1 if (sp.shadow is not None and sp.shadow.dtype == torch.float16) else 0
            ext.dp_adamw(*self.dp.peers(), self._rlo, self._rhi, self._rstart, self._total4, self.exp_avg,
                         self.exp_avg_sq, shadow_code, scale, skip, float(lr), float(b1), float(b2), float(eps),
                         float(wd), float(bc1), float(bc2), bool(decoupled))
            self.dp.barrier_after_step()
        elif sp.data.is_cuda:
            ext = _ext.require()
            scale = self.grad_scale if self.grad_scale is not None else torch.ones(1, device=sp.data.device)
            skip = self.found_inf if self.found_inf is not None else torch.zeros(1, device=sp.data.device, dtype=torch.int32)
            ext.adamw_step(sp.data, sp.grad, self.exp_avg, self.exp_avg_sq,
                           sp.shadow if sp.shadow is not None else torch.empty(0, device=sp.data.device),
                           scale, skip, float(lr), float(b1), float(b2), float(eps), float(wd),
                           float(bc1), float(bc2), bool(decoupled))
        else:
            grad = sp.grad
            if self.grad_scale is not None:
                grad = grad * self.grad_scale
            if self.found_inf is not None and bool(self.found_inf.item()):
                return loss
            if wd != 0:
                if decoupled:
                    sp.data.mul_(1.0 - lr * wd)
                else:
                    grad = grad + wd * sp.data
            self.exp_avg.mul_(b1).add_(grad, alpha=1.0 - b1)
            self.exp_avg_sq.mul_(b2).addcmul_(grad, grad, value=1.0 - b2)
            denom = (self.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
            sp.data.addcdiv_(self.exp_avg, denom, value=-lr / bc1)
            sp.refresh_shadow()
        for p in sp.params:
            torch.autograd.graph.increment_version(p)
        return loss

    # --------------------------------------------------------------- state
    def state_dict(self):
        """torch.optim.AdamW layout.  With the data-parallel sharded step every rank holds the moments of
        its owned slices only (zero elsewhere): they are summed over dp first, so every rank must call
        this (the trainer builds the checkpoint dictionary on every rank)."""
        g = dict(self.param_groups[0])
        g["params"] = list(range(len(self._given)))
        state = {}
        exp_avg, exp_avg_sq = self.exp_avg, self.exp_avg_sq
        if self.dp is not None and self.step_count > 0:
            import torch.distributed as dist

            from ..parallel import comm

            exp_avg, exp_avg_sq = exp_avg.clone(), exp_avg_sq.clone()
            dist.all_reduce(exp_avg, group=comm.get_group("dp"))
            dist.all_reduce(exp_avg_sq, group=comm.get_group("dp"))
        if self.step_count > 0:
            for i, p in enumerate(self._given):
                j = self._space_index[id(p)]
                state[i] = {
                    "step": torch.tensor(float(self.step_count)),
                    "exp_avg": self.space.view(exp_avg, j).detach().clone(),
                    "exp_avg_sq": self.space.view(exp_avg_sq, j).detach().clone(),
                }
        return {"state": state, "param_groups": [g]}

    def load_state_dict(self, sd):
        groups = sd["param_groups"]
        for k, v in groups[0].items():
            if k != "params":
                self.param_groups[0][k] = v
        steps = []
        for i, st in sd["state"].items():
            j = self._space_index[id(self._given[int(i)])]
            self.space.view(self.exp_avg, j).copy_(st["exp_avg"])
            self.space.view(self.exp_avg_sq, j).copy_(st["exp_avg_sq"])
            steps.append(float(st["step"]))
        self.step_count = int(max(steps)) if steps else 0
        if self.dp is not None:
            self._zero_unowned()


def set_optimizer(cfg, net, shadow_dtype: Optional[torch.dtype] = None,
                  space: Optional[FlatParamSpace] = None):
    o = cfg.optimizer
    params = list(net.parameters())
    if o.optimizer == "adam":
        return FusedAdamW(params, lr=o.lr, betas=(0.9, 0.95), weight_decay=0.0,
                          decoupled_weight_decay=False, shadow_dtype=shadow_dtype, space=space)
    if o.optimizer == "adamw":
        return FusedAdamW(params, lr=o.lr, betas=(0.9, 0.95), weight_decay=o.weight_decay,
                          decoupled_weight_decay=True, shadow_dtype=shadow_dtype, space=space)
    if o.optimizer == "sgd":
        return torch.optim.SGD(params, lr=o.lr, momentum=0.9)
    raise ValueError(f"unknown optimizer {o.optimizer!r}")


def set_scheduler(cfg, opt):
    o = cfg.optimizer
    total = o.max_iterations
    if o.scheduler == "cosine":
        return lr_scheduler.CosineAnnealingLR(opt, T_max=total)
    if o.scheduler == "cosine_warmup":
        warm = o.warmup_steps
        return lr_scheduler.LambdaLR(
            opt, lambda x: min((x + 1) / warm, 0.5 * (1 + np.cos(np.pi * x / total))))
    if o.scheduler == "cooldown":
        if o.cooldown_fraction is not None:
            cooldown_steps = int(o.cooldown_to_iter * o.cooldown_fraction)
            constant_steps = (o.cooldown_to_iter - o.cooldown_from_iter) - cooldown_steps
            if constant_steps < 0:
                raise AssertionError("cooldown fraction too large; must cooldown from an earlier iteration")
        else:
            constant_steps = 0
            cooldown_steps = o.cooldown_to_iter - o.cooldown_from_iter

        def scale(x):
            if x <= constant_steps:
                return 1.0
            return 1 - math.sqrt((x - constant_steps) / cooldown_steps)

        return lr_scheduler.LambdaLR(opt, scale)
    if o.scheduler == "fixed_warmup":
        warm = o.warmup_steps
        return lr_scheduler.LambdaLR(opt, lambda x: (x + 1) / warm if x < warm else 1.0)
    return None
