"""Dynamic fp16 loss scaling whose unscale and inf check ride on the fused optimizer step.

``torch.amp.GradScaler.unscale_`` walks every gradient once more (an inf/nan check and a multiply per
tensor) before clipping, and its ``step`` reads the result back to the host.  With the flat gradient
buffer and the fused AdamW kernel neither pass is needed: the gradient norm that clipping computes
anyway is the norm of the scaled gradients, so

* the true norm is that norm divided by the scale, and the clip coefficient divided by the scale is
  the single factor the kernel applies to every gradient (unscale and clip in one multiply);
* a non-finite norm means some gradient is inf or nan: the kernel's skip flag (device memory) drops
  the step, and the scale update below reads the same flag.

The scale and its growth counter stay on the device (no host synchronisation per step).  The update
rule and the ``state_dict`` keys are those of ``torch.amp.GradScaler`` (checkpoints keep the
reference's ``grad_scaler_state_dict`` entry): on an inf / nan step the scale is multiplied by
``backoff_factor`` and the counter reset; after ``growth_interval`` finite steps in a row it is
multiplied by ``growth_factor``.
"""

from __future__ import annotations

import torch


class DeviceLossScaler:
    def __init__(self, device, enabled: bool = True, init_scale: float = 2.0 ** 16, growth_factor: float = 2.0,
                 backoff_factor: float = 0.5, growth_interval: int = 2000):
        self._enabled = bool(enabled)
        self.growth_factor, self.backoff_factor = float(growth_factor), float(backoff_factor)
        self.growth_interval = int(growth_interval)
        self._scale = torch.full((1,), float(init_scale), dtype=torch.float32, device=device)
        self._tracker = torch.zeros(1, dtype=torch.int32, device=device)

    def is_enabled(self) -> bool:
        return self._enabled

    def scale(self, loss: torch.Tensor) -> torch.Tensor:
        # the fp32 scale promotes a 16-bit loss to fp32 (2**16 itself overflows fp16), as GradScaler does
        return loss * self._scale if self._enabled else loss

    def inv_scale(self) -> torch.Tensor:
        """1 / scale as a device tensor [1]."""
        return 1.0 / self._scale

    def update(self, found_inf: torch.Tensor) -> None:
        """``found_inf``: device tensor [1], nonzero when this step's gradients were not finite."""
        if not self._enabled:
            return
        bad = found_inf.reshape(1) != 0
        grown = self._tracker + 1
        grow = (~bad) & (grown >= self.growth_interval)
        self._scale.copy_(torch.where(bad, self._scale * self.backoff_factor,
                                      torch.where(grow, self._scale * self.growth_factor, self._scale)))
        self._tracker.copy_(torch.where(bad | grow, torch.zeros_like(grown), grown))

    # GradScaler's checkpoint layout
    def state_dict(self):
        if not self._enabled:
            return {}
        return {"scale": float(self._scale.item()), "growth_factor": self.growth_factor,
                "backoff_factor": self.backoff_factor, "growth_interval": self.growth_interval,
                "_growth_tracker": int(self._tracker.item())}

    def load_state_dict(self, state):
        if not self._enabled or not state:
            return
        self._scale.fill_(float(state["scale"]))
        self.growth_factor = float(state["growth_factor"])
        self.backoff_factor = float(state["backoff_factor"])
        self.growth_interval = int(state["growth_interval"])
        self._tracker.fill_(int(state["_growth_tracker"]))
