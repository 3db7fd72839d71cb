"""FLOP-budget sweep over (embed, depth) configurations (reference ``scripts/sweep_flops.py``).

For every compute budget and model configuration, prints the per-step training FLOPs
(forward x 3 for forward + backward, global batch 16 at 720 x 1440), the parameter count and
the number of iterations the budget buys, keeping configurations that need between 1e3 and
1.2e5 iterations.  ``python -m neural_scaling_weather_b200.utils.sweep_flops``.
"""

from __future__ import annotations

import argparse
from typing import List, Sequence, Tuple

from .. import config as C
from .flops import FlopsCalculator

CONFIGS = [(192, 6), (256, 8), (384, 8), (512, 8), (512, 12), (640, 12), (768, 12), (768, 16), (1024, 12),
           (1024, 16), (1024, 24), (1536, 16)]
BUDGETS = [6e17, 1e18, 3e18, 6e18, 1e19, 3e19, 6e19]


def sweep(configs: Sequence[Tuple[int, int]] = CONFIGS, budgets: Sequence[float] = BUDGETS, patch: int = 4,
          global_batch: int = 16, h: int = 720, w: int = 1440, min_iters: float = 1e3,
          max_iters: float = 1.2e5) -> List[Tuple[int, int, int, float, float, float, float]]:
    cfg = C.compose("default")
    c_in = 71 + len(cfg.data.invariants)
    c_out = 71
    rows = []
    for budget in budgets:
        for embed, depth in configs:
            cfg.model.embed_dim = embed
            cfg.model.depth = depth
            cfg.model.patch_size = patch
            cfg.train.temporal_context_window = 1
            fl = FlopsCalculator(cfg, h=h, w=w, c_in=c_in, c_out=c_out)
            per_step = fl.flops() * 1e12 * 3 * global_batch
            params = fl.param_count()
            iters = budget / per_step
            if min_iters <= iters <= max_iters:
                rows.append((embed, depth, patch, per_step, params, iters, per_step * iters))
    return rows


def _table(rows, title_iters_fmt="{:10.0f}"):
    print(f"{'embed':>6} {'depth':>6} {'patch':>5} {'per_step_flop':>13} {'param(m)':>10} {'num_iters':>10} "
          f"{'used_flop':>12}")
    print("-" * 80)
    for e, d, p, ps, pm, it, used in rows:
        print(f"{e:6} {d:6} {p:5} {ps:13.2e} {pm:10.1f} {title_iters_fmt.format(it)} {used:12.2e}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--patch", type=int, default=4)
    ap.add_argument("--global-batch", type=int, default=16)
    a = ap.parse_args(argv)
    rows = sweep(patch=a.patch, global_batch=a.global_batch)
    _table(sorted(rows, key=lambda r: r[-1]))
    print()
    _table(sorted(rows, key=lambda r: r[4]), "{:10.1f}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
