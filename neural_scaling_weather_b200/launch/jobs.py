"""Job tooling for training / inference runs on B200 nodes.

Covers the job layer of the reference (``batchsub.py:1-175``, ``submit_batch.sh``,
``submit_batch_inference.sh``, ``jobs/*``): pick a window size for a patch size, build the
``key=value`` overrides that :mod:`train` / :mod:`inference` accept, and produce the launch
command.  The reference targets Slurm clusters of 4-GPU A100 / GH200 nodes through
containers; here a node is 8 B200s and every node runs one ``torchrun`` with one process per
GPU (NCCL over NVLink inside the node).

``python -m neural_scaling_weather_b200.launch.jobs --mode train --nodes 2 --sp2 2`` prints
the overrides, the generated batch script and the ``sbatch`` command; ``--submit`` asks for
confirmation before running ``sbatch`` (nothing is submitted without it).
"""

from __future__ import annotations

import argparse
import math
import shlex
import subprocess
import sys
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

GPUS_PER_NODE = 8


def window_size_for(patch: int, sp1: int = 1, sp2: int = 1, img_size: Sequence[int] = (720, 1440),
                    base_patch: int = 4, base_window: Sequence[int] = (9, 18)) -> Tuple[int, int]:
    """Window (height, width) in patches for ``patch``, keeping the physical window area of
    ``base_window`` at ``base_patch`` roughly constant (reference ``batchsub.py:5-41``).

    The height is the largest divisor of the patch-grid height that is at most the scaled
    base height and whose double divides the grid width; the width is twice the height.  The
    window must tile both the global grid and every rank's local grid under ``sp1 x sp2``.
    """
    H, W = img_size
    target = max(1, math.ceil(base_window[0] * base_patch / patch))
    gh, gw = H // patch, W // patch
    best = 1
    for h in range(1, gh + 1):
        if gh % h == 0 and 2 * h <= gw and gw % (2 * h) == 0 and h <= target:
            best = max(best, h)
    wh, ww = best, 2 * best
    if gh % wh or gw % ww:
        raise ValueError(f"window {wh}x{ww} does not tile the {gh}x{gw} patch grid")
    if (H // sp1) // patch % wh or (W // sp2) // patch % ww:
        raise ValueError(f"window {wh}x{ww} does not tile the local grid of sp1={sp1} sp2={sp2}")
    return wh, ww


@dataclass
class JobSpec:
    """One run: model size, parallel layout and the launch shape."""

    run_name: str = "scaling"
    run_tag: str = "p4-e1024-d16-lr5em4"
    mode: str = "train"  # or "inference"
    nodes: int = 1
    batch_size: int = 16
    rollout_steps: int = 1
    embed_dim: int = 1024
    depth: int = 16
    head_dim: int = 64
    patch_size: int = 4
    lr: float = 5e-4
    sp1: int = 1
    sp2: int = 1
    tp: int = 1
    max_iterations: int = 200000
    micro_batch_size: int = 1
    # cooldown branch (reference: optimizer.scheduler=cooldown from a saved iteration)
    cooldown_from_iter: Optional[int] = None
    cooldown_to_iter: Optional[int] = None
    cooldown_fraction: float = 0.05
    exp_root: str = "/expts"
    extra: Dict[str, str] = field(default_factory=dict)

    @property
    def num_heads(self) -> int:
        return self.embed_dim // self.head_dim

    @property
    def tag(self) -> str:
        if self.cooldown_from_iter is not None and self.cooldown_to_iter is not None:
            return f"{self.run_tag}-cool{self.cooldown_to_iter}"
        return self.run_tag


def train_overrides(spec: JobSpec) -> Dict[str, str]:
    wh, ww = window_size_for(spec.patch_size, spec.sp1, spec.sp2)
    o = {
        "data.batch_size": str(spec.batch_size),
        "optimizer.lr": str(spec.lr),
        "parallelism.sp1": str(spec.sp1),
        "parallelism.sp2": str(spec.sp2),
        "parallelism.tp": str(spec.tp),
        "train.num_rollout_steps": str(spec.rollout_steps),
        "model.patch_size": str(spec.patch_size),
        "model.embed_dim": str(spec.embed_dim),
        "model.depth": str(spec.depth),
        "model.num_heads": str(spec.num_heads),
        "model.window_size": f"[{wh},{ww}]",
        "optimizer": "adamw",
        "train.clip_grad_norm": "1.0",
        "optimizer.max_iterations": str(spec.max_iterations),
        "parallelism.micro_batch_size": str(spec.micro_batch_size),
    }
    if spec.cooldown_from_iter is not None and spec.cooldown_to_iter is not None:
        o.update({
            "train.branch_from": f"{spec.exp_root}/{spec.run_name}/{spec.run_tag}/checkpoints/"
                                 f"ckpt_iter{spec.cooldown_from_iter}.tar",
            "optimizer.scheduler": "cooldown",
            "optimizer.cooldown_to_iter": str(spec.cooldown_to_iter),
            "optimizer.cooldown_from_iter": str(spec.cooldown_from_iter),
            "optimizer.cooldown_fraction": str(spec.cooldown_fraction),
        })
    return o


def inference_overrides(spec: JobSpec) -> Dict[str, str]:
    base = f"{spec.exp_root}/{spec.run_name}/{spec.run_tag}"
    return {
        "inference.checkpoint": f"{base}/checkpoints/ckpt_best.tar",
        "inference.checkpoint_hyperparams": f"{base}/hyperparameters.yaml",
        "parallelism.sp1": "1",
        "parallelism.sp2": "1",
    }


def build_overrides(spec: JobSpec) -> List[str]:
    o = train_overrides(spec) if spec.mode == "train" else inference_overrides(spec)
    o.update(spec.extra)
    return [f"run_name={spec.run_name}", f"run_tag={spec.tag}"] + [f"{k}={v}" for k, v in o.items()]


def torchrun_command(spec: JobSpec, entry: Optional[str] = None, master_addr: str = "127.0.0.1",
                     master_port: int = 29500) -> List[str]:
    """One node's launch: ``torchrun`` with one process per GPU (single node: 127.0.0.1)."""
    entry = entry or ("train.py" if spec.mode == "train" else "inference.py")
    return [sys.executable, "-m", "torch.distributed.run", f"--nnodes={spec.nodes}",
            f"--nproc-per-node={GPUS_PER_NODE}", f"--master-addr={master_addr}", f"--master-port={master_port}",
            entry] + build_overrides(spec)


def slurm_script(spec: JobSpec, time_limit: str = "06:00:00", partition: Optional[str] = None) -> str:
    """Batch script: one task per node, each running torchrun over the node's 8 GPUs; the first
    node of the allocation is the rendezvous host."""
    entry = "train.py" if spec.mode == "train" else "inference.py"
    overrides = " ".join(shlex.quote(a) for a in build_overrides(spec))
    lines = [
        "#!/bin/bash",
        f"#SBATCH --job-name={spec.run_name}",
        f"#SBATCH --nodes={spec.nodes}",
        "#SBATCH --ntasks-per-node=1",
        f"#SBATCH --gpus-per-node={GPUS_PER_NODE}",
        f"#SBATCH --time={time_limit}",
    ]
    if partition:
        lines.append(f"#SBATCH --partition={partition}")
    lines += [
        "set -euo pipefail",
        'MASTER_ADDR=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)',
        "export MASTER_ADDR MASTER_PORT=29500",
        "export NCCL_DEBUG=${NCCL_DEBUG:-WARN}",
        "srun --kill-on-bad-exit=1 python -m torch.distributed.run "
        f"--nnodes={spec.nodes} --nproc-per-node={GPUS_PER_NODE} "
        '--rdzv-backend=c10d --rdzv-endpoint="$MASTER_ADDR:$MASTER_PORT" '
        f"{entry} {overrides}",
    ]
    return "\n".join(lines) + "\n"


def sbatch_command(script_path: str) -> List[str]:
    return ["sbatch", script_path]


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--mode", choices=["train", "inference"], default="train")
    ap.add_argument("--run-name", default="scaling")
    ap.add_argument("--run-tag", default="p4-e1024-d16-lr5em4")
    ap.add_argument("--nodes", type=int, default=1)
    ap.add_argument("--embed-dim", type=int, default=1024)
    ap.add_argument("--depth", type=int, default=16)
    ap.add_argument("--patch-size", type=int, default=4)
    ap.add_argument("--lr", type=float, default=5e-4)
    ap.add_argument("--batch-size", type=int, default=16)
    ap.add_argument("--sp1", type=int, default=1)
    ap.add_argument("--sp2", type=int, default=1)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--cooldown-from", type=int, default=None)
    ap.add_argument("--cooldown-to", type=int, default=None)
    ap.add_argument("--script", default="submit_b200.sh", help="where to write the batch script")
    ap.add_argument("--submit", action="store_true", help="run sbatch after confirmation")
    a = ap.parse_args(argv)
    spec = JobSpec(run_name=a.run_name, run_tag=a.run_tag, mode=a.mode, nodes=a.nodes, embed_dim=a.embed_dim,
                   depth=a.depth, patch_size=a.patch_size, lr=a.lr, batch_size=a.batch_size, sp1=a.sp1, sp2=a.sp2,
                   tp=a.tp, cooldown_from_iter=a.cooldown_from, cooldown_to_iter=a.cooldown_to)
    print("overrides:", " ".join(build_overrides(spec)))
    with open(a.script, "w") as f:
        f.write(slurm_script(spec))
    cmd = sbatch_command(a.script)
    print("batch script:", a.script)
    print("command:", " ".join(cmd))
    if not a.submit:
        return 0
    try:
        resp = input("Submit with sbatch? [y/N]: ").strip().lower()
    except EOFError:
        resp = ""
    if resp not in ("y", "yes"):
        print("not submitted")
        return 0
    return subprocess.run(cmd).returncode


if __name__ == "__main__":
    sys.exit(main())
