"""Job tooling: window-size selection, override construction and Slurm/torchrun launch."""

from .jobs import (  # noqa: F401
    JobSpec,
    build_overrides,
    inference_overrides,
    sbatch_command,
    slurm_script,
    torchrun_command,
    train_overrides,
    window_size_for,
)
