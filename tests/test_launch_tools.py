"""Job tooling and FLOP sweep (CPU)."""

import pytest

from neural_scaling_weather_b200.launch import (
    JobSpec,
    build_overrides,
    slurm_script,
    torchrun_command,
    window_size_for,
)
from neural_scaling_weather_b200.models.layers import drop_path
from neural_scaling_weather_b200.utils.sweep_flops import sweep


def test_window_size_keeps_area_and_divides():
    assert window_size_for(4, 1, 1) == (9, 18)  # the reference's base window
    assert window_size_for(2, 1, 2) == (18, 36)
    assert window_size_for(8, 1, 1) == (5, 10)
    for p in (1, 2, 4, 8):
        wh, ww = window_size_for(p)
        assert (720 // p) % wh == 0 and (1440 // p) % ww == 0 and ww == 2 * wh


def test_window_size_rejects_untileable_local_grid():
    with pytest.raises(ValueError):
        window_size_for(4, 1, 7)  # 1440/7 is not a whole number of 18-wide windows


def test_overrides_and_commands():
    spec = JobSpec(nodes=2, sp2=2, cooldown_from_iter=42000, cooldown_to_iter=50000)
    o = build_overrides(spec)
    assert "model.window_size=[9,18]" in o and "parallelism.sp2=2" in o and "model.num_heads=16" in o
    assert "run_tag=p4-e1024-d16-lr5em4-cool50000" in o
    assert any(a.startswith("train.branch_from=") and a.endswith("ckpt_iter42000.tar") for a in o)
    cmd = torchrun_command(spec)
    assert "--nproc-per-node=8" in cmd and "--master-addr=127.0.0.1" in cmd and "train.py" in cmd
    script = slurm_script(spec)
    assert "#SBATCH --nodes=2" in script and "--rdzv-endpoint" in script and "train.py" in script
    inf = build_overrides(JobSpec(mode="inference"))
    assert any(a.startswith("inference.checkpoint=") for a in inf)


def test_sweep_rows_within_iteration_bounds():
    rows = sweep()
    assert rows
    for e, d, p, per_step, params, iters, used in rows:
        assert 1e3 <= iters <= 1.2e5
        assert abs(per_step * iters - used) < 1e-6 * used


def test_drop_path():
    import torch

    x = torch.ones(1000, 3)
    assert torch.equal(drop_path(x, 0.5, training=False), x)
    y = drop_path(x, 0.25, training=True)
    kept = (y[:, 0] != 0).float().mean().item()
    assert 0.65 < kept < 0.85 and torch.allclose(y[y != 0], torch.full_like(y[y != 0], 1 / 0.75))


def test_profiler_ranks_epoch_window_and_ranges(monkeypatch):
    """NVTX ranges only on the profiled ranks, and the CUDA-profiler window opens for
    profile_epoch and closes on the next epoch (calls recorded through stand-ins, no GPU)."""
    import torch

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.utils import profiler as P

    calls = []
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda.profiler, "start", lambda: calls.append("start"))
    monkeypatch.setattr(torch.cuda.profiler, "stop", lambda: calls.append("stop"))
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(f"push:{name}"))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append("pop"))
    cfg = C.create(dict(profiler=dict(enabled=True, profile_ranks=[0], profile_epoch=1)))
    prof = P.init_profiler(cfg)

    @P.profile("mlp")
    def f(x):
        return x + 1

    try:
        prof.set_epoch(0)
        assert f(1) == 2
        prof.set_epoch(1)
        with P.profile_range("forward pass"):
            pass
        prof.set_epoch(2)
        assert calls == ["push:mlp", "pop", "start", "push:forward pass", "pop", "stop"]
        calls.clear()
        prof.current_rank = 1  # not a profiled rank: no ranges, no window
        prof.set_epoch(1)
        assert f(2) == 3 and calls == []
    finally:
        P._profiler = None
