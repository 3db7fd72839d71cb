"""bench.py's configurations: the headline default and the hybrid / large / rollout layouts (CPU only:
argument parsing and the rank layout, no model is built)."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _parse(monkeypatch, *argv):
    import bench

    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    return bench, bench.parse()


def test_default_is_the_headline_configuration(monkeypatch):
    bench, a = _parse(monkeypatch)
    assert a.config == "dp" and a.gpus == 1 and a.global_batch == 16 and a.depth == 16
    assert (a.tp, a.sp1, a.sp2) == (1, 1, 1) and a.loss == "mse" and a.rollout == 1
    assert a.model_name == "swin-p4-e1024-d16" and a.model["embed_dim"] == 1024
    assert bench.layout(a, 8) == (8, "dp8")


@pytest.mark.parametrize("cfg,world,want", [("hybrid", 8, (2, "sp2=2 x tp=2 x dp=2")),
                                             ("hybrid", 4, (1, "sp2=2 x tp=2 x dp=1")),
                                             ("large", 8, (1, "sp2=2 x tp=4 x dp=1")),
                                             ("rollout", 8, (2, "sp2=2 x tp=2 x dp=2"))])
def test_other_layouts(monkeypatch, cfg, world, want):
    bench, a = _parse(monkeypatch, "--config", cfg)
    assert bench.layout(a, world) == want
    if cfg == "large":
        assert a.model["embed_dim"] == 2048 and a.depth == 24 and a.model["num_heads"] == 32
        assert a.loss == "amse" and a.rollout == 2 and a.global_batch == 4
    if cfg == "hybrid":
        assert a.global_batch == 8


def test_layout_overrides_and_rejections(monkeypatch):
    bench, a = _parse(monkeypatch, "--config", "large", "--tp", "2", "--depth", "4")
    assert a.depth == 4 and a.model["depth"] == 4 and bench.layout(a, 4) == (1, "sp2=2 x tp=2 x dp=1")
    with pytest.raises(SystemExit):
        bench.layout(a, 6)  # 6 GPUs do not divide into tp 2 x sp2 2
