"""Config composition, rank grid and shard-shape arithmetic (pure CPU)."""

import itertools
import os
import sys

import pytest

from neural_scaling_weather_b200 import config as C
from neural_scaling_weather_b200.parallel.helpers import (
    compute_split_shapes,
    compute_split_shapes_for_patching,
)
from neural_scaling_weather_b200.parallel.rank_grid import RankGrid

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def test_compose_defaults():
    cfg = C.compose("default")
    assert cfg.model.embed_dim == 1024 and cfg.model.window_size == [9, 18]
    assert cfg.optimizer.optimizer == "adam" and isinstance(cfg.optimizer.lr, float)
    assert cfg.optimizer.lr == pytest.approx(5e-4)
    assert cfg.parallelism.order == "sp1-sp2-tp-pp-dp"
    assert cfg.hydra.run.dir == "/expts/default/00"
    assert getattr(cfg.model, "coord_pos_embed", None) is True
    assert getattr(cfg.train, "limit_validation", "missing") == "missing"


def test_compose_overrides():
    cfg = C.compose("default", ["optimizer=adamw", "model.depth=24", "run_name=abc", "hydra=local",
                                "+train.extra=3", "~data.read_local", "loss=mse_weighted",
                                "model.window_size=[4,8]"])
    assert cfg.optimizer.weight_decay == pytest.approx(1e-4)
    assert cfg.model.depth == 24
    assert cfg.hydra.run.dir == "./outputs/abc/00"
    assert cfg.train.extra == 3
    assert "read_local" not in cfg.data
    assert cfg.loss.area_weights is True and cfg.loss.sfc_weights == "graphcast"
    assert list(cfg.model.window_size) == [4, 8]
    with pytest.raises(C.ConfigError):
        C.compose("default", ["model.not_a_key=1"])


def test_debug_overlay_and_yaml_roundtrip(tmp_path):
    cfg = C.compose("default", ["debug=check"])
    assert cfg.run_tag == "check" and cfg.disable_auto_resume is True
    assert cfg.data.batch_size == 4 and cfg.logging.log_to_wandb is False
    p = tmp_path / "hp.yaml"
    C.save(cfg, str(p))
    back = C.load(str(p))
    assert C.to_container(back) == C.to_container(cfg)


def _independent_groups(sizes, names, token):
    """Brute force: ranks sharing every coordinate outside ``token`` form one group."""
    world = 1
    for s in sizes:
        world *= s
    sel = token.split("-")

    def coords(r):
        out = {}
        for n, s in zip(names, sizes):
            out[n] = r % s
            r //= s
        return out

    groups = {}
    for r in range(world):
        c = coords(r)
        key = tuple(c[n] for n in names if n not in sel)
        groups.setdefault(key, []).append(r)
    return sorted(groups.values())


@pytest.mark.parametrize("tp,sp1,sp2,dp", [(1, 1, 1, 8), (2, 1, 2, 2), (4, 1, 2, 1), (2, 2, 2, 3),
                                            (1, 3, 1, 2)])
def test_rank_grid_groups(tp, sp1, sp2, dp):
    g = RankGrid(tp=tp, dp=dp, pp=1, sp1=sp1, sp2=sp2, order="sp1-sp2-tp-pp-dp")
    for token in ["tp", "dp", "sp1", "sp2", "sp1-sp2", "tp-sp1-sp2", "dp-sp1-sp2", "pp"]:
        got = g.get_ranks(token)
        assert sorted(got) == _independent_groups(g.ordered_sizes, g.names, token)
        for grp in got:
            assert grp == sorted(grp)


def test_rank_grid_megatron_example():
    g = RankGrid(tp=2, dp=2, pp=2, sp1=1, sp2=1, order="tp-pp-dp")
    assert g.get_ranks("dp") == [[0, 4], [1, 5], [2, 6], [3, 7]]
    assert g.get_ranks("tp") == [[0, 1], [2, 3], [4, 5], [6, 7]]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "utils")), reason="reference copy absent")
def test_rank_grid_matches_reference_listing():
    sys.path.insert(0, REF)
    try:
        import importlib

        rg = importlib.import_module("utils.rank_generator")
    finally:
        sys.path.remove(REF)
    for tp, sp1, sp2, dp in itertools.product([1, 2], [1, 2], [1, 2, 3], [1, 2]):
        for order in ["sp1-sp2-tp-pp-dp", "tp-dp", "sp1-sp2-tp-dp-pp"]:
            try:
                ref = rg.RankGenerator(tp=tp, dp=dp, pp=1, sp1=sp1, sp2=sp2, order=order)
            except RuntimeError:
                with pytest.raises(RuntimeError):
                    RankGrid(tp=tp, dp=dp, pp=1, sp1=sp1, sp2=sp2, order=order)
                continue
            mine = RankGrid(tp=tp, dp=dp, pp=1, sp1=sp1, sp2=sp2, order=order)
            for token in ["tp", "dp", "sp1", "sp2", "sp1-sp2", "tp-sp1-sp2", "dp-sp1-sp2", "pp"]:
                assert mine.get_ranks(token) == ref.get_ranks(token), (tp, sp1, sp2, dp, order, token)


def test_split_shapes():
    for size in range(1, 60):
        for n in range(1, min(size, 8) + 1):
            s = compute_split_shapes(size, n)
            assert len(s) == n and sum(s) == size and min(s) > 0
    assert compute_split_shapes_for_patching(721, 4, 4) == [180, 180, 180, 181]
    assert compute_split_shapes_for_patching(1440, 2, 4) == [720, 720]
    assert compute_split_shapes_for_patching(720, 3, 4) == [240, 240, 240]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "config")), reason="reference copy absent")
def test_config_tree_keeps_every_reference_key_and_default():
    """Every file of the reference's YAML tree exists here with every key and the same default value
    (the defaults list included), except the data loader: DALI is not available, so `synthetic` (same
    stateful sampling semantics) is the default.  Keys added here (e.g. train.cuda_graphs) are allowed."""
    import yaml

    def flat(d, pre=""):
        out = {}
        for k, v in (d or {}).items():
            out.update(flat(v, f"{pre}{k}.") if isinstance(v, dict) else {f"{pre}{k}": v})
        return out

    mine = os.path.join(os.path.dirname(C.__file__), "yaml")
    allowed = {("data/latlon_025deg.yaml", "loader"): ("dali", "synthetic")}
    n = 0
    for root, _, files in os.walk(os.path.join(REF, "config")):
        for f in files:
            if not f.endswith(".yaml"):
                continue
            rel = os.path.relpath(os.path.join(root, f), os.path.join(REF, "config"))
            ours = os.path.join(mine, rel)
            assert os.path.exists(ours), rel
            a = flat(yaml.safe_load(open(os.path.join(root, f))))
            b = flat(yaml.safe_load(open(ours)))
            for k, v in a.items():
                assert k in b, (rel, k)
                if (rel, k) in allowed:
                    assert (v, b[k]) == allowed[(rel, k)], (rel, k, v, b[k])
                else:
                    assert b[k] == v, (rel, k, v, b[k])
                n += 1
    assert n > 50
