"""Trainer, checkpoint format, resume exactness and host-side fault injection (CPU/gloo)."""

import os

import numpy as np
import pytest
import torch

from tests.dist_utils import run

BASE = ["parallelism.backend=gloo", "model.embed_dim=32", "model.depth=2", "model.num_heads=2",
        "model.window_size=[4,8]", "model.patch_size=2", "data.synthetic.nlat=32", "data.synthetic.nlon=64",
        "data.synthetic.n_samples=40", "data.levels=[500]", "data.batch_size=2", "optimizer=adamw",
        "train.clip_grad_norm=1.0", "logging.log_to_wandb=false", "logging.log_to_screen=false",
        "train.seed=7", "data.limit_nsamples_val=2"]


def _train(rank, world, exp_dir, extra, crash_at, out_path):
    import torch

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.training.trainer import Trainer

    cfg = C.compose("default", BASE + [f"hydra.run.dir={exp_dir}"] + list(extra))
    t = Trainer(cfg)
    if crash_at is not None:
        orig = t.optimizer_step

        def step_then_maybe_crash():
            orig()
            if t.iters == crash_at and rank == world - 1:
                # fault injection on the host: the last rank dies between steps
                os._exit(17)

        t.init_exp_dir(t.exp_dir)
        t.build()
        t.optimizer_step = step_then_maybe_crash
        t.train()
    else:
        t.launch()
    if rank == 0 and out_path:
        torch.save({k: v.detach().clone() for k, v in t.model.state_dict().items()}, out_path)


def test_checkpoint_format_and_keys(tmp_path):
    run(_train, 1, str(tmp_path / "a"), ["optimizer.max_iterations=4", "train.log_every=2"], None, None)
    ck = torch.load(tmp_path / "a" / "checkpoints" / "ckpt.tar", weights_only=False)
    assert set(ck) == {"iters", "n_mbs", "n_mbs_in_epoch", "epoch", "model_state", "optimizer_state_dict",
                       "scheduler_state_dict", "grad_scaler_state_dict", "best_loss", "best_iter",
                       "micro_batch_size"}
    assert ck["iters"] == 4
    assert all(k.startswith("module.model.") for k in ck["model_state"])
    assert "module.model.blocks.0.attn.q.weight" in ck["model_state"]
    assert (tmp_path / "a" / "checkpoints" / "ckpt_iter2.tar").exists()
    assert (tmp_path / "a" / "checkpoints" / "ckpt_best.tar").exists()
    lines = open(tmp_path / "a" / "logs.txt").read().strip().split("\n")
    head = lines[0].split(",")
    for key in ["iter", "train_time", "val_time", "val_nsteps", "flops_consumed", "learning_rate", "wt_norm",
                "val_loss", "best_val_loss", "best_iter", "train_loss", "grad", "val_rmse_u10m",
                "samples_per_sec", "tflops_per_sec", "mfu"]:
        assert key in head, key
    row = dict(zip(head, lines[-1].split(",")))
    assert float(row["samples_per_sec"]) > 0 and 0 < float(row["mfu"]) < 1
    # the optimizer state loads into torch.optim.AdamW
    model_params = [torch.zeros_like(v) for k, v in ck["model_state"].items()]
    opt = torch.optim.AdamW([torch.nn.Parameter(p) for p in model_params], lr=1e-3)
    opt.load_state_dict(ck["optimizer_state_dict"])


@pytest.mark.parametrize("world", [1, 2])
def test_resume_after_rank_failure_is_exact(tmp_path, world):
    """Uninterrupted run vs. a run whose last rank dies after step 4 (last checkpoint at 3), then auto-resumes."""
    ext = ["optimizer.max_iterations=6", "train.log_every=3"]
    full = str(tmp_path / "full.pt")
    run(_train, world, str(tmp_path / "u"), ext, None, full)
    with pytest.raises(AssertionError):
        run(_train, world, str(tmp_path / "r"), ext, 4, None, timeout=120)
    assert (tmp_path / "r" / "checkpoints" / "ckpt.tar").exists()
    resumed = str(tmp_path / "resumed.pt")
    run(_train, world, str(tmp_path / "r"), ext, None, resumed)
    a, b = torch.load(full), torch.load(resumed)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_finetune_and_branch(tmp_path):
    ext = ["optimizer.max_iterations=4", "train.log_every=2"]
    run(_train, 1, str(tmp_path / "base"), ext, None, None)
    ck = str(tmp_path / "base" / "checkpoints" / "ckpt.tar")
    run(_train, 1, str(tmp_path / "ft"), ext + [f"train.finetune_from={ck}"], None, None)
    ck2 = torch.load(tmp_path / "ft" / "checkpoints" / "ckpt.tar", weights_only=False)
    assert ck2["iters"] == 4
    run(_train, 1, str(tmp_path / "br"), ["optimizer.scheduler=cooldown", "optimizer.cooldown_from_iter=4",
                                          "optimizer.cooldown_to_iter=6", "optimizer.cooldown_fraction=0.2",
                                          "train.log_every=2", f"train.branch_from={ck}"], None, None)
    ck3 = torch.load(tmp_path / "br" / "checkpoints" / "ckpt.tar", weights_only=False)
    assert ck3["iters"] == 6


def test_synthetic_loader_semantics():
    from neural_scaling_weather_b200.data.synthetic import SyntheticERA5, SyntheticLoader

    ds = SyntheticERA5(nlat=16, nlon=32, sfc_vars=["a", "b"], pl_vars=[], levels=[], n_times=30, dt_scale=2,
                       invariants=["lsm", "coslat"], micro_batch_size=1)
    assert ds.n_samples_total == 30 - 2
    # determinism and advection: the next model step is the field shifted east by v cells
    a = ds.generate(np.array([10]))
    b = ds.generate(np.array([10]))
    assert torch.equal(a, b)
    ds0 = SyntheticERA5(nlat=16, nlon=32, sfc_vars=["a"], pl_vars=[], levels=[], n_times=30, dt_scale=2,
                        noise=0.0, invariants=[])
    f0 = ds0.generate(np.array([0]))[0, 0]
    f1 = ds0.generate(np.array([2]))[0, 0]
    v = int(ds0.v[0].item())
    assert torch.allclose(torch.roll(f0, v, dims=-1), f1, atol=1e-5)
    # epoch order: numpy default_rng(seed + ckpt_epoch + epoch) permutation, contiguous dp shard
    order = ds.epoch_indices(1)
    assert np.array_equal(order, np.random.default_rng(42 + 1).permutation(ds.n_samples_total))
    # resume skips n_mbs_in_epoch micro-batches once
    loader = SyntheticLoader(ds, 1)
    full = [x for x in loader]
    ds.set_dataset_state({"n_mbs_in_epoch": 5, "epoch": 0})
    loader2 = SyntheticLoader(ds, 1)
    resumed = [x for x in loader2]
    assert len(resumed) == len(full) - 5
    assert torch.equal(resumed[0], full[5])
    assert len([x for x in loader2]) == len(full)


def test_weight_cache_needs_the_same_live_parameter():
    """A cached cast / transpose is served only for the parameter object it was made from:
    ids are reused after a parameter is freed (a new model built in the same process)."""
    from neural_scaling_weather_b200.ops import weights

    p1 = torch.nn.Parameter(torch.randn(4, 3))
    t1 = weights.get_t([p1], p1.detach())
    assert t1.shape == (3, 4)
    assert weights.get_t([p1], p1.detach()) is t1  # cached
    refs, ver, t = weights._cache[("T", (id(p1),), torch.float32)]
    p2 = torch.nn.Parameter(torch.randn(5, 2))
    # an entry left by another parameter under p2's id is not used
    weights._cache[("T", (id(p2),), torch.float32)] = (refs, (p2._version,), t)
    assert weights.get_t([p2], p2.detach()).shape == (2, 5)
    c1 = weights.get(p1, torch.bfloat16)
    weights._cache[(id(p2), torch.bfloat16)] = weights._cache[(id(p1), torch.bfloat16)]
    c2 = weights.get(p2, torch.bfloat16)
    assert c1.shape == (4, 3) and c2.shape == (5, 2)
    with torch.no_grad():
        p1.add_(1.0)  # a new version is rebuilt
    assert torch.equal(weights.get(p1, torch.bfloat16), p1.detach().to(torch.bfloat16))


def test_device_prefetch_passes_through_on_cpu():
    from neural_scaling_weather_b200.data import device_prefetch

    src = [torch.full((2, 3), float(i)) for i in range(5)]
    out = list(device_prefetch(iter(src), "cpu"))
    assert len(out) == 5 and all(a is b for a, b in zip(out, src))


def test_checkpoint_checksum_detects_corruption(tmp_path):
    """atomic_save records a SHA-256 beside the file; verified_load refuses a corrupted file,
    completes a record left pending by an interrupted save, and loads record-less files."""
    import shutil

    from neural_scaling_weather_b200.utils.checkpoint_io import atomic_save, verified_load

    p = str(tmp_path / "ckpt.tar")
    atomic_save({"a": torch.arange(10)}, p)
    assert os.path.exists(p + ".sha256") and not os.path.exists(p + ".tmp")
    assert torch.equal(verified_load(p)["a"], torch.arange(10))
    # a save interrupted between its two renames: new file in place, its record still pending
    shutil.copy(p + ".sha256", str(tmp_path / "old.sha256"))
    atomic_save({"a": torch.arange(12)}, p)
    os.replace(p + ".sha256", p + ".sha256.tmp")
    shutil.copy(str(tmp_path / "old.sha256"), p + ".sha256")
    assert torch.equal(verified_load(p)["a"], torch.arange(12))
    assert not os.path.exists(p + ".sha256.tmp")
    # one flipped byte is caught
    data = bytearray(open(p, "rb").read())
    data[len(data) // 2] ^= 0xFF
    open(p, "wb").write(bytes(data))
    with pytest.raises(RuntimeError, match="SHA-256"):
        verified_load(p)
    # files without a record (the reference's checkpoints) load unchecked
    q = str(tmp_path / "ref.tar")
    torch.save({"b": 1}, q)
    assert verified_load(q)["b"] == 1


def _infer(rank, world, exp_dir, ckpt_dir, out_path, threshold="1e9"):
    import torch

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.inference.inferencer import Inferencer

    cfg = C.compose("default", BASE + [
        f"hydra.run.dir={exp_dir}", f"inference.checkpoint={ckpt_dir}/checkpoints/ckpt.tar",
        f"inference.checkpoint_hyperparams={ckpt_dir}/hyperparameters.yaml",
        "inference.start_date='2018-01-01T00'", "inference.end_date='2018-01-02T12'",
        "inference.time_horizon_in_hours=12", "inference.spectra_times_in_hours=[6]",
        f"inference.unstable_rmse_threshold={threshold}"])
    out = Inferencer(cfg).launch()
    if rank == 0:
        torch.save({"rmse": out["rmse"], "acc": out["acc"], "spectra": out["spectra"][6],
                    "unstable": out["unstable"]}, out_path)


def test_inference_rollout_scores_and_dp_split(tmp_path):
    """Train a tiny model briefly, then roll it out from four initial conditions (every 12 h)
    to 12 h (the instability cut is lifted: a two-step model is far from the reference's
    threshold): RMSE / ACC per channel and lead, power spectra at 6 h and the .npy outputs; the ICs
    split over two dp ranks (round-robin, sums all-reduced) give the single-rank scores."""
    ckpt_dir = str(tmp_path / "train")
    run(_train, 1, ckpt_dir, ["optimizer.max_iterations=2", "train.log_every=2"], None, None)
    one, two = str(tmp_path / "one.pt"), str(tmp_path / "two.pt")
    run(_infer, 1, str(tmp_path / "inf1"), ckpt_dir, one)
    run(_infer, 2, str(tmp_path / "inf2"), ckpt_dir, two)
    a, b = torch.load(one), torch.load(two)
    n_ch = a["rmse"].shape[0]
    assert a["rmse"].shape == (n_ch, 2) and a["acc"].shape == (n_ch, 2)
    assert a["spectra"].shape[:2] == (2, n_ch)
    assert torch.isfinite(a["rmse"]).all() and (a["rmse"] > 0).all()
    assert (a["acc"].abs() <= 1 + 1e-5).all()
    assert a["unstable"] == b["unstable"] == 0
    for k in ("rmse", "acc", "spectra"):
        assert torch.allclose(a[k], b[k], rtol=1e-5, atol=1e-7), k
    assert (tmp_path / "inf1" / "rmse_u10m.npy").exists()
    assert (tmp_path / "inf1" / "spectra_u10m_6h.npy").exists()
    # every IC over the cut (threshold 0): all four dropped, counted once across the dp ranks
    cut = str(tmp_path / "cut.pt")
    run(_infer, 2, str(tmp_path / "inf3"), ckpt_dir, cut, "0")
    c = torch.load(cut)
    assert c["unstable"] == 4 and torch.equal(c["rmse"], torch.zeros_like(c["rmse"]))


def _bench_infer(rank, world, exp_dir, out_path):
    import numpy as np
    import torch

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.inference.benchmarks import ForecastSource
    from neural_scaling_weather_b200.inference.inferencer import Inferencer

    class TruthOnWB2Grid(ForecastSource):
        """The dataset's own future fields in physical units, laid out like a WeatherBench2 store
        (south to north, with a south-pole row); 't2m' is missing from it."""

        inf = None

        def fetch(self, ic, leads_h, var, level):
            name = var if level is None else f"{var}{level}"
            chans = list(self.inf.metadata["channels"])
            if name not in chans or name == "t2m":
                return None
            ci = chans.index(name)
            ds = self.inf.test_dataset
            out = []
            for h in leads_h:
                x = ds.get_samples([ic + np.timedelta64(int(h), "h")]).numpy()
                phys = (x * ds.stds + ds.means)[0, ci]  # model grid, north to south
                pole = np.full((1, phys.shape[1]), 1e6, dtype=np.float32)  # must be cut
                out.append(np.concatenate([phys, pole], 0)[::-1])
            return np.stack(out)

    src = TruthOnWB2Grid()
    cfg = C.compose("default", BASE + [
        f"hydra.run.dir={exp_dir}", "inference.run_benchmark=hres", "inference.checkpoint_hyperparams=null",
        "inference.start_date='2018-01-01T00'", "inference.end_date='2018-01-02T12'",
        "inference.time_horizon_in_hours=12", "inference.spectra_times_in_hours=[6]",
        "inference.unstable_rmse_threshold=1e9", "inference.log_sfc=['u10m','t2m']", "inference.log_var=['z']"])
    inf = Inferencer(cfg, bench_source=src)
    src.inf = inf
    out = inf.launch()
    if rank == 0:
        torch.save({"rmse": out["rmse"], "acc": out["acc"], "channels": list(inf.metadata["channels"]),
                    "model": inf.model}, out_path)


def test_benchmark_forecast_scored_in_place_of_the_model(tmp_path):
    """inference.run_benchmark scores a third-party forecast instead of the model: fields matched to the
    channels by name, flipped from south-north to north-south with the pole row cut, scored against the
    same targets.  A source that returns the truth scores RMSE 0 and ACC 1 on its channels; the channel it
    lacks (t2m) stays zero, as in the reference."""
    out = str(tmp_path / "bench.pt")
    run(_bench_infer, 1, str(tmp_path / "inf"), out)
    r = torch.load(out, weights_only=False)
    assert r["model"] is None
    chans = r["channels"]
    t2m = chans.index("t2m")
    others = [i for i in range(len(chans)) if i != t2m]
    assert r["rmse"][others].abs().max() < 1e-3
    assert (r["acc"][others] - 1).abs().max() < 1e-4
    assert (r["rmse"][t2m] > 1.0).all()


def test_benchmark_channel_names_and_grid_layout():
    """Channel names split into variable and pressure level; the assembled shard is flipped to north-south,
    cut to the model's rows and sliced to this rank's part of the grid."""
    import numpy as np

    from neural_scaling_weather_b200.inference.benchmarks import ForecastSource, assemble, split_channel

    assert split_channel("z500") == ("z", 500) and split_channel("u10m") == ("u10m", None)
    assert split_channel("t2m") == ("t2m", None) and split_channel(b"q850") == ("q", 850)

    class Ramp(ForecastSource):
        def fetch(self, ic, leads_h, var, level):
            if var != "u":
                return None
            lat = np.arange(5, dtype=np.float32)[:, None] * np.ones((1, 6), np.float32)  # row index, S->N
            return np.stack([lat + 100 * i for i in range(len(leads_h))])

    fc, found = assemble(Ramp(), None, [6, 12], ["t2m", "u500"], slice(1, 3), slice(2, 5), n_lat=4)
    assert found == [1] and fc.shape == (2, 2, 2, 3)
    # model rows (north to south) are source rows 4, 3, 2, 1; this shard takes model rows 1..2 -> 3, 2
    assert torch.equal(fc[0, 1, :, 0], torch.tensor([3.0, 2.0])) and torch.equal(fc[1, 1, :, 0], torch.tensor([103.0, 102.0]))
    assert torch.count_nonzero(fc[:, 0]) == 0


def test_device_loss_scaler_follows_torch_grad_scaler():
    """The device-side loss scaler's back-off / growth rule and checkpoint keys match
    torch.amp.GradScaler on the same sequence of finite and non-finite steps."""
    from neural_scaling_weather_b200.training.loss_scale import DeviceLossScaler

    kw = dict(init_scale=1024.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=3)
    ours = DeviceLossScaler("cpu", **kw)
    ref = torch.amp.GradScaler("cpu", **kw)
    p = torch.nn.Parameter(torch.ones(4))
    opt = torch.optim.SGD([p], lr=0.0)
    for bad in [0, 0, 1, 0, 0, 0, 0, 1, 1, 0, 0, 0, 0, 0, 0, 0]:
        opt.zero_grad()
        ref.scale((p * (float("inf") if bad else 1.0)).sum()).backward()
        ref.step(opt)
        ref.update()
        ours.update(torch.tensor([bad], dtype=torch.int32))
        assert ours.state_dict()["scale"] == ref.get_scale()
        assert ours.state_dict()["_growth_tracker"] == ref.state_dict()["_growth_tracker"]
    assert set(ours.state_dict()) == set(ref.state_dict())
    fresh = DeviceLossScaler("cpu", **kw)
    fresh.load_state_dict(ref.state_dict())
    assert fresh.state_dict() == ours.state_dict()


def test_weight_cache_entries_built_in_inference_mode_stay_usable_in_training():
    """Casts, concatenations, transposes and derived tensors of the weight cache that are first built
    during validation or a rollout (torch.inference_mode) are ordinary tensors: the training forward that
    finds them in the cache afterwards can still build its autograd graph through them."""
    from neural_scaling_weather_b200.ops import weights as wcache

    wcache.clear()
    w1, w2 = torch.nn.Parameter(torch.randn(4, 3)), torch.nn.Parameter(torch.randn(2, 3))
    with torch.inference_mode():
        a = wcache.get(w1, torch.bfloat16)
        c = wcache.get_cat([w1, w2], torch.bfloat16)
        t = wcache.get_t([w1, w2], c)
        d = wcache.get_derived(("double",), [w1], lambda: w1.detach() * 2)
    assert not any(x.is_inference() for x in (a, c, t, d))
    assert wcache.get(w1, torch.bfloat16) is a and wcache.get_derived(("double",), [w1], lambda: None) is d

    class Through(torch.autograd.Function):  # returns a cached tensor, as the positional embedding does
        @staticmethod
        def forward(ctx, w):
            return d.view_as(d)

        @staticmethod
        def backward(ctx, g):
            return 2 * g

    Through.apply(w1).sum().backward()
    assert torch.equal(w1.grad, torch.full_like(w1, 2.0))
    wcache.clear()


def _random_init_infer(rank, world, exp_dir, out_path):
    import torch

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.inference.inferencer import Inferencer

    cfg = C.compose("default", BASE + [
        f"hydra.run.dir={exp_dir}", f"inference.checkpoint={exp_dir}/none.tar", "inference.checkpoint_hyperparams=null",
        "inference.random_init=true", "inference.start_date='2018-01-01T00'", "inference.end_date='2018-01-01T12'",
        "inference.time_horizon_in_hours=6", "inference.spectra_times_in_hours=[]",
        "inference.unstable_rmse_threshold=1e30"])
    out = Inferencer(cfg).launch()
    if rank == 0:
        torch.save({"rmse": out["rmse"]}, out_path)


def test_inference_without_checkpoint_needs_random_init(tmp_path):
    """inference.random_init=true rolls out random-init weights when the checkpoint does not exist (the
    benchmark's rollout); without it a missing checkpoint is an error."""
    out = str(tmp_path / "r.pt")
    run(_random_init_infer, 1, str(tmp_path / "inf"), out)
    r = torch.load(out)
    assert torch.isfinite(r["rmse"]).all() and (r["rmse"] > 0).all()

    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.inference.inferencer import Inferencer

    cfg = C.compose("default", BASE + [f"hydra.run.dir={tmp_path / 'inf2'}", f"inference.checkpoint={tmp_path}/none.tar",
                                       "inference.checkpoint_hyperparams=null"])
    inf = Inferencer.__new__(Inferencer)  # the checkpoint check only (no process group needed)
    inf.cfg, inf.world_rank, inf.log_to_screen = cfg, 0, False
    with pytest.raises(FileNotFoundError):
        inf.init_exp_dir(str(tmp_path / "inf2"))
