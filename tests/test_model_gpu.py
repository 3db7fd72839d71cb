"""End-to-end model numerics on the GPU path (bf16 kernels) against the fp32 CPU oracle."""

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from neural_scaling_weather_b200 import config as C  # noqa: E402
from neural_scaling_weather_b200.models import get_model  # noqa: E402
from neural_scaling_weather_b200.ops import _ext  # noqa: E402
from neural_scaling_weather_b200.utils.misc import create_dummy_metadata  # noqa: E402


def _cfg(embed=64, depth=2, heads=4, window=(4, 8), patch=2, nrs=1):
    return C.create(dict(
        model=dict(arch="swin", embed_dim=embed, patch_size=patch, depth=depth, window_size=list(window),
                   num_heads=heads, dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=["a", "b", "c"]),
        train=dict(temporal_context_window=1, num_rollout_steps=nrs),
        parallelism=dict(use_transformer_engine=False)))


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("nrs", [1, 2])
def test_model_forward_backward_matches_cpu(nrs):
    torch.manual_seed(0)
    H, W, Cc = 32, 64, 5
    md = create_dummy_metadata(H, W, Cc)
    cfg = _cfg(nrs=nrs)
    cpu = get_model(cfg, md)
    gpu = get_model(cfg, md).cuda()
    gpu.load_state_dict(cpu.state_dict())
    x = torch.randn(2, 1, Cc + 3, H, W)
    y = torch.randn(2, nrs, Cc, H, W)
    out_c = cpu(x)
    loss_c = ((out_c - y) ** 2).mean()
    loss_c.backward()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out_g = gpu(x.cuda())
    loss_g = ((out_g.float() - y.cuda()) ** 2).mean()
    loss_g.backward()
    assert rel(out_g.cpu(), out_c) < 3e-2
    gc = dict(cpu.named_parameters())
    for name, p in gpu.named_parameters():
        assert p.grad is not None, name
        assert rel(p.grad.cpu(), gc[name].grad) < 8e-2, name
    assert _ext.require().read_error_flag(True) == 0


def test_trainer_steps_on_gpu(tmp_path):
    from neural_scaling_weather_b200.training.trainer import Trainer

    cfg = C.compose("default", [
        f"hydra.run.dir={tmp_path}", "parallelism.backend=nccl", "model.embed_dim=64", "model.depth=2",
        "model.num_heads=4", "model.window_size=[4,8]", "model.patch_size=2", "data.synthetic.nlat=32",
        "data.synthetic.nlon=64", "data.synthetic.n_samples=40", "data.levels=[500]", "data.batch_size=2",
        "optimizer=adamw", "optimizer.max_iterations=4", "train.log_every=2", "train.amp_dtype=bf16",
        "train.clip_grad_norm=1.0", "logging.log_to_wandb=false", "train.seed=1"])
    import os

    os.environ.setdefault("MASTER_PORT", "29533")
    t = Trainer(cfg)
    t.launch()
    assert t.iters == 4
    assert (tmp_path / "checkpoints" / "ckpt.tar").exists()
    assert _ext.require().read_error_flag(True) == 0
    import torch.distributed as dist

    dist.destroy_process_group()


def test_trainer_stops_when_device_error_word_is_set(tmp_path):
    """A kernel whose bounded wait runs out sets the device error word and returns with
    incomplete outputs; training must stop with DeviceError and write no checkpoint.  The
    word is set from the host here (no kernel is made to fail)."""
    import os

    import torch.distributed as dist

    from neural_scaling_weather_b200.ops._ext import DeviceError
    from neural_scaling_weather_b200.training.trainer import Trainer

    os.environ.setdefault("MASTER_PORT", "29535")
    cfg = C.compose("default", [
        f"hydra.run.dir={tmp_path}", "parallelism.backend=nccl", "model.embed_dim=64", "model.depth=2",
        "model.num_heads=4", "model.window_size=[4,8]", "model.patch_size=2", "data.synthetic.nlat=32",
        "data.synthetic.nlon=64", "data.synthetic.n_samples=40", "data.levels=[500]", "data.batch_size=2",
        "optimizer=adamw", "optimizer.max_iterations=4", "train.log_every=2", "train.amp_dtype=bf16",
        "logging.log_to_wandb=false", "train.seed=1"])
    t = Trainer(cfg)
    t.init_exp_dir(t.exp_dir)
    t.build()
    ext = _ext.require()
    assert ext.read_error_flag(True) == 0
    ext.set_error_flag(1)
    try:
        with pytest.raises(DeviceError) as info:
            t.train()
        assert info.value.code == 1
        assert t.iters < 4
        assert not (tmp_path / "checkpoints" / "ckpt.tar").exists()
    finally:
        ext.read_error_flag(True)
        dist.destroy_process_group()
    assert ext.read_error_flag(True) == 0


def test_trainer_fp16_loss_scaling_on_the_fused_step(tmp_path):
    """fp16 training: the gradient norm of the scaled gradients gives the inf check and, divided by the
    scale, the clip; the fused AdamW kernel unscales and clips in one multiply.  A step whose gradients
    hold an inf leaves every parameter unchanged and halves the scale; the next finite step updates."""
    import os

    import torch.distributed as dist

    from neural_scaling_weather_b200.training.loss_scale import DeviceLossScaler
    from neural_scaling_weather_b200.training.trainer import Trainer

    os.environ.setdefault("MASTER_PORT", "29536")
    cfg = C.compose("default", [
        f"hydra.run.dir={tmp_path}", "parallelism.backend=nccl", "model.embed_dim=64", "model.depth=2",
        "model.num_heads=4", "model.window_size=[4,8]", "model.patch_size=2", "data.synthetic.nlat=32",
        "data.synthetic.nlon=64", "data.synthetic.n_samples=40", "data.levels=[500]", "data.batch_size=2",
        "optimizer=adamw", "optimizer.max_iterations=4", "train.amp_dtype=fp16", "train.clip_grad_norm=1.0",
        "logging.log_to_wandb=false", "train.seed=1"])
    t = Trainer(cfg)
    t.init_exp_dir(t.exp_dir)
    t.build()
    try:
        assert isinstance(t.gscaler, DeviceLossScaler) and t.gscaler.is_enabled()
        batches = iter(t.train_data_loader)
        b = next(batches).cuda()
        s0 = float(t.gscaler._scale.item())
        # a finite step updates the parameters
        before = t.space.data.clone()
        t.train_step(b, is_optimizer_step=False)
        t.train_step(b, is_optimizer_step=True)
        torch.cuda.synchronize()
        assert not torch.equal(t.space.data, before) and torch.isfinite(t.space.data).all()
        assert float(t.gscaler._scale.item()) == s0
        # an inf in one gradient: the step is skipped and the scale backs off
        before = t.space.data.clone()
        t.train_step(b, is_optimizer_step=False)
        t.space.grad[3] = float("inf")
        t.train_step(b, is_optimizer_step=True)
        torch.cuda.synchronize()
        assert torch.equal(t.space.data, before)
        assert float(t.gscaler._scale.item()) == s0 * 0.5
        # and training goes on
        t.train_step(b, is_optimizer_step=False)
        t.train_step(b, is_optimizer_step=True)
        torch.cuda.synchronize()
        assert not torch.equal(t.space.data, before) and torch.isfinite(t.space.data).all()
        assert t.gscaler.state_dict()["scale"] == s0 * 0.5
    finally:
        dist.destroy_process_group()


def test_trainer_cuda_graph_matches_eager(tmp_path):
    """Micro-batches replayed from a captured CUDA graph (derived weight copies refreshed in
    place after each optimizer step) follow the eager loss and parameter trajectory."""
    import os

    import torch.distributed as dist

    from neural_scaling_weather_b200.ops import weights as wcache
    from neural_scaling_weather_b200.training.trainer import Trainer

    os.environ.setdefault("MASTER_PORT", "29534")
    results = []
    for graphs in (False, True):
        wcache.clear()
        cfg = C.compose("default", [
            f"hydra.run.dir={tmp_path}/g{int(graphs)}", "parallelism.backend=nccl", "model.embed_dim=128",
            "model.depth=2", "model.num_heads=2", "model.window_size=[4,8]", "model.patch_size=2",
            "data.synthetic.nlat=32", "data.synthetic.nlon=64", "data.synthetic.n_samples=40", "data.levels=[500]",
            "data.batch_size=4", "optimizer=adamw", "optimizer.scheduler=null", "train.amp_dtype=bf16",
            "train.clip_grad_norm=1.0", "logging.log_to_wandb=false", "train.seed=1", "train.save_checkpoint=false",
            f"train.cuda_graphs={'true' if graphs else 'false'}"])
        t = Trainer(cfg)
        t.init_exp_dir(t.exp_dir)
        t.build()
        it = iter(t.train_data_loader)
        batches = [next(it).to("cuda") for _ in range(4)]
        losses = []
        for step in range(5):
            for i in range(t.gradient_accum_steps):
                loss = t.train_step(batches[(step + i) % 4], is_optimizer_step=(i == t.gradient_accum_steps - 1))
                losses.append(float(loss))
        if graphs:
            assert t._graph is not None, "the micro-batch was not captured"
        flat = torch.cat([p.detach().flatten().float() for p in t.model.parameters()])
        results.append((losses, flat))
        assert _ext.require().read_error_flag(True) == 0
        dist.destroy_process_group()
    (le, pe), (lg, pg) = results
    for a, b in zip(le, lg):
        assert abs(a - b) <= 2e-3 * max(1.0, abs(a)), (le, lg)
    assert rel(pg, pe) < 2e-3


def test_device_prefetch_copies_ahead_on_a_side_stream():
    from neural_scaling_weather_b200.data import device_prefetch

    src = [torch.randn(3, 1000).pin_memory() for _ in range(6)] + [torch.ones(2, device="cuda")]
    seen = []
    for i, d in enumerate(device_prefetch(iter(src), "cuda", depth=2)):
        assert d.is_cuda
        seen.append(d.clone() * 2)  # consumed on the compute stream
    torch.cuda.synchronize()
    assert len(seen) == len(src)
    for a, b in zip(seen, src):
        assert torch.equal(a.cpu(), b.cpu() * 2)


def test_inference_bf16_matches_fp32_on_gpu(tmp_path):
    """The inferencer on CUDA: the same random-weight model rolled out from two ICs in fp32
    (plain-PyTorch operators, fp32 arithmetic) and in bf16 (the fused kernels) gives close
    RMSE / ACC, and reports a device-timed step."""
    import os

    import torch.distributed as dist

    from neural_scaling_weather_b200.inference.inferencer import Inferencer

    os.environ.setdefault("MASTER_PORT", "29534")
    base = ["parallelism.backend=nccl", "model.embed_dim=64", "model.depth=2", "model.num_heads=4",
            "model.window_size=[4,8]", "model.patch_size=2", "data.synthetic.nlat=32", "data.synthetic.nlon=64",
            "data.synthetic.n_samples=40", "data.levels=[500]", "logging.log_to_wandb=false",
            "inference.random_init=true", f"inference.checkpoint={tmp_path}/no_ckpt.tar",
            f"inference.checkpoint_hyperparams={tmp_path}/no_hp.yaml",
            "inference.start_date='2018-01-01T00'", "inference.end_date='2018-01-01T12'",
            "inference.time_horizon_in_hours=12", "inference.spectra_times_in_hours=[]",
            "inference.unstable_rmse_threshold=1e9"]
    res = {}
    for prec in ("fp32", "bf16"):
        torch.manual_seed(0)
        cfg = C.compose("default", base + [f"hydra.run.dir={tmp_path / prec}", f"inference.precision={prec}"])
        res[prec] = Inferencer(cfg).launch()
        dist.destroy_process_group()
    a, b = res["fp32"], res["bf16"]
    assert torch.isfinite(b["rmse"]).all() and (b["rmse"] > 0).all()
    assert rel(b["rmse"], a["rmse"]) < 3e-2
    assert (b["acc"] - a["acc"]).abs().max().item() < 2e-2
    assert b["ms_per_step"] is not None and b["ms_per_step"] > 0
    assert _ext.require().read_error_flag(True) == 0


@pytest.mark.parametrize("nrs", [1, 2])
def test_weight_grads_written_in_place_match_returned_grads(nrs):
    """With the optimizer's flat fp32 gradient buffer as .grad, the weight-gradient kernel adds dW / db
    into it in place (no autograd accumulation); the result equals the gradients autograd receives
    when .grad starts unset, and the in-place hook (the data-parallel reducer's trigger) runs once per
    parameter even when a rollout applies the model twice."""
    from neural_scaling_weather_b200.ops import gradsink
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace

    torch.manual_seed(0)
    H, W, Cc = 32, 64, 5
    md = create_dummy_metadata(H, W, Cc)
    cfg = _cfg(embed=128, heads=2, nrs=nrs)
    a = get_model(cfg, md).cuda()
    b = get_model(cfg, md).cuda()
    b.load_state_dict(a.state_dict())
    space = FlatParamSpace([p for p in b.parameters()])

    class Counter:
        def __init__(self):
            self.n = {}

        def hit(self, p):
            self.n[id(p)] = self.n.get(id(p), 0) + 1

    cnt = Counter()
    gradsink.register(cnt.hit)
    x = torch.randn(2, 1, Cc + 3, H, W, device="cuda")
    y = torch.randn(2, nrs, Cc, H, W, device="cuda")
    for m in (a, b):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = m(x)
        ((out.float() - y) ** 2).mean().backward()
    torch.cuda.synchronize()
    gradsink.unregister(cnt.hit)
    ga = dict(a.named_parameters())
    n_in_place = 0
    for name, p in b.named_parameters():
        assert p.grad is not None and p.grad.data_ptr() >= space.grad.data_ptr(), name
        assert rel(p.grad, ga[name].grad) < 1e-4, name
        if id(p) in cnt.n:
            assert cnt.n[id(p)] == 1, name
            n_in_place += 1
    assert n_in_place >= 8  # the linear / MLP / patch-embed / head weights and biases
    assert _ext.require().read_error_flag(True) == 0
