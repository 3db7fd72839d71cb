"""Distributed primitives and the sharded model against the single-rank oracle (gloo, CPU).

Pattern of the reference's tests (``tests/test_all.py``, ``tests/test_distributed_roll.py``):
run the op as if non-distributed on the full tensor, then on shards, gather the outputs
and gradients and compare.
"""

import pytest
import torch

from tests.dist_utils import run

pytestmark = pytest.mark.timeout(900) if hasattr(pytest.mark, "timeout") else []


# ----------------------------------------------------------------------------- roll
def _roll_worker(rank, world, sp1, sp2, H, W, shifts):
    import torch

    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes, offsets
    from neural_scaling_weather_b200.parallel.mappings import roll_forward_reverseroll_backward

    comm.init_model_parallel_info(tp=1, sp1=sp1, sp2=sp2, dp=world // (sp1 * sp2))
    torch.manual_seed(0)
    x = torch.randn(2, 1, H, W, 3, dtype=torch.float64)
    g = torch.randn(2, 1, H, W, 3, dtype=torch.float64)
    ref = torch.roll(x, shifts=shifts, dims=(2, 3))
    s1 = compute_split_shapes(H, sp1)
    s2 = compute_split_shapes(W, sp2)
    r1, r2 = comm.get_rank("sp1"), comm.get_rank("sp2")
    o1, o2 = offsets(s1)[r1], offsets(s2)[r2]
    xl = x[:, :, o1:o1 + s1[r1], o2:o2 + s2[r2]].clone().requires_grad_()
    y = roll_forward_reverseroll_backward(xl, shifts, (-3, -2), ["sp1", "sp2"], shapes=(s1, s2))
    assert torch.equal(y, ref[:, :, o1:o1 + s1[r1], o2:o2 + s2[r2]])
    gl = g[:, :, o1:o1 + s1[r1], o2:o2 + s2[r2]]
    y.backward(gl)
    gref = torch.roll(g, shifts=tuple(-s for s in shifts), dims=(2, 3))
    assert torch.equal(xl.grad, gref[:, :, o1:o1 + s1[r1], o2:o2 + s2[r2]])


@pytest.mark.parametrize("sp1,sp2,H,W,shifts", [
    (1, 2, 8, 16, (-2, -4)), (2, 1, 9, 16, (3, 5)), (2, 2, 10, 12, (-4, -5)),
    (1, 4, 6, 17, (-1, -9)), (4, 1, 13, 8, (7, 0)),
])
def test_distributed_roll(sp1, sp2, H, W, shifts):
    run(_roll_worker, sp1 * sp2, sp1, sp2, H, W, shifts)


def _gather_worker(rank, world):
    import torch

    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.helpers import _gather, _reduce_scatter, _split, compute_split_shapes

    comm.init_model_parallel_info(tp=world, dp=1)
    shapes = compute_split_shapes(11, world)
    full = torch.arange(11 * 3, dtype=torch.float32).view(11, 3)
    part = _split(full, 0, "tp", shapes)
    back = _gather(part, 0, shapes, "tp")
    assert torch.equal(back, full)
    rs = _reduce_scatter(full * (rank + 1), 0, shapes, "tp")
    tot = sum(range(1, world + 1))
    assert torch.equal(rs, _split(full * tot, 0, "tp", shapes))


def test_gather_split_reduce_scatter():
    run(_gather_worker, 3)


# ----------------------------------------------------------------------------- sharded model
def _tiny_cfg(nrs=1):
    from neural_scaling_weather_b200 import config as C

    return C.create(dict(
        model=dict(arch="swin", embed_dim=32, patch_size=2, depth=2, window_size=[4, 8], num_heads=4,
                   dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=["a"]),
        train=dict(temporal_context_window=1, num_rollout_steps=nrs),
        parallelism=dict(use_transformer_engine=False)))


def _shard_param(name, full, p, comm):
    """Slice a full (single-rank) parameter to this rank's shard per comm_metadata."""
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes, offsets

    out = full
    for dim, grp in enumerate(p.comm_metadata["sharded"]):
        if grp is None or comm.get_size(grp) == 1:
            continue
        n = comm.get_size(grp)
        shapes = compute_split_shapes(full.shape[dim], n)
        r = comm.get_rank(grp)
        out = out.narrow(dim, offsets(shapes)[r], shapes[r])
    return out


def _gather_param_grad(g, p, comm):
    import torch.distributed as dist

    from neural_scaling_weather_b200.parallel.helpers import _gather

    out = g
    for dim, grp in enumerate(p.comm_metadata["sharded"]):
        if grp is None or comm.get_size(grp) == 1:
            continue
        out = _gather(out, dim, None, grp)
    return out


def _model_worker(rank, world, tp, sp1, sp2, H, W):
    import torch

    from neural_scaling_weather_b200.losses import WeightedLoss
    from neural_scaling_weather_b200.models import get_model
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.grad_sync import GradReducer, order_params
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes_for_patching, offsets
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace
    from neural_scaling_weather_b200.utils.misc import create_dummy_metadata, split_dummy_metadata

    Cc, p = 4, 2
    dp = world // (tp * sp1 * sp2)
    cfg = _tiny_cfg()
    torch.manual_seed(0)
    md_full = create_dummy_metadata(H, W, Cc)
    md_full["area_weights"] = torch.rand(H, 1)
    x = torch.randn(2 * dp, 1, Cc + 1, H, W)
    y = torch.randn(2 * dp, 1, Cc, H, W)

    # single-rank oracle (groups absent -> sizes 1)
    ref = get_model(cfg, md_full)
    loss_ref = WeightedLoss(area_weighting=True, weights=md_full["area_weights"])
    out_ref = ref(x)
    l_ref = loss_ref(out_ref, y)
    l_ref.backward()

    comm.init_model_parallel_info(tp=tp, sp1=sp1, sp2=sp2, dp=dp)
    s1 = compute_split_shapes_for_patching(H, sp1, p)
    s2 = compute_split_shapes_for_patching(W, sp2, p)
    md = split_dummy_metadata(md_full, s1, s2)
    md["area_weights"] = md_full["area_weights"][md["sp_slices"][0]]
    model = get_model(cfg, md)
    full_state = dict(ref.named_parameters())
    with torch.no_grad():
        for name, prm in model.named_parameters():
            prm.copy_(_shard_param(name, full_state[name].detach(), prm, comm))
    space = FlatParamSpace(order_params(list(model.parameters())))
    reducer = GradReducer(space, broadcast_from_root=False)
    r1, r2, rd = comm.get_rank("sp1"), comm.get_rank("sp2"), comm.get_rank("dp")
    o1, o2 = offsets(s1)[r1], offsets(s2)[r2]
    xl = x[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]]
    yl = y[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]]
    loss_fn = WeightedLoss(area_weighting=True, weights=md["area_weights"])
    out = model(xl)
    assert torch.allclose(out, out_ref[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]],
                          atol=1e-5, rtol=1e-4)
    loss = loss_fn(out, yl)
    # dp ranks see different samples; the global loss is the dp mean
    loss.backward()
    reducer.finish()
    for name, prm in model.named_parameters():
        g = _gather_param_grad(prm.grad, prm, comm)
        gr = full_state[name].grad
        err = ((g - gr).norm() / gr.norm().clamp_min(1e-12)).item()
        assert err < 1e-4, (name, err)


@pytest.mark.parametrize("tp,sp1,sp2,H,W", [
    (1, 1, 2, 16, 32), (1, 2, 1, 16, 32), (2, 1, 1, 16, 32), (2, 1, 2, 16, 32), (1, 2, 2, 16, 32),
    (1, 1, 1, 16, 32),
])
def test_sharded_model_matches_single_rank(tp, sp1, sp2, H, W):
    world = tp * sp1 * sp2 * (2 if tp * sp1 * sp2 == 1 else 1)
    run(_model_worker, world, tp, sp1, sp2, H, W)


def _train_worker(rank, world, sp2, steps, result_path):
    """tiny Swin, gloo world 2 with sp2=2, 3 Adam steps."""
    import torch

    from neural_scaling_weather_b200.losses import WeightedLoss
    from neural_scaling_weather_b200.models import get_model
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.grad_sync import GradReducer, order_params
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes_for_patching, offsets
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace, FusedAdamW
    from neural_scaling_weather_b200.data.synthetic import SyntheticERA5
    from neural_scaling_weather_b200 import config as C

    cfg = C.create(dict(
        model=dict(arch="swin", embed_dim=64, patch_size=2, depth=2, window_size=[4, 8], num_heads=4,
                   dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=[]), train=dict(temporal_context_window=1, num_rollout_steps=1),
        parallelism=dict(use_transformer_engine=False)))
    if sp2 > 1:
        comm.init_model_parallel_info(tp=1, sp1=1, sp2=sp2, dp=1)
    ds = SyntheticERA5(nlat=32, nlon=64, sfc_vars=["a", "b", "c", "d"], pl_vars=["e"], levels=[500, 850],
                       n_times=40, dt_scale=1, model_patch_size=2, invariants=[], advect_min=1,
                       advect_max=1)
    torch.manual_seed(0)
    model = get_model(cfg, ds.metadata)
    space = FlatParamSpace(order_params(list(model.parameters())))
    reducer = GradReducer(space, broadcast_from_root=False)
    opt = FusedAdamW(list(model.parameters()), lr=1e-3, betas=(0.9, 0.95), space=space,
                     decoupled_weight_decay=False)
    loss_fn = WeightedLoss(area_weighting=True, weights=ds.metadata["area_weights"])
    for step in range(steps):
        batch = torch.stack([ds.generate(ds.window_hours(step * 3 + k)) for k in range(2)])
        loss = loss_fn(model(batch[:, :1]), batch[:, 1:])
        loss.backward()
        reducer.finish()
        opt.step()
        opt.zero_grad()
    # gather the final weights to rank 0
    if rank == 0:
        torch.save({k: v.detach().clone() for k, v in model.state_dict().items()}, result_path)


def test_config0_sp2_training_matches_single_rank(tmp_path):
    run(_train_worker, 1, 1, 3, str(tmp_path / "single.pt"))
    run(_train_worker, 2, 2, 3, str(tmp_path / "sp2.pt"))
    a = torch.load(tmp_path / "single.pt")
    b = torch.load(tmp_path / "sp2.pt")
    for k in a:
        assert torch.allclose(a[k], b[k], atol=1e-5, rtol=1e-4), k


def test_fused_collectives_not_available_without_cuda_group():
    """The symmetric-memory path is only taken for CUDA groups of 2..8 ranks; elsewhere the
    row-parallel linear falls back to GEMM + all-reduce mapping."""
    from neural_scaling_weather_b200.parallel import symm

    assert symm.available("tp") is False
    symm.disable("tp", "test")
    assert symm.available("tp") is False
    symm.reset()


# ----------------------------------------------------------------------------- data sharding
def _epoch_coverage_worker(rank, world, out_dir):
    import numpy as np
    import torch
    import torch.distributed as dist

    from neural_scaling_weather_b200.data.synthetic import SyntheticERA5
    from neural_scaling_weather_b200.parallel import comm

    comm.init_model_parallel_info(tp=1, sp1=1, sp2=1, dp=world)
    ds = SyntheticERA5(nlat=8, nlon=16, sfc_vars=["a"], pl_vars=[], levels=[], n_times=103, dt_scale=3,
                       invariants=[], micro_batch_size=1)
    for epoch in range(2):
        idx = torch.from_numpy(ds.epoch_indices(epoch).astype(np.int64))
        parts = [torch.zeros_like(idx) for _ in range(world)]
        dist.all_gather(parts, idx)
        if rank == 0:
            allidx = torch.cat(parts).numpy()
            # no sample twice in an epoch, every rank the same count, all of them valid starts
            assert len(np.unique(allidx)) == len(allidx) == world * ds.n_samples_shard
            assert allidx.min() >= 0 and allidx.max() < ds.n_samples_total
            # the union is the first world * shard entries of that epoch's global permutation
            perm = np.random.default_rng(ds.seed + epoch).permutation(ds.n_samples_total)
            assert np.array_equal(allidx, perm[:world * ds.n_samples_shard])
        # each window is temporal_context + rollout steps at the dataset's stride
        hrs = ds.window_hours(int(idx[0]))
        assert len(hrs) == ds.temporal_context_window + ds.num_rollout_steps
        assert np.all(np.diff(hrs) == 3)


@pytest.mark.parametrize("world", [2, 3])
def test_epoch_covers_every_sample_once_across_dp_ranks(tmp_path, world):
    """The DALI-epoch check of the reference (``tests/test_dali_es.py``) for the synthetic
    loader: one epoch over all dp ranks emits every sample window exactly once."""
    run(_epoch_coverage_worker, world, str(tmp_path))


def test_fused_halo_roll_not_available_on_cpu():
    """The peer-memory roll is only taken for CUDA tensors in an NCCL sp1 x sp2 group; CPU tensors use the
    portable exchange."""
    from neural_scaling_weather_b200.parallel import halo

    x = torch.zeros(1, 1, 8, 8, 16)
    assert halo.available(x, (-2, -3), (-3, -2), ("sp1", "sp2"), ([8], [8])) is False
    assert halo._norm(-4, 180) == -4 and halo._norm(176, 180) == -4 and halo._norm(9, 360) == 9
