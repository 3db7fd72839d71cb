"""Sharded metrics and losses against one rank, and the window partition round trip (CPU, gloo).

Counterparts of the reference's ``tests/test_metrics.py`` (weighted RMSE under dp x sp1 x sp2 against a
single rank) and ``tests/test_windows.py`` (window partition -> reverse, locally and on the gathered
field).
"""

import pytest
import torch

from tests.dist_utils import run


def _metrics_worker(rank, world, dp, sp1, sp2):
    import numpy as np
    import torch
    import torch.distributed as dist

    from neural_scaling_weather_b200.losses import WeightedLoss, WeightedMSE, WeightedRMSE
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.helpers import compute_split_shapes, offsets
    from neural_scaling_weather_b200.utils.misc import build_spherical_area_weights

    B, T, C, H, W = 4, 1, 3, 12, 20
    g = torch.Generator().manual_seed(3)
    pred = torch.randn(B, T, C, H, W, dtype=torch.float64, generator=g)
    targ = torch.randn(B, T, C, H, W, dtype=torch.float64, generator=g)
    aw = torch.as_tensor(build_spherical_area_weights(np.linspace(90, -90, H + 1)[:-1]))[:, None]
    # single-rank oracle: before the groups exist every getter reports size 1
    p = pred.clone().requires_grad_()
    rmse_ref = WeightedRMSE(weights=aw)(p, targ)
    mse_ref = WeightedMSE(weights=aw)(p, targ)
    loss_ref = WeightedLoss(area_weighting=True, weights=aw)(p, targ)
    loss_ref.backward()

    comm.init_model_parallel_info(tp=1, sp1=sp1, sp2=sp2, dp=dp)
    hs, ws = compute_split_shapes(H, sp1), compute_split_shapes(W, sp2)
    r1, r2, rd = comm.get_rank("sp1"), comm.get_rank("sp2"), comm.get_rank("dp")
    h0, w0, b0 = offsets(hs)[r1], offsets(ws)[r2], rd * (B // dp)
    sl = (slice(b0, b0 + B // dp), slice(None), slice(None), slice(h0, h0 + hs[r1]), slice(w0, w0 + ws[r2]))
    awl = aw[h0:h0 + hs[r1]]
    pl = pred[sl].clone().requires_grad_()
    rmse = WeightedRMSE(weights=awl)(pl, targ[sl])
    mse = WeightedMSE(weights=awl)(pl, targ[sl])
    loss = WeightedLoss(area_weighting=True, weights=awl)(pl, targ[sl])
    loss.backward()

    def dp_mean(v):
        v = v.detach().clone()
        if dp > 1:
            dist.all_reduce(v, group=comm.get_group("dp"))
            v /= dp
        return v

    # RMSE is averaged over the batch after the square root: per-rank means over equal dp shards
    # the per-channel sums accumulate in fp32 in a shard-dependent order: agreement to fp32 rounding
    assert torch.allclose(dp_mean(rmse), rmse_ref, rtol=1e-6), (rank, rmse, rmse_ref)
    assert torch.allclose(dp_mean(mse), mse_ref, rtol=1e-6), (rank, mse, mse_ref)
    assert torch.allclose(dp_mean(loss), loss_ref.detach(), rtol=1e-6)
    # the local loss is a mean over the local batch: its gradient is dp times the global one
    assert torch.allclose(pl.grad / dp, p.grad[sl], rtol=1e-6, atol=1e-12)


@pytest.mark.parametrize("dp,sp1,sp2", [(1, 2, 1), (1, 1, 2), (2, 1, 2), (1, 2, 2)])
def test_weighted_metrics_sharded_match_single_rank(dp, sp1, sp2):
    """Weighted RMSE, MSE and the training loss (value and gradient) with the batch over dp and an uneven
    grid split over sp1 x sp2 equal the single-rank result."""
    run(_metrics_worker, dp * sp1 * sp2, dp, sp1, sp2)


def test_window_partition_round_trip_and_sharding():
    """Window partition then reverse is the identity; the windows of a shard whose extents the window
    divides are exactly the gathered field's windows over that shard's area."""
    from neural_scaling_weather_b200.ops.reference import window_partition, window_reverse

    B, T, H, W, C = 2, 2, 12, 24, 5
    win = (3, 6)
    x = torch.randn(B, T, H, W, C)
    w = window_partition(x, win)
    assert w.shape == (B * (H // 3) * (W // 6), T * 3 * 6, C)
    assert torch.equal(window_reverse(w, win, B, T, H, W), x)
    # two longitude shards of 12 columns (each divisible by the window width)
    full = w.view(B, H // 3, W // 6, T * 18, C)
    for k in range(2):
        shard = x[:, :, :, 12 * k:12 * (k + 1)]
        ws = window_partition(shard, win).view(B, H // 3, 2, T * 18, C)
        assert torch.equal(ws, full[:, :, 2 * k:2 * (k + 1)])
    # a rolled field partitions into the rolled windows (shifted-window attention's layout)
    xr = torch.roll(x, shifts=(-1, -3), dims=(2, 3))
    assert torch.equal(window_reverse(window_partition(xr, win), win, B, T, H, W), xr)
