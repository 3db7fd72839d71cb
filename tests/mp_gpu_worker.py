"""torchrun worker: sharded model on GPUs (NCCL) against the single-GPU result.

Usage: ``torchrun --nproc-per-node N tests/mp_gpu_worker.py <tp> <sp1> <sp2>``.  Every rank
builds the same full model on its GPU, runs it unsharded (groups absent), then shards the
weights by ``comm_metadata``, runs the distributed forward/backward with the fused kernels
and compares outputs and gathered gradients.  Exits non-zero on mismatch.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import datetime  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    tp, sp1, sp2 = (int(a) for a in sys.argv[1:4])
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.losses import WeightedLoss
    from neural_scaling_weather_b200.models import get_model
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.parallel.grad_sync import GradReducer, order_params
    from neural_scaling_weather_b200.parallel.helpers import (
        _gather,
        compute_split_shapes,
        compute_split_shapes_for_patching,
        offsets,
    )
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace
    from neural_scaling_weather_b200.utils.misc import create_dummy_metadata, split_dummy_metadata

    dev = torch.device("cuda", local)
    H, W, Cc, p = 36, 144, 6, 2
    dp = world // (tp * sp1 * sp2)
    cfg = C.create(dict(
        model=dict(arch="swin", embed_dim=128, patch_size=p, depth=2, window_size=[9, 18], num_heads=4,
                   dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=["a"]), train=dict(temporal_context_window=1, num_rollout_steps=1),
        parallelism=dict(use_transformer_engine=False)))
    torch.manual_seed(0)
    md_full = create_dummy_metadata(H, W, Cc)
    md_full["area_weights"] = torch.rand(H, 1)
    x = torch.randn(2 * dp, 1, Cc + 1, H, W)
    y = torch.randn(2 * dp, 1, Cc, H, W)
    ref = get_model(cfg, md_full).to(dev)
    loss_ref = WeightedLoss(area_weighting=True, weights=md_full["area_weights"]).to(dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out_ref = ref(x.to(dev))
        l_ref = loss_ref(out_ref.float(), y.to(dev))
    l_ref.backward()

    comm.init_model_parallel_info(tp=tp, sp1=sp1, sp2=sp2, dp=dp)
    s1 = compute_split_shapes_for_patching(H, sp1, p)
    s2 = compute_split_shapes_for_patching(W, sp2, p)
    md = split_dummy_metadata(md_full, s1, s2)
    md["area_weights"] = md_full["area_weights"][md["sp_slices"][0]]
    model = get_model(cfg, md).to(dev)
    full = dict(ref.named_parameters())
    with torch.no_grad():
        for name, prm in model.named_parameters():
            src = full[name].detach()
            for dim, grp in enumerate(prm.comm_metadata["sharded"]):
                if grp is None or comm.get_size(grp) == 1:
                    continue
                shapes = compute_split_shapes(src.shape[dim], comm.get_size(grp))
                src = src.narrow(dim, offsets(shapes)[comm.get_rank(grp)], shapes[comm.get_rank(grp)])
            prm.copy_(src)
    space = FlatParamSpace(order_params(list(model.parameters())))
    reducer = GradReducer(space, broadcast_from_root=False)
    r1, r2, rd = comm.get_rank("sp1"), comm.get_rank("sp2"), comm.get_rank("dp")
    o1, o2 = offsets(s1)[r1], offsets(s2)[r2]
    xl = x[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]].to(dev)
    yl = y[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]].to(dev)
    loss_fn = WeightedLoss(area_weighting=True, weights=md["area_weights"]).to(dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(xl)
        loss = loss_fn(out.float(), yl)
    loss.backward()
    reducer.finish()
    torch.cuda.synchronize()
    ok = True
    want = out_ref[2 * rd:2 * rd + 2, :, :, o1:o1 + s1[r1], o2:o2 + s2[r2]].float()
    err = ((out.float() - want).norm() / want.norm()).item()
    if err > 3e-2:
        print(f"[rank {rank}] output mismatch {err}", flush=True)
        ok = False
    for name, prm in model.named_parameters():
        g = prm.grad
        for dim, grp in enumerate(prm.comm_metadata["sharded"]):
            if grp is not None and comm.get_size(grp) > 1:
                g = _gather(g.contiguous(), dim, None, grp)
        gr = full[name].grad
        e = ((g - gr).norm() / gr.norm().clamp_min(1e-12)).item()
        if e > 8e-2:
            print(f"[rank {rank}] grad mismatch {name} {e}", flush=True)
            ok = False
    from neural_scaling_weather_b200.ops import _ext

    if _ext.require().read_error_flag(True) != 0:
        ok = False
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    comm.reset()
    dist.destroy_process_group()
    if rank == 0:
        print("MULTIGPU_OK" if flag.item() == 0 else "MULTIGPU_FAIL", flush=True)
    sys.exit(0 if flag.item() == 0 else 1)


if __name__ == "__main__":
    main()
