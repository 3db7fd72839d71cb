"""torchrun worker: the fused data-parallel path against the NCCL reducer.

Usage: ``torchrun --nproc-per-node N tests/mp_dp_fused_worker.py``.  Every rank trains the same tiny
model twice from the same initialisation on rank-specific data (two micro-batches per step, clip
1.0, AdamW, bf16): once with ``FusedDPReducer`` (peer-memory reduce of each bucket's owned slice,
sharded AdamW that stores the new parameters into every rank, flag barrier) and once with the NCCL
bucket all-reduce and the full AdamW on every rank.  Parameters, losses and the checkpointed AdamW
moments must agree.  Prints DP_FUSED_OK.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import datetime  # noqa: E402
from contextlib import nullcontext  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    os.environ["NSW_FUSED_DP"] = "1"
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from neural_scaling_weather_b200 import config as C
    from neural_scaling_weather_b200.models import get_model
    from neural_scaling_weather_b200.ops import _ext
    from neural_scaling_weather_b200.parallel import comm, dp_fused
    from neural_scaling_weather_b200.parallel.grad_sync import GradReducer, order_params
    from neural_scaling_weather_b200.training.grad_norm import ShardedNorm
    from neural_scaling_weather_b200.training.optimizer import FlatParamSpace, FusedAdamW
    from neural_scaling_weather_b200.utils.misc import create_dummy_metadata

    comm.init_model_parallel_info(tp=1, sp1=1, sp2=1, dp=world)
    H, W, Cc = 32, 64, 5
    cfg = C.create(dict(
        model=dict(arch="swin", embed_dim=128, patch_size=2, depth=2, window_size=[4, 8], num_heads=2,
                   dropout=0.0, mlp_ratio=4, coord_pos_embed=True),
        data=dict(invariants=["a"]), train=dict(temporal_context_window=1, num_rollout_steps=1),
        parallelism=dict(use_transformer_engine=False)))
    md = create_dummy_metadata(H, W, Cc)

    def run(fused):
        torch.manual_seed(0)
        model = get_model(cfg, md).to(dev)
        params = [p for p in model.parameters() if p.requires_grad]
        space = FlatParamSpace(order_params(params), shadow_dtype=torch.bfloat16)
        if fused:
            ok, why = dp_fused.available(space, "adamw", False)
            assert ok, why
            reducer = dp_fused.FusedDPReducer(space, bucket_cap_mb=0.5)  # several buckets
        else:
            reducer = GradReducer(space, bucket_cap_mb=0.5)
        opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.01, space=space)
        if fused:
            opt.enable_dp_sharding(reducer)
        norms = ShardedNorm(space, owned=reducer.owned if fused else None)
        losses, grad_norms = [], []
        for step in range(4):
            for mb in range(2):
                g = torch.Generator().manual_seed(1000 * rank + 10 * step + mb)
                x = torch.randn(1, 1, Cc + 1, H, W, generator=g).to(dev)
                y = torch.randn(1, 1, Cc, H, W, generator=g).to(dev)
                with (reducer.no_sync() if mb == 0 else nullcontext()):
                    with torch.autocast("cuda", dtype=torch.bfloat16):
                        out = model(x)
                    loss = ((out.float() - y) ** 2).mean()
                    (loss / 2).backward()
                losses.append(float(loss))
            reducer.finish()
            norm = norms.norm("grad")
            opt.grad_scale = ShardedNorm.clip_coef(norm, 1.0)
            grad_norms.append(float(norm))
            opt.step()
            opt.zero_grad()
        torch.cuda.synchronize()
        sd = opt.state_dict()
        m = torch.cat([sd["state"][i]["exp_avg"].flatten() for i in sorted(sd["state"])])
        return space.data.clone(), space.shadow.clone(), losses, grad_norms, m

    p_f, s_f, l_f, n_f, m_f = run(True)
    p_n, s_n, l_n, n_n, m_n = run(False)
    assert _ext.require().read_error_flag(True) == 0
    rel = ((p_f - p_n).norm() / p_n.norm()).item()
    assert rel < 1e-5, rel
    assert torch.equal(s_f, p_f.to(torch.bfloat16)), "shadow not in sync with the parameters"
    for a, b in zip(n_f, n_n):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(b)), (n_f, n_n)
    for a, b in zip(l_f, l_n):
        assert abs(a - b) <= 1e-4 * max(1.0, abs(b)), (l_f, l_n)
    assert ((m_f - m_n).norm() / m_n.norm()).item() < 1e-5
    # every rank holds the same parameters
    ref = p_f.clone()
    dist.broadcast(ref, src=0)
    assert torch.equal(ref, p_f), "ranks diverged"
    dist.barrier()
    if rank == 0:
        print(f"DP_FUSED_OK rel={rel:.2e}")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
