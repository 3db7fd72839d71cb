"""torchrun worker: the fused GEMM + all-reduce (ops.linear_allreduce) against GEMM + NCCL.

Usage: ``torchrun --nproc-per-node N tests/mp_fused_tp_worker.py``.  Every rank holds its own
input / weight shards and the same bias and residual; the fused kernel's result must match the
NCCL all-reduce of the local GEMMs on every rank, over several launches of one shape (the
epoch-tagged flags are reused), two shapes, a CUDA-graph replay and the backward pass.
Prints FUSED_TP_OK on rank 0 and exits non-zero on a mismatch.
"""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from neural_scaling_weather_b200 import ops
    from neural_scaling_weather_b200.ops import _ext
    from neural_scaling_weather_b200.parallel import comm, symm

    comm.init_model_parallel_info(tp=world, sp1=1, sp2=1, dp=1)
    assert symm.available("tp"), "symmetric memory not available"
    ok = True
    for (M, N, K) in [(4100, 1024, 512), (777, 256, 128)]:
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn(M, K, device=dev, generator=g).bfloat16()
        w = torch.nn.Parameter(0.05 * torch.randn(N, K, device=dev, generator=g))
        gs = torch.Generator(device=dev).manual_seed(7)  # same on every rank
        b = torch.nn.Parameter(torch.randn(N, device=dev, generator=gs))
        res = torch.randn(M, N, device=dev, generator=gs).bfloat16()
        ref = x.float() @ w.detach().bfloat16().float().t()
        dist.all_reduce(ref)
        ref = ref + b.detach() + res.float()
        for it in range(4):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = ops.linear_allreduce(x, w, b, residual=res, group="tp")
            e = rel(y, ref)
            if e > 1e-2:
                print(f"[rank {rank}] M={M} launch {it}: mismatch {e}", flush=True)
                ok = False
        # CUDA graph: the epoch lives in device memory, so replays stay correct
        if M == 4100:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    ops.linear_allreduce(x, w, b, residual=res, group="tp")
            torch.cuda.current_stream().wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    yg = ops.linear_allreduce(x, w, b, residual=res, group="tp")
            for it in range(3):
                graph.replay()
                torch.cuda.synchronize()
                e = rel(yg, ref)
                if e > 1e-2:
                    print(f"[rank {rank}] graph replay {it}: mismatch {e}", flush=True)
                    ok = False
            del graph
        # backward: the all-reduce passes gradients through (row-parallel linear)
        xg = x.detach().float().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = ops.linear_allreduce(xg, w, b, residual=None, group="tp")
        dy = torch.randn(M, N, device=dev, generator=gs)
        (y.float() * dy).sum().backward()
        dx_ref = dy @ w.detach().bfloat16().float()
        dw_ref = dy.t() @ x.float()
        if rel(xg.grad, dx_ref) > 2e-2 or rel(w.grad, dw_ref) > 2e-2 or rel(b.grad, dy.sum(0)) > 2e-2:
            print(f"[rank {rank}] backward mismatch {rel(xg.grad, dx_ref)} {rel(w.grad, dw_ref)}", flush=True)
            ok = False
        # column-parallel linear of a replicated input: the data-gradient all-reduce runs in the
        # dgrad GEMM's epilogue; against the NCCL composition
        xr = torch.randn(M, N, device=dev, generator=gs).bfloat16()  # replicated input (K_in = N)
        wc = torch.nn.Parameter(0.05 * torch.randn(K, N, device=dev, generator=g))  # local column shard
        bc = torch.nn.Parameter(torch.randn(K, device=dev, generator=g))
        dyc = torch.randn(M, K, device=dev, generator=g)
        x1 = xr.detach().float().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            yc = ops.linear_colparallel(x1, wc, bc, activation="gelu", group="tp")
        (yc.float() * dyc).sum().backward()
        x2 = xr.detach().float().requires_grad_()
        from neural_scaling_weather_b200.parallel.mappings import identity_forward_allreduce_backward

        with torch.autocast("cuda", dtype=torch.bfloat16):
            yr = ops.linear(identity_forward_allreduce_backward(x2, "tp"), wc, bc, activation="gelu")
        (yr.float() * dyc).sum().backward()
        if rel(yc, yr) > 1e-3 or rel(x1.grad, x2.grad) > 1e-2:
            print(f"[rank {rank}] colparallel mismatch {rel(yc, yr)} {rel(x1.grad, x2.grad)}", flush=True)
            ok = False
    if _ext.require().read_error_flag(True) != 0:
        print(f"[rank {rank}] device error flag set", flush=True)
        ok = False
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    torch.cuda.synchronize()
    symm.reset()
    comm.reset()
    dist.destroy_process_group()
    if rank == 0:
        print("FUSED_TP_OK" if flag.item() == 0 else "FUSED_TP_FAIL", flush=True)
    sys.exit(0 if flag.item() == 0 else 1)


if __name__ == "__main__":
    main()
