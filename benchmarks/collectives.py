"""Timing of the fused tensor-parallel GEMM + all-reduce against GEMM then NCCL all-reduce.

``python -m torch.distributed.run --nproc-per-node N benchmarks/collectives.py``
(N = 2..8 GPUs of one node).  Shape: a row-parallel projection of the Swin p4-e1024 block
(64800 tokens, 1024 outputs, 1024 / N inputs per rank) with bias and residual.  Times are CUDA
events on each rank around several launches, reported as the maximum over ranks; the roofline
is the slower of the GEMM at the measured bf16 rate and the bytes that cross a rank's NVLink in one
direction (its (N - 1) 16-bit partials pushed to the peers) at 770 GB/s.  By default the launches
are replayed from one CUDA graph, so the figures are device time without host launch gaps
(``--graph 0``: eager launches).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=64800)
    ap.add_argument("--N", type=int, default=1024)
    ap.add_argument("--K", type=int, default=1024, help="full input width (split over the ranks)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--graph", type=int, default=1, help="1: time the launches replayed from a CUDA graph")
    a = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from neural_scaling_weather_b200.ops import _ext, linear_allreduce
    from neural_scaling_weather_b200.parallel import comm, symm

    comm.init_model_parallel_info(tp=world, sp1=1, sp2=1, dp=1)
    ext = _ext.require()
    M, N, K = a.M, a.N, a.K // world
    x = torch.randn(M, K, device=dev).bfloat16()
    w = torch.nn.Parameter(0.02 * torch.randn(N, K, device=dev))
    b = torch.nn.Parameter(torch.zeros(N, device=dev))
    res = torch.randn(M, N, device=dev).bfloat16()
    wb = w.detach().bfloat16()

    def fused():
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            return linear_allreduce(x, w, b, residual=res, group="tp")

    def baseline():
        y = ext.gemm(x, wb)
        dist.all_reduce(y, group=comm.get_group("tp"))
        return y + b.detach().bfloat16() + res

    def gemm_only():  # the local GEMM with the same epilogue, no reduction: the compute part alone
        return ext.gemm(x, wb, b.detach(), res)

    out = {}
    for name, fn in (("fused", fused), ("gemm_then_nccl", baseline), ("gemm_only", gemm_only)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        run = lambda: [fn() for _ in range(a.iters)]  # noqa: E731
        if a.graph:  # the launches replay from one CUDA graph: device time, no host launch gaps
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    run()
            torch.cuda.current_stream().wait_stream(s)
            g.replay()
            torch.cuda.synchronize()
            dist.barrier()
            run = g.replay
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        out[name] = round(ms.item(), 4)
        if a.graph:
            del g
            torch.cuda.synchronize()
    assert ext.read_error_flag(True) == 0
    flops = 2.0 * M * N * K
    peer_bytes = (world - 1) * M * N * 2
    roof_ms = max(flops / 1649.8e12, peer_bytes / 770e9) * 1e3
    if rank == 0:
        print(json.dumps({"op": "row-parallel linear + all-reduce", "world": world, "M": M, "N": N, "K_per_rank": K,
                          "fused_ms": out["fused"], "gemm_then_nccl_ms": out["gemm_then_nccl"],
                          "gemm_only_ms": out["gemm_only"], "graph": bool(a.graph),
                          "roofline_ms": round(roof_ms, 4), "fused_of_roofline": round(roof_ms / out["fused"], 3)}))
    symm.reset()
    comm.reset()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
