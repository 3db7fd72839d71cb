"""Peer-to-peer bandwidth between the GPUs of one node through symmetric memory.

``python -m torch.distributed.run --nproc-per-node 2 benchmarks/p2p_bandwidth.py [--mb 133]``

Every rank allocates a symmetric buffer, then copies its next peer's buffer into local memory
(``pull``) and its local buffer into the next peer's buffer (``push``), all ranks at once, with
``Tensor.copy_`` on a view of the peer's memory.  Times are CUDA events around several copies, the
maximum over ranks; the bandwidth is per direction of one GPU's links.  The all-reduce kernels of
this repository move their partial tiles over the same mappings, so this is their link ceiling.
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
    ap.add_argument("--mb", type=float, default=132.7, help="bytes per copy, in MB (default: 64800 x 1024 bf16)")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import torch.distributed._symmetric_memory as symm

    n = int(a.mb * 1e6) // 2
    buf = symm.empty(n, dtype=torch.bfloat16, device=dev)
    buf.normal_()
    h = symm.rendezvous(buf, dist.group.WORLD)
    peer = (rank + 1) % world
    remote = h.get_buffer(peer, (n,), torch.bfloat16)
    mine = torch.empty(n, dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    dist.barrier()
    out = {}
    for name, fn in (("pull", lambda: mine.copy_(remote)), ("push", lambda: remote.copy_(mine)),
                     ("local", lambda: mine.copy_(buf))):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        out[name] = {"ms": round(ms.item(), 4), "gbs": round(2 * n / (ms.item() * 1e-3) / 1e9, 1)}
    if rank == 0:
        print(json.dumps({"op": "peer copy through symmetric memory", "world": world, "bytes": 2 * n, **out}))
    del remote, h
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
