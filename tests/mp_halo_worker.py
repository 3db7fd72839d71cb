"""torchrun worker: the peer-memory sharded roll (parallel.halo) against ``torch.roll`` of the full field.

Usage: ``torchrun --nproc-per-node N tests/mp_halo_worker.py`` (N = 2: sp1 x sp2 = 1 x 2 and 2 x 1;
N = 4: 2 x 2 as well).  Every rank builds the same global (B, T, H, W, C) field, keeps its shard,
rolls it and compares with its shard of ``torch.roll`` of the global field (exact: a roll is a copy),
for both shift signs, uneven shards, many launches in a row (the epoch flags and band buffers are
reused), a CUDA-graph replay and the autograd mapping's backward (the reverse roll).  Then times the
fused roll against the NCCL roll at the production shard (180 x 180 patches, C = 1024, bf16).
Prints HALO_OK on rank 0 and exits non-zero on a mismatch.
"""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def shard(x, comm, shapes):
    from neural_scaling_weather_b200.parallel.helpers import offsets

    i1, i2 = comm.get_rank("sp1"), comm.get_rank("sp2")
    h0, w0 = offsets(shapes[0])[i1], offsets(shapes[1])[i2]
    return x[:, :, h0:h0 + shapes[0][i1], w0:w0 + shapes[1][i2]].contiguous()


def split(n, parts):
    base, rem = divmod(n, parts)
    return [base + (1 if i < rem else 0) for i in range(parts)]


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from neural_scaling_weather_b200.ops import _ext
    from neural_scaling_weather_b200.parallel import comm, halo
    from neural_scaling_weather_b200.parallel.helpers import _distributed_roll
    from neural_scaling_weather_b200.parallel.mappings import roll_forward_reverseroll_backward

    layouts = [(1, world), (world, 1)] + ([(2, world // 2)] if world == 4 else [])
    ok = True
    for sp1, sp2 in layouts:
        comm.reset()
        halo.reset()
        comm.init_model_parallel_info(tp=1, sp1=sp1, sp2=sp2, dp=world // (sp1 * sp2))
        for (H, W, C, dtype) in [(16, 24, 64, torch.bfloat16), (18, 25, 32, torch.float32)]:
            shapes = (split(H, sp1), split(W, sp2))
            g = torch.Generator(device=dev).manual_seed(5)  # the same global field on every rank
            xg = torch.randn(2, 1, H, W, C, device=dev, generator=g).to(dtype)
            xl = shard(xg, comm, shapes)
            for shifts in [(-4, -9), (4, 9), (0, -9), (-4, 0), (3, -5), (-5, 11)]:
                if not halo.available(xl, shifts, (-3, -2), ("sp1", "sp2"), shapes):
                    if (sp1 == 1 or abs(shifts[0]) < min(shapes[0])) and (sp2 == 1 or abs(shifts[1]) < min(shapes[1])):
                        print(f"[rank {rank}] fused roll unexpectedly unavailable for {shifts} {shapes}", flush=True)
                        ok = False
                    continue
                ref = shard(torch.roll(xg, shifts, dims=(2, 3)), comm, shapes)
                for it in range(3):
                    out = halo.roll(xl, shifts, shapes)
                    if not torch.equal(out, ref):
                        print(f"[rank {rank}] sp={sp1}x{sp2} {H}x{W} shift {shifts} launch {it}: mismatch "
                              f"{(out.float() - ref.float()).abs().max().item()}", flush=True)
                        ok = False
            # autograd mapping: forward roll, backward reverse roll
            shifts = (-4, -9) if min(shapes[0]) > 4 or sp1 == 1 else (-2, -9)
            if halo.available(xl, shifts, (-3, -2), ("sp1", "sp2"), shapes):
                xa = xl.clone().requires_grad_(True)
                y = roll_forward_reverseroll_backward(xa, shifts, (-3, -2), ["sp1", "sp2"], shapes=shapes)
                gy = shard(torch.roll(xg, (1, 2), dims=(2, 3)), comm, shapes)  # any field
                y.backward(gy)
                gref = shard(torch.roll(torch.roll(xg, (1, 2), dims=(2, 3)), tuple(-s for s in shifts), dims=(2, 3)),
                             comm, shapes)
                if not torch.equal(xa.grad, gref):
                    print(f"[rank {rank}] sp={sp1}x{sp2} backward mismatch", flush=True)
                    ok = False
        # CUDA graph: two rolls of opposite sign captured once and replayed
        H, W, C = 16, 24, 64
        shapes = (split(H, sp1), split(W, sp2))
        g = torch.Generator(device=dev).manual_seed(9)
        xg = torch.randn(1, 1, H, W, C, device=dev, generator=g).bfloat16()
        static = shard(xg, comm, shapes)
        sh = (-2, -3)
        halo.roll(static, sh, shapes)  # buffers exist before capture
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                a = halo.roll(static, sh, shapes)
                b = halo.roll(a, (-sh[0], -sh[1]), shapes)
        torch.cuda.current_stream().wait_stream(s)
        for it in range(5):
            xg = torch.randn(1, 1, H, W, C, device=dev, generator=g).bfloat16()
            static.copy_(shard(xg, comm, shapes))
            graph.replay()
            torch.cuda.synchronize()
            if not (torch.equal(a, shard(torch.roll(xg, sh, dims=(2, 3)), comm, shapes)) and torch.equal(b, static)):
                print(f"[rank {rank}] sp={sp1}x{sp2} graph replay {it}: mismatch", flush=True)
                ok = False
        del graph
        torch.cuda.synchronize()
        dist.barrier()

    # timing at the production shard: fused vs NCCL roll (device-timed, max over ranks)
    comm.reset()
    halo.reset()
    comm.init_model_parallel_info(tp=1, sp1=1, sp2=world, dp=1)
    shapes = ([180], split(360, world))
    x = torch.randn(1, 1, 180, shapes[1][0], 1024, device=dev).bfloat16()
    shifts = (-4, -9)

    def fused():
        return halo.roll(x, shifts, shapes)

    def nccl():
        y = _distributed_roll(x, shifts[0], 2, "sp1", shapes[0])
        return _distributed_roll(y, shifts[1], 3, "sp2", shapes[1])

    res = {}
    for name, fn in (("fused", fused), ("nccl", nccl)):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(50):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 50 * 1000.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = t.item()
    if not torch.equal(fused(), nccl()):
        print(f"[rank {rank}] fused and NCCL rolls differ at the production shape", flush=True)
        ok = False
    err = _ext.require().read_error_flag(True)
    if err != 0:
        print(f"[rank {rank}] device error word {err}", flush=True)
        ok = False
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        mb = x.numel() * x.element_size() / 1e6
        print(f"roll of a {tuple(x.shape)} bf16 shard ({mb:.1f} MB), sp2={world}: fused {res['fused']:.1f} us, "
              f"NCCL {res['nccl']:.1f} us", flush=True)
        if flag.item() == 1:
            print("HALO_OK", flush=True)
    halo.reset()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
