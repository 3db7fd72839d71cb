"""Run a function on N CPU processes with the gloo backend (multi-rank tests without GPUs)."""

import os
import sys
import traceback

import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _entry(rank, world, port, fn, args, errq):
    try:
        if ROOT not in sys.path:
            sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["RANK"] = str(rank)
        os.environ["WORLD_SIZE"] = str(world)
        os.environ["LOCAL_RANK"] = str(rank)
        import torch
        import torch.distributed as dist

        torch.set_num_threads(1)
        # the parent holds the rendezvous store on this port (bound before any rank started)
        store = dist.TCPStore("127.0.0.1", port, world_size=world + 1, is_master=False)
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world)
        try:
            fn(rank, world, *args)
        finally:
            from neural_scaling_weather_b200.parallel import comm

            comm.reset()
            dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise


def run(fn, world: int, *args, timeout: float = 600):
    import torch.distributed as dist

    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    # the parent binds the rendezvous store on an OS-chosen port and keeps it for the run, so no
    # other process can take the port between choosing it and the ranks' rendezvous
    store = dist.TCPStore("127.0.0.1", 0, world_size=world + 1, is_master=True, wait_for_workers=False)
    port = store.port
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    if errors:
        raise AssertionError("worker failure:\n" + "\n".join(f"[rank {r}] {tb}" for r, tb in errors))
    if alive:
        raise AssertionError(f"{len(alive)} workers timed out")
    del store
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"worker exit codes {bad}")
