"""Shard-shape arithmetic and the collective primitives built on torch.distributed.

Reference behaviour (``distributed/helpers.py``):

* ``compute_split_shapes(size, n)`` (``:31-46``): balanced uneven split, div-up first and
  floor when the last shard would be empty.
* ``compute_split_shapes_for_patching(size, n, p)`` (``:54-66``): split in patch units,
  then give the leftover pixels to the last shard (721 rows in 4 parts at p=4 ->
  180, 180, 180, 181).
* ``_reduce/_split/_gather/_reduce_scatter`` (``:69-182``), a cyclic roll of a tensor
  sharded along one dimension (``:192-277``) and an all-to-all re-shard (``:279-297``).
* ``init_params_for_shared_weights`` (``:6-27``).

The distributed roll here is written as a general interval exchange: each rank computes
which slice of every peer's shard lands in its output after the global cyclic shift and
posts one send/receive per overlapping peer (``batch_isend_irecv``).  For the shifts the
model uses (smaller than every shard) this is exactly one slab to one neighbour, as in the
reference; unlike the reference it stays correct when a shift spans several shards.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import comm


# ---------------------------------------------------------------------------
# shapes


def compute_split_shapes(size: int, num_chunks: int) -> List[int]:
    if num_chunks == 1:
        return [size]
    chunk = (size + num_chunks - 1) // num_chunks
    last = size - chunk * (num_chunks - 1)
    if last <= 0:
        chunk = size // num_chunks
        last = size - chunk * (num_chunks - 1)
    return [chunk] * (num_chunks - 1) + [last]


def compute_split_shapes_for_patching(size: int, num_chunks: int, patch_size: int) -> List[int]:
    shapes = compute_split_shapes(size // patch_size, num_chunks)
    if patch_size == 1:
        return shapes
    shapes = [s * patch_size for s in shapes]
    shapes[-1] += size % patch_size
    return shapes


def split_tensor_along_dim(tensor: torch.Tensor, dim: int, num_chunks: int,
                           sections: Optional[Sequence[int]] = None):
    if dim < 0:
        dim += tensor.dim()
    if dim >= tensor.dim():
        raise ValueError(f"cannot split along dim {dim} of a {tensor.dim()}-d tensor")
    if tensor.shape[dim] < num_chunks:
        raise ValueError(f"cannot split dim {dim} of size {tensor.shape[dim]} into {num_chunks}")
    if sections is None:
        sections = compute_split_shapes(tensor.shape[dim], num_chunks)
    return list(torch.split(tensor, list(sections), dim=dim))


def offsets(shapes: Sequence[int]) -> List[int]:
    out, acc = [], 0
    for s in shapes:
        out.append(acc)
        acc += s
    return out


# ---------------------------------------------------------------------------
# primitives


def _reduce(x: torch.Tensor, comm_name: str) -> torch.Tensor:
    if comm.get_size(comm_name) == 1:
        return x
    x = x.contiguous()
    dist.all_reduce(x, group=comm.get_group(comm_name))
    return x


def _split(x: torch.Tensor, dim: int, comm_name: str, sections=None) -> torch.Tensor:
    n = comm.get_size(comm_name)
    if n == 1:
        return x
    parts = split_tensor_along_dim(x, dim, n, sections)
    return parts[comm.get_rank(comm_name)].contiguous()


def _gather(x: torch.Tensor, dim: int, shapes, comm_name: str) -> torch.Tensor:
    n = comm.get_size(comm_name)
    if shapes is not None and len(shapes) != n:
        raise ValueError(f"expected {n} shard shapes, got {len(shapes)}")
    if dim < 0:
        dim += x.dim()
    if dim >= x.dim():
        raise ValueError(f"cannot gather along dim {dim} of a {x.dim()}-d tensor")
    if n == 1:
        return x
    x = x.contiguous()
    shape = list(x.shape)
    bufs = []
    for r in range(n):
        if shapes is not None:
            shape[dim] = shapes[r]
        bufs.append(torch.empty(shape, dtype=x.dtype, device=x.device))
    if shapes is None or len(set(shapes)) == 1 or x.device.type == "cuda":
        dist.all_gather(bufs, x, group=comm.get_group(comm_name))
    else:
        # gloo's all_gather needs equal sizes: pad to the largest shard
        mx = max(shapes)
        pshape = list(x.shape)
        pshape[dim] = mx
        padded = torch.zeros(pshape, dtype=x.dtype, device=x.device)
        padded.narrow(dim, 0, x.shape[dim]).copy_(x)
        pbufs = [torch.empty_like(padded) for _ in range(n)]
        dist.all_gather(pbufs, padded, group=comm.get_group(comm_name))
        bufs = [b.narrow(dim, 0, shapes[r]) for r, b in enumerate(pbufs)]
    return torch.cat(bufs, dim=dim).contiguous()


def _reduce_scatter(x: torch.Tensor, dim: int, shapes, comm_name: str) -> torch.Tensor:
    n = comm.get_size(comm_name)
    if dim < 0:
        dim += x.dim()
    if n == 1:
        return x
    parts = [p.contiguous() for p in split_tensor_along_dim(x.contiguous(), dim, n, shapes)]
    me = comm.get_rank(comm_name)
    if x.device.type == "cuda" and (shapes is None or len(set(shapes)) == 1):
        out = torch.empty_like(parts[me])
        dist.reduce_scatter(out, parts, group=comm.get_group(comm_name))
        return out
    # portable path (gloo / uneven): all-reduce then keep the local slice
    full = x.contiguous().clone()
    dist.all_reduce(full, group=comm.get_group(comm_name))
    return split_tensor_along_dim(full, dim, n, shapes)[me].contiguous()


def _distributed_roll(x: torch.Tensor, shift: int, shift_dim: int, comm_name: str,
                      shapes: Optional[Sequence[int]] = None) -> torch.Tensor:
    """Cyclic roll by ``shift`` of a tensor sharded along ``shift_dim`` over ``comm_name``.

    ``shapes`` are the per-rank extents along ``shift_dim``; when omitted they are
    exchanged once with an all-gather of the local extent.
    """
    if shift_dim < 0:
        shift_dim += x.dim()
    n = comm.get_size(comm_name)
    if n == 1:
        return torch.roll(x, shifts=(shift,), dims=(shift_dim,))
    if shift == 0:
        return x
    me = comm.get_rank(comm_name)
    group = comm.get_group(comm_name)
    if shapes is None:
        t = torch.tensor([x.shape[shift_dim]], dtype=torch.int64,
                         device=x.device if x.device.type == "cuda" else "cpu")
        lst = [torch.zeros_like(t) for _ in range(n)]
        dist.all_gather(lst, t, group=group)
        shapes = [int(v.item()) for v in lst]
    total = sum(shapes)
    starts = offsets(shapes)
    s = shift % total
    grank = comm.get_group_ranks(comm_name)

    def pieces(dst: int):
        """(src_rank, src_lo, dst_lo, length) covering rank dst's output after the shift."""
        out = []
        a, b = starts[dst], starts[dst] + shapes[dst]
        pos = a
        while pos < b:
            src_g = (pos - s) % total
            # owner of global index src_g
            r = max(i for i in range(n) if starts[i] <= src_g)
            run = min(b - pos, starts[r] + shapes[r] - src_g)
            out.append((r, src_g - starts[r], pos - a, run))
            pos += run
        return out

    x = x.contiguous()
    out = torch.empty_like(x)
    ops = []
    recv_bufs = []
    # what I receive
    for (src, src_lo, dst_lo, ln) in pieces(me):
        if src == me:
            out.narrow(shift_dim, dst_lo, ln).copy_(x.narrow(shift_dim, src_lo, ln))
        else:
            buf = torch.empty_like(out.narrow(shift_dim, dst_lo, ln)).contiguous()
            recv_bufs.append((buf, dst_lo, ln))
            ops.append(dist.P2POp(dist.irecv, buf, grank[src], group=group))
    # what I send
    send_keep = []
    for dst in range(n):
        if dst == me:
            continue
        for (src, src_lo, dst_lo, ln) in pieces(dst):
            if src == me:
                piece = x.narrow(shift_dim, src_lo, ln).contiguous()
                send_keep.append(piece)
                ops.append(dist.P2POp(dist.isend, piece, grank[dst], group=group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    for buf, dst_lo, ln in recv_bufs:
        out.narrow(shift_dim, dst_lo, ln).copy_(buf)
    return out


def _transpose(x: torch.Tensor, dim0: int, dim1: int, dim0_split_sizes, dim1_split_sizes,
               comm_name: str) -> torch.Tensor:
    """All-to-all re-shard: split ``dim0`` across the group, gather ``dim1``."""
    n = comm.get_size(comm_name)
    me = comm.get_rank(comm_name)
    send = [p.contiguous() for p in split_tensor_along_dim(x, dim0, n, dim0_split_sizes)]
    shape = list(send[me].shape)
    recv = []
    for ln in dim1_split_sizes:
        shape[dim1] = ln
        recv.append(torch.empty(shape, dtype=x.dtype, device=x.device))
    if n == 1:
        return x
    dist.all_to_all(recv, send, group=comm.get_group(comm_name))
    return torch.cat(recv, dim=dim1)


def init_params_for_shared_weights(model) -> None:
    """Broadcast every parameter from the root of each group it is ``shared`` in."""
    with torch.no_grad():
        for p in model.parameters():
            if not hasattr(p, "comm_metadata"):
                p.comm_metadata = {"sharded": [], "shared": ["tp-sp1-sp2"], "reduce": []}
            for g in p.comm_metadata["shared"]:
                if comm.get_size(g) > 1:
                    dist.broadcast(p.data, src=comm.get_root(g), group=comm.get_group(g))
