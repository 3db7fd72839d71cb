"""Autograd-aware collectives (forward/backward pairs) for model parallelism.

Same pairs as ``distributed/mappings.py:24-214`` of the reference:

=============================================  ===================  =====================
wrapper                                        forward              backward
=============================================  ===================  =====================
``identity_forward_allreduce_backward``        identity             all-reduce
``allreduce_forward_identity_backward``        all-reduce           identity
``allgather_forward_split_backward``           all-gather           split
``split_forward_allgather_backward``           split                all-gather
``reducescatter_forward_allgather_backward``   reduce-scatter       all-gather
``allgather_forward_reducescatter_backward``   all-gather           reduce-scatter
``roll_forward_reverseroll_backward``          distributed roll     reverse roll
``transpose_forward_transpose_backward``       all-to-all           inverse all-to-all
=============================================  ===================  =====================

Each wrapper opens a profiler range with the reference's range name.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from ..utils.profiler import profile
from .helpers import _distributed_roll, _gather, _reduce, _reduce_scatter, _split, _transpose


class _IdentityFwdAllReduceBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm_name):
        ctx.comm_name = comm_name
        return x

    @staticmethod
    def backward(ctx, g):
        return _reduce(g.clone(), ctx.comm_name), None


class _AllReduceFwdIdentityBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm_name):
        return _reduce(x.clone(), comm_name)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _AllGatherFwdSplitBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, shapes, comm_name):
        ctx.args = (dim, shapes, comm_name)
        return _gather(x, dim, shapes, comm_name)

    @staticmethod
    def backward(ctx, g):
        dim, shapes, comm_name = ctx.args
        return _split(g, dim, comm_name, shapes), None, None, None


class _SplitFwdAllGatherBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, shapes, comm_name):
        ctx.args = (dim, shapes, comm_name)
        return _split(x, dim, comm_name, shapes)

    @staticmethod
    def backward(ctx, g):
        dim, shapes, comm_name = ctx.args
        return _gather(g, dim, shapes, comm_name), None, None, None


class _ReduceScatterFwdAllGatherBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, shapes, comm_name):
        ctx.args = (dim, shapes, comm_name)
        return _reduce_scatter(x, dim, shapes, comm_name)

    @staticmethod
    def backward(ctx, g):
        dim, shapes, comm_name = ctx.args
        return _gather(g, dim, shapes, comm_name), None, None, None


class _AllGatherFwdReduceScatterBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, shapes, comm_name):
        ctx.args = (dim, shapes, comm_name)
        return _gather(x, dim, shapes, comm_name)

    @staticmethod
    def backward(ctx, g):
        dim, shapes, comm_name = ctx.args
        return _reduce_scatter(g, dim, shapes, comm_name), None, None, None


class _RollFwdReverseRollBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, shifts, dims, comm_names, shapes):
        if not (len(shifts) == len(dims) == len(comm_names)):
            raise ValueError("shifts, dims and comm_names must have equal length")
        ctx.args = (shifts, dims, comm_names, shapes)
        return _roll_all(x, shifts, dims, comm_names, shapes)

    @staticmethod
    def backward(ctx, g):
        shifts, dims, comm_names, shapes = ctx.args
        return _roll_all(g, tuple(-s for s in shifts), dims, comm_names, shapes), None, None, None, None


def _roll_all(x, shifts, dims, comm_names, shapes):
    """Roll along every (dim, group): one peer-memory kernel for the (H, W) roll over sp1 x sp2 where it
    applies (``parallel.halo``), else one NCCL exchange per dimension."""
    from . import halo

    if halo.available(x, shifts, dims, comm_names, shapes):
        return halo.roll(x, shifts, shapes)
    shapes = shapes or [None] * len(shifts)
    for sh, d, c, s in zip(shifts, dims, comm_names, shapes):
        if sh != 0:
            x = _distributed_roll(x, sh, d, c, s)
    return x


class _TransposeFwdTransposeBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dims, dim0_split_sizes, dim1_split_sizes, comm_name):
        ctx.args = (dims, dim0_split_sizes, dim1_split_sizes, comm_name)
        return _transpose(x, dims[0], dims[1], dim0_split_sizes, dim1_split_sizes, comm_name)

    @staticmethod
    def backward(ctx, g):
        dims, s0, s1, comm_name = ctx.args
        return _transpose(g, dims[1], dims[0], s1, s0, comm_name), None, None, None, None


@profile("identity-allreduce")
def identity_forward_allreduce_backward(x, comm_name):
    return _IdentityFwdAllReduceBwd.apply(x, comm_name)


@profile("allreduce-identity")
def allreduce_forward_identity_backward(x, comm_name):
    return _AllReduceFwdIdentityBwd.apply(x, comm_name)


@profile("allgather-split")
def allgather_forward_split_backward(x, dim, shapes, comm_name):
    return _AllGatherFwdSplitBwd.apply(x, dim, shapes, comm_name)


@profile("allgather-reducescatter")
def allgather_forward_reducescatter_backward(x, dim, shapes, comm_name):
    return _AllGatherFwdReduceScatterBwd.apply(x, dim, shapes, comm_name)


@profile("reducescatter-allgather")
def reducescatter_forward_allgather_backward(x, dim, shapes, comm_name):
    return _ReduceScatterFwdAllGatherBwd.apply(x, dim, shapes, comm_name)


@profile("split-allgather")
def split_forward_allgather_backward(x, dim, shapes, comm_name):
    return _SplitFwdAllGatherBwd.apply(x, dim, shapes, comm_name)


@profile("roll")
def roll_forward_reverseroll_backward(x, shifts, dims, comm_names,
                                      shapes: Optional[Sequence] = None):
    return _RollFwdReverseRollBwd.apply(x, tuple(shifts), tuple(dims), tuple(comm_names),
                                        tuple(shapes) if shapes is not None else None)


@profile("transpose-transpose")
def transpose_forward_transpose_backward(x, dims, dim0_split_sizes, dim1_split_sizes, comm_name):
    return _TransposeFwdTransposeBwd.apply(x, dims, dim0_split_sizes, dim1_split_sizes, comm_name)
