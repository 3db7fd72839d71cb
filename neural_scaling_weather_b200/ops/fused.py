"""Autograd functions binding the sm_100a kernels (CUDA tensors only).

Forward GEMMs run on the tcgen05 kernel with their epilogues fused (bias, GELU with the
pre-activation saved for backward, residual add, broadcast positional-embedding add).
Backward data-gradient GEMMs also run on the tcgen05 kernel (against a cached
transposed weight).  Weight-gradient GEMMs (dW = dy^T x, token-major operands read
MN-major by TMA) run on the tcgen05 CTA-pair kernel with the bias gradient (the column sums
of dy) from the same pass, accumulating in fp32 straight into ``param.grad`` where that is
the optimizer's flat buffer (``gradsink``).  Shapes the tcgen05 kernels cannot take (K or N
not a multiple of 8: only tiny test models) use cuBLAS plus the fused epilogue kernel.
"""

from __future__ import annotations

import os
import weakref
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import gradsink
from . import weights as wcache
from ._ext import require
from .geometry import WindowGeometry

DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _cdtype(x: torch.Tensor) -> torch.dtype:
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16


def _weight_t(params: Sequence[torch.Tensor], w: torch.Tensor) -> torch.Tensor:
    """Cached contiguous transpose of a (concatenated) weight, keyed on the live parameters."""
    return wcache.get_t(params, w)


def gemm(a: torch.Tensor, b: torch.Tensor, bias=None, residual=None, res_period: int = 0,
         act: int = 0, preact: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``epilogue(a @ b.T)``; a [M, K], b [N, K] in the compute dtype."""
    ext = require()
    a = a.contiguous()
    if ext.gemm_supported(a, b, False):
        return ext.gemm(a, b, bias, residual, res_period, act, preact)
    acc = torch.mm(a, b.t())
    if bias is None and residual is None and act == 0:
        return acc
    y, pre = ext.bias_act_residual(acc, bias, residual, res_period, act, preact is not None, DT[a.dtype])
    if preact is not None:
        preact.copy_(pre)
    return y


def wgrad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """fp32 ``dy^T @ x`` (tcgen05 weight-gradient kernel; cuBLAS for shapes it cannot take)."""
    ext = require()
    if ext.wgrad_supported(dy, x):
        return ext.wgrad(dy, x)
    return torch.mm(dy.t(), x, out_dtype=torch.float32)


def weight_grads(dy: torch.Tensor, x: torch.Tensor, ws: Sequence[torch.Tensor], bs: Sequence[torch.Tensor]):
    """Gradients of weights ``ws`` stacked along the rows of ``dy^T x`` (weight i owns the columns
    ``[off_i, off_i + rows_i)`` of ``dy``) and of their biases ``bs`` (one per weight, or none).

    dW and db come from one tcgen05 pass (one launch for equally shaped weights, e.g. the q / k / v
    projections); where ``param.grad`` is the flat fp32 buffer the kernel adds into it and the
    returned entry is ``None`` (``gradsink``).  Returns (grads_w, grads_b) in the order of ``ws``/``bs``.
    """
    ext = require()
    with_b = len(bs) == len(ws)
    rows = [w.shape[0] for w in ws]
    total = sum(rows)
    dy_all = dy[:, :total]
    if len(ws) <= 4 and len(set(rows)) == 1 and ext.wgrad_supported(dy_all, x):
        n, K = rows[0], x.shape[1]
        tws = [gradsink.target(w) for w in ws]
        tbs = [gradsink.target(b) for b in bs] if with_b else []
        acc = any(t is not None for t in tws)
        outs = [t.view(-1) if t is not None else
                (torch.zeros if acc else torch.empty)(n * K, dtype=torch.float32, device=dy.device) for t in tws]
        dbs = None
        db_acc = False
        if with_b:
            db_acc = any(t is not None for t in tbs)
            dbs = [t if t is not None else (torch.zeros if db_acc else torch.empty)(n, dtype=torch.float32,
                                                                                   device=dy.device) for t in tbs]
        ext.wgrad_segments(dy_all, x, outs, acc, dbs, db_acc)
        gw = [None if t is not None else o.view(w.shape) for t, o, w in zip(tws, outs, ws)]
        gb: List[Optional[torch.Tensor]] = []
        if with_b:
            gb = [None if t is not None else d.to(b.dtype) for t, d, b in zip(tbs, dbs, bs)]
        for w, t in zip(ws, tws):
            gradsink.done(w, t is not None)
        for b, t in zip(bs if with_b else [], tbs):
            gradsink.done(b, t is not None)
    else:
        gw, gb = [], []
        off = 0
        for i, w in enumerate(ws):
            dyi = dy[:, off:off + rows[i]]
            off += rows[i]
            gw.append(wgrad(dyi, x).view(w.shape))
            if with_b:
                gb.append(ext.col_sum(dyi.contiguous()).to(bs[i].dtype))
        for p in list(ws) + (list(bs) if with_b else []):
            gradsink.done(p, False)
    if not with_b and len(bs):  # one bias over all rows
        gb = [ext.col_sum(dy.contiguous()).to(bs[0].dtype)]
        gradsink.done(bs[0], False)
    return gw, gb


def _grad_out(g: Optional[torch.Tensor], p: torch.Tensor) -> Optional[torch.Tensor]:
    return None if g is None else g.to(p.dtype)


# ---------------------------------------------------------------------------- RMSNorm
def _norm_weight_grad(ctx, w, dw, t):
    """The norm weight's gradient for autograd: None when the kernel added it into the optimizer's buffer
    ``t`` (the reducer is told), else the fresh tensor."""
    if not ctx.needs_input_grad[1]:
        return None
    gradsink.done(w, t is not None)
    return None if t is not None else dw.to(w.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        ext = require()
        dt = _cdtype(x)
        x2 = x.reshape(-1, x.shape[-1]).to(dt).contiguous()
        y, rstd = ext.rmsnorm_fwd(x2, w.detach().float().contiguous(), eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        ctx.in_dtype = x.dtype
        ctx.eps = eps
        if ctx.needs_input_grad[1]:
            gradsink.use([w])
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        ext = require()
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).to(x2.dtype).contiguous()
        t = gradsink.target(w)
        dx, dw = ext.rmsnorm_bwd(dy2, x2, w.detach().float().contiguous(), rstd, ctx.eps, dw_into=t)
        return dx.view(ctx.shape).to(ctx.in_dtype), _norm_weight_grad(ctx, w, dw, t), None


class _RMSNormSkip(torch.autograd.Function):
    """(rms_norm(x), x) from one node: the skip connection's gradient arrives here together with
    the normalised branch's and is added inside the RMSNorm backward kernel (no separate add
    of two activation-sized gradients)."""

    @staticmethod
    def forward(ctx, x, w, eps):
        ext = require()
        dt = _cdtype(x)
        x2 = x.reshape(-1, x.shape[-1]).to(dt).contiguous()
        y, rstd = ext.rmsnorm_fwd(x2, w.detach().float().contiguous(), eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        ctx.in_dtype = x.dtype
        ctx.eps = eps
        if ctx.needs_input_grad[1]:
            gradsink.use([w])
        return y.view(x.shape), x.view_as(x)

    @staticmethod
    def backward(ctx, dy, dskip):
        ext = require()
        x2, w, rstd = ctx.saved_tensors
        if dy is None:
            if ctx.needs_input_grad[1]:
                gradsink.done(w, False)
            return dskip, None, None
        dy2 = dy.reshape(x2.shape).to(x2.dtype).contiguous()
        add = None if dskip is None else dskip.reshape(x2.shape).to(x2.dtype).contiguous()
        t = gradsink.target(w)
        dx, dw = ext.rmsnorm_bwd(dy2, x2, w.detach().float().contiguous(), rstd, ctx.eps, add, dw_into=t)
        return dx.view(ctx.shape).to(ctx.in_dtype), _norm_weight_grad(ctx, w, dw, t), None


def rms_norm_skip_cuda(x, w, eps=None):
    eps = float(torch.finfo(torch.float32).eps) if eps is None else float(eps)
    return _RMSNormSkip.apply(x, w, eps)


def rms_norm_cuda(x, w, eps=None):
    eps = float(torch.finfo(torch.float32).eps) if eps is None else float(eps)
    return _RMSNorm.apply(x, w, eps)


# ---------------------------------------------------------------------------- Linear
class _Linear(torch.autograd.Function):
    """``act(x W^T + b) + residual`` with W / b possibly concatenated parts.  With ``ctx.group`` set
    (a column-parallel linear whose input is replicated over that group) the data gradient is
    all-reduced over the group inside the dgrad GEMM's epilogue (peer loads over NVLink), which is
    the reference's ``copy_to_parallel_region`` backward (``distributed/mappings.py:24-46``)."""

    @staticmethod
    def forward(ctx, x, residual, act, nw, nb, group, *params):
        ws, bs = params[:nw], params[nw:nw + nb]
        dt = _cdtype(x)
        K = x.shape[-1]
        x2 = x.reshape(-1, K).to(dt)
        W = wcache.get_cat(ws, dt)
        if W.dim() != 2:
            W = W.reshape(W.shape[0], -1)
        N = W.shape[0]
        b = None
        if nb:
            b = bs[0].detach().float() if nb == 1 else torch.cat([t.detach().float() for t in bs])
        res2 = residual.reshape(-1, N).to(dt).contiguous() if residual is not None else None
        needs_grad = ctx.needs_input_grad[0] or any(ctx.needs_input_grad[5:])
        pre = None
        if act and needs_grad:
            pre = torch.empty(x2.shape[0], N, dtype=dt, device=x.device)
        y = gemm(x2, W, b, res2, 0, act, pre)
        ctx.save_for_backward(x2, pre)
        ctx.params = ws
        ctx.bparams = list(bs)
        ctx.group = group
        if any(ctx.needs_input_grad[6:]):
            gradsink.use(list(ws) + list(bs))
        ctx.W = W
        ctx.act, ctx.nw, ctx.nb = act, nw, nb
        ctx.shapes = [w.shape for w in ws]
        ctx.bsizes = [t.numel() for t in bs]
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.has_res = residual is not None
        ctx.res_dtype = residual.dtype if residual is not None else None
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        ext = require()
        x2, pre = ctx.saved_tensors
        W = ctx.W
        N = W.shape[0]
        dy2 = dy.reshape(-1, N).to(x2.dtype).contiguous()
        du = ext.gelu_bwd(dy2, pre) if ctx.act else dy2
        dx = None
        if ctx.needs_input_grad[0]:
            Wt = _weight_t(ctx.params, W)
            if ctx.group is not None:
                from ..parallel import symm

                bufs = symm.allreduce_buffers(ctx.group, du.shape[0], Wt.shape[0], du.dtype, du.device)
                dx = ext.gemm_allreduce(du.contiguous(), Wt, None, None, bufs.part_ptrs, bufs.flag_ptrs, bufs.rank)
            else:
                dx = gemm(du, Wt)
            dx = dx.view(ctx.x_shape).to(ctx.x_dtype)
        grads_w: List[Optional[torch.Tensor]] = [None] * ctx.nw
        grads_b: List[Optional[torch.Tensor]] = [None] * ctx.nb
        if any(ctx.needs_input_grad[6:]):
            gw, gb = weight_grads(du, x2, ctx.params, ctx.bparams)
            grads_w = [None if g is None else g.reshape(shp) for g, shp in zip(gw, ctx.shapes)]
            grads_b = gb
        dres = dy.to(ctx.res_dtype) if ctx.has_res else None
        return (dx, dres, None, None, None, None, *grads_w, *grads_b)


def _as_list(t):
    if t is None:
        return []
    if isinstance(t, torch.Tensor):
        return [t]
    return list(t)


def linear_cuda(x, weight, bias=None, residual=None, activation=None, allreduce_group=None):
    ws = _as_list(weight)
    bs = _as_list(bias)
    act = {None: 0, "gelu": 1}[activation]
    return _Linear.apply(x, residual, act, len(ws), len(bs), allreduce_group, *ws, *bs)


# ---------------------------------------------------------------------------- MLP
class _MLP(torch.autograd.Function):
    """fc1 + bias + GELU -> fc2 + bias (+ residual) with a fused backward.

    Forward: two tcgen05 GEMMs; the first's epilogue writes h = GELU(u) and, from the same
    erf / exp, GELU'(u) (saved for backward instead of u).
    Backward: du = (dy @ W2) * GELU'(u) in ONE GEMM epilogue (a plain multiply by the saved
    tensor), dx = du @ W1; weight gradients by cuBLAS with fp32 output.  Shapes the tcgen05
    kernel cannot take save u and use the GELU-backward kernel.
    """

    @staticmethod
    def forward(ctx, x, residual, w1, b1, w2, b2):
        ext = require()
        dt = _cdtype(x)
        K = x.shape[-1]
        x2 = x.reshape(-1, K).to(dt)
        W1 = wcache.get(w1, dt)
        W2 = wcache.get(w2, dt)
        N = W2.shape[0]
        H = W1.shape[0]
        needs_grad = any(ctx.needs_input_grad)
        u = torch.empty(x2.shape[0], H, dtype=dt, device=x.device) if needs_grad else None
        x2 = x2.contiguous()
        ctx.aux_is_grad = _MLP_SAVE_GELU_GRAD and ext.gemm_supported(x2, W1, False)
        # act 3: u holds GELU'(pre-activation); act 1: u holds the pre-activation itself
        h = gemm(x2, W1, b1.detach().float(), None, 0, 3 if ctx.aux_is_grad else 1, u)
        res2 = residual.reshape(-1, N).to(dt).contiguous() if residual is not None else None
        y = gemm(h, W2, b2.detach().float(), res2)
        ctx.save_for_backward(x2, u, h)
        ctx.w1, ctx.w2, ctx.W1, ctx.W2 = w1, w2, W1, W2
        ctx.b1, ctx.b2 = b1, b2
        if any(ctx.needs_input_grad[2:]):
            gradsink.use([w1, b1, w2, b2])
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.res_dtype = residual.dtype if residual is not None else None
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        ext = require()
        x2, u, h = ctx.saved_tensors
        N = ctx.W2.shape[0]
        dy2 = dy.reshape(-1, N).to(x2.dtype).contiguous()
        (dW2,), (db2,) = weight_grads(dy2, h, [ctx.w2], [ctx.b2])
        W2t = _weight_t([ctx.w2], ctx.W2)
        if ctx.aux_is_grad:
            if ext.gemm_supported(dy2, W2t, False):
                du = ext.gemm(dy2, W2t, None, u, 0, 4)  # epilogue: * GELU'(u) (saved)
            else:
                du = (gemm(dy2, W2t).float() * u.float()).to(u.dtype)
        elif ext.gemm_supported(dy2, W2t, False):
            du = ext.gemm(dy2, W2t, None, u, 0, 2)  # epilogue: * GELU'(u)
        else:
            du = ext.gelu_bwd(gemm(dy2, W2t).contiguous(), u)
        (dW1,), (db1,) = weight_grads(du, x2, [ctx.w1], [ctx.b1])
        dx = None
        if ctx.needs_input_grad[0]:
            W1t = _weight_t([ctx.w1], ctx.W1)
            dx = gemm(du, W1t).view(ctx.x_shape).to(ctx.x_dtype)
        dres = dy.to(ctx.res_dtype) if ctx.res_dtype is not None else None
        return dx, dres, _grad_out(dW1, ctx.w1), db1, _grad_out(dW2, ctx.w2), db2


# Which tensor the fc1 forward saves for the backward.  True: GELU'(u), formed from the same
# erf / exp as GELU (epilogue act 3), and the data-gradient GEMM multiplies by it (act 4).  False:
# the pre-activation u (act 1), with GELU'(u) formed in the data-gradient epilogue (act 2).
# Measured at 64800 x 4096 x 1024 (bf16, one B200): act 1 + act 2 = 0.556 + 0.552 ms against
# act 3 + act 4 = 0.616 + 0.516 ms, so the pre-activation is saved.
_MLP_SAVE_GELU_GRAD = False


def mlp_cuda(x, w1, b1, w2, b2, residual=None):
    return _MLP.apply(x, residual, w1, b1, w2, b2)


# ---------------------------------------------------------------------------- attention
def _geom_ints(B, T, H, W, nh, hd, g: WindowGeometry):
    return [B, T, H, W, nh, hd, g.window[0], g.window[1], g.shift[0], g.shift[1], int(g.mask),
            int(g.mask_shift), int(g.row_offset), int(g.h_global if g.h_global else H)]


# forward kernel choice (0: default = warp-specialised tcgen05; 1: mma.sync; 2: persistent tcgen05)
ATTN_FWD_IMPL = int(os.environ.get("NSW_ATTN_FWD_IMPL", "0"))


class _WindowAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, gi, scale):
        ext = require()
        qkv2 = qkv.contiguous()
        out, lse = ext.window_attn_fwd(qkv2, qw.detach().float().contiguous(),
                                       kw.detach().float().contiguous(), gi, scale, ATTN_FWD_IMPL)
        ctx.save_for_backward(qkv2, qw, kw, out, lse)
        ctx.gi, ctx.scale = gi, scale
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            gradsink.use([qw, kw])
        return out

    @staticmethod
    def backward(ctx, dout):
        ext = require()
        qkv, qw, kw, out, lse = ctx.saved_tensors
        # QK-norm weight gradients straight into the optimizer's gradient buffer where possible
        tq, tk = gradsink.target(qw), gradsink.target(kw)
        inplace = tq is not None and tk is not None
        dqkv, dqw, dkw = ext.window_attn_bwd(qkv, qw.detach().float().contiguous(),
                                             kw.detach().float().contiguous(), out,
                                             dout.to(qkv.dtype).contiguous(), lse, ctx.gi, ctx.scale,
                                             dqw_into=tq if inplace else None, dkw_into=tk if inplace else None)
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            gradsink.done(qw, inplace)
            gradsink.done(kw, inplace)
        if inplace:
            return dqkv, None, None, None, None
        return dqkv, dqw.to(qw.dtype), dkw.to(kw.dtype), None, None


def window_attention_cuda(qkv, q_norm_w, k_norm_w, num_heads, head_dim, geom: WindowGeometry, scale):
    B, T, H, W, C3 = qkv.shape
    dt = _cdtype(qkv)
    gi = _geom_ints(B, T, H, W, num_heads, head_dim, geom)
    out = _WindowAttn.apply(qkv.to(dt), q_norm_w, k_norm_w, gi, float(scale))
    return out.view(B, T, H, W, num_heads * head_dim)


# ---------------------------------------------------------------------------- patch embed
class _PatchEmbed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, add, p):
        ext = require()
        dt = _cdtype(x)
        N, C, H, Wd = x.shape
        h, wn = H // p, Wd // p
        E = w.shape[0]
        cols = ext.im2col(x.contiguous(), p, DT[dt])
        W2 = wcache.get(w, dt).reshape(E, -1)
        res, period = None, 0
        if add is not None:
            res = add.reshape(-1, E).to(dt).contiguous()
            period = res.shape[0]
        y = gemm(cols, W2, b.detach().float() if b is not None else None, res, period)
        ctx.save_for_backward(cols)
        ctx.w_param, ctx.W2 = w, W2
        ctx.b_param = b
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            gradsink.use([w] + ([b] if b is not None else []))
        ctx.meta = (N, C, H, Wd, p, h, wn, E, x.dtype, add is not None,
                    add.dtype if add is not None else None, period)
        ctx.has_b = b is not None
        return y.view(N, h, wn, E)

    @staticmethod
    def backward(ctx, dy):
        ext = require()
        (cols,) = ctx.saved_tensors
        N, C, H, Wd, p, h, wn, E, xdt, has_add, add_dt, period = ctx.meta
        dy2 = dy.reshape(-1, E).to(cols.dtype).contiguous()
        gw, gb = weight_grads(dy2, cols, [ctx.w_param], [ctx.b_param] if ctx.has_b else [])
        dW = None if gw[0] is None else gw[0].view(ctx.w_param.shape).to(ctx.w_param.dtype)
        db = gb[0] if ctx.has_b else None
        dadd = None
        if has_add:
            if dy2.shape[0] == period:  # one image per positional-embedding period: no reduction
                dadd = dy2.view(-1, h, wn, E).to(add_dt)
            else:
                dadd = dy2.float().view(-1, period, E).sum(0).view(-1, h, wn, E).to(add_dt)
        dx = None
        if ctx.needs_input_grad[0]:
            Wt = _weight_t([ctx.w_param], ctx.W2)
            dcols = gemm(dy2, Wt)
            dx = ext.col2im(dcols, N, C, H, Wd, p, DT[xdt])
        return dx, dW, db, dadd, None


def patch_embed_cuda(x, weight, bias, patch_size, add=None):
    return _PatchEmbed.apply(x, weight, bias, add, int(patch_size))


# ---------------------------------------------------------------------------- coordinate positional embedding
# patch columns of constant coordinate fields: key -> (weak reference to the field, its columns)
_COORD_COLS: Dict[Tuple, Tuple["weakref.ref", torch.Tensor]] = {}


def _coord_cols(coords: torch.Tensor, p: int, dt: torch.dtype) -> torch.Tensor:
    key = (id(coords), coords.data_ptr(), tuple(coords.shape), p, dt)
    hit = _COORD_COLS.get(key)
    if hit is not None and hit[0]() is coords:
        return hit[1]
    cols = wcache.normal_tensor(lambda: require().im2col(coords.contiguous(), p, DT[dt]))
    for k in [k for k, v in _COORD_COLS.items() if v[0]() is None]:  # fields of models that are gone
        del _COORD_COLS[k]
    _COORD_COLS[key] = (weakref.ref(coords), cols)
    return cols


class _CoordPosEmbed(torch.autograd.Function):
    """The coordinate positional embedding: a patch projection of the model's constant (T, 4, H, W)
    coordinate field (reference ``models/swin.py:270-284``, which re-runs the projection in every
    forward).  The field never changes, so its patch columns are built once; the projection depends
    only on the weights, so it is computed once per weight version (``ops.weights.get_derived``: a
    cache hit while the parameters' versions are unchanged, rebuilt in place after each optimizer step
    for captured CUDA graphs) instead of once per micro-batch.  The backward is the projection's
    weight and bias gradient from the cached columns."""

    @staticmethod
    def forward(ctx, coords, w, b, p):
        dt = _cdtype(coords)
        cols = _coord_cols(coords, p, dt)
        T, _, H, Wd = coords.shape
        h, wn, E = H // p, Wd // p, w.shape[0]

        def build():
            return gemm(cols, wcache.get(w, dt).reshape(E, -1), b.detach().float() if b is not None else None
                        ).view(T, h, wn, E)

        pos = wcache.get_derived(("coord_pos", p, dt, tuple(coords.shape), coords.data_ptr()),
                                 [w] + ([b] if b is not None else []), build)
        ctx.save_for_backward(cols)
        ctx.w_param, ctx.b_param, ctx.E = w, b, E
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            gradsink.use([w] + ([b] if b is not None else []))
        return pos.view_as(pos)

    @staticmethod
    def backward(ctx, dpos):
        (cols,) = ctx.saved_tensors
        dy = dpos.reshape(-1, ctx.E).to(cols.dtype).contiguous()
        gw, gb = weight_grads(dy, cols, [ctx.w_param], [ctx.b_param] if ctx.b_param is not None else [])
        dW = None if gw[0] is None else gw[0].view(ctx.w_param.shape).to(ctx.w_param.dtype)
        db = gb[0] if ctx.b_param is not None else None
        return None, dW, db, None


def coord_pos_embed_cuda(coords, weight, bias, patch_size):
    return _CoordPosEmbed.apply(coords, weight, bias, int(patch_size))


# ---------------------------------------------------------------------------- head
class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, p, C):
        ext = require()
        dt = _cdtype(x)
        B, T, h, wn, E = x.shape
        x2 = x.reshape(-1, E).to(dt).contiguous()
        W = wcache.get(w, dt)
        y2 = gemm(x2, W)
        out = ext.unpatchify(y2, B, T, h, wn, p, C)
        ctx.save_for_backward(x2)
        ctx.w_param, ctx.W = w, W
        ctx.meta = (B, T, h, wn, E, p, C, x.dtype)
        if ctx.needs_input_grad[1]:
            gradsink.use([w])
        return out

    @staticmethod
    def backward(ctx, dout):
        ext = require()
        (x2,) = ctx.saved_tensors
        B, T, h, wn, E, p, C, xdt = ctx.meta
        dy2 = ext.patchify(dout.to(x2.dtype).contiguous(), h, wn, p, C)
        (gw,), _ = weight_grads(dy2, x2, [ctx.w_param], [])
        dW = _grad_out(gw, ctx.w_param)
        dx = None
        if ctx.needs_input_grad[0]:
            Wt = _weight_t([ctx.w_param], ctx.W)
            dx = gemm(dy2, Wt).view(B, T, h, wn, E).to(xdt)
        return dx, dW, None, None


def head_unpatchify_cuda(x, weight, patch_size, out_chans):
    return _Head.apply(x, weight, int(patch_size), int(out_chans))


# ---------------------------------------------------------------------------- losses
class _WeightedSSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, aw, cw):
        ext = require()
        xc, yc = x.contiguous(), y.contiguous()
        awc = aw.float().contiguous().view(-1) if aw is not None else None
        cwc = cw.float().contiguous().view(-1) if cw is not None else None
        ctx.save_for_backward(xc, yc)
        ctx.w = (awc, cwc)
        return ext.weighted_sse(xc, yc, awc, cwc)

    @staticmethod
    def backward(ctx, g):
        ext = require()
        x, y = ctx.saved_tensors
        awc, cwc = ctx.w
        gs = g.detach().float().reshape(1).contiguous()
        dx = ext.weighted_sse_bwd(x, y, awc, cwc, gs) if ctx.needs_input_grad[0] else None
        dy = None
        if ctx.needs_input_grad[1]:
            dy = -ext.weighted_sse_bwd(x, y, awc, cwc, gs).to(y.dtype)
        return dx, dy, None, None


def weighted_sse_cuda(x, y, area_w=None, ch_w=None):
    return _WeightedSSE.apply(x, y, area_w, ch_w)


def weighted_se_per_channel_cuda(x, y, area_w):
    ext = require()
    return ext.weighted_se_per_plane(x.detach().contiguous(), y.detach().contiguous(),
                                     area_w.detach().float().contiguous().view(-1))


# ---------------------------------------------------------------------------- GEMM + all-reduce
class _LinearAllReduce(torch.autograd.Function):
    """y = all_reduce_group(x W^T) + b + residual with the reduction inside the GEMM epilogue
    (peer loads of every rank's partial tile over NVLink, tile by tile, while the next tile's
    MMAs run).  Backward is the row-parallel linear's: the all-reduce passes gradients through."""

    @staticmethod
    def forward(ctx, x, residual, group, w, b):
        from ..parallel import symm

        ext = require()
        dt = _cdtype(x)
        K = x.shape[-1]
        x2 = x.reshape(-1, K).to(dt).contiguous()
        W = wcache.get(w, dt)
        M, N = x2.shape[0], W.shape[0]
        bufs = symm.allreduce_buffers(group, M, N, dt, x.device)
        res2 = residual.reshape(-1, N).to(dt).contiguous() if residual is not None else None
        bias = b.detach().float().contiguous() if b is not None else None
        y = ext.gemm_allreduce(x2, W, bias, res2, bufs.part_ptrs, bufs.flag_ptrs, bufs.rank)
        ctx.save_for_backward(x2)
        ctx.w, ctx.W = w, W
        ctx.b = b
        ctx.has_b = b is not None
        if ctx.needs_input_grad[3] or ctx.needs_input_grad[4]:
            gradsink.use([w] + ([b] if b is not None else []))
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.res_dtype = residual.dtype if residual is not None else None
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        ext = require()
        (x2,) = ctx.saved_tensors
        W = ctx.W
        N = W.shape[0]
        dy2 = dy.reshape(-1, N).to(x2.dtype).contiguous()
        dx = gemm(dy2, _weight_t([ctx.w], W)).view(ctx.x_shape).to(ctx.x_dtype) if ctx.needs_input_grad[0] else None
        gw, gb = weight_grads(dy2, x2, [ctx.w], [ctx.b] if ctx.has_b else [])
        dW = None if gw[0] is None else gw[0].reshape(ctx.w.shape).to(ctx.w.dtype)
        db = gb[0] if ctx.has_b else None
        dres = dy.to(ctx.res_dtype) if ctx.res_dtype is not None else None
        return dx, dres, None, dW, db


def linear_allreduce_cuda(x, w, b, residual, group):
    return _LinearAllReduce.apply(x, residual, group, w, b)
