"""Plain-PyTorch definitions of every fused operator (the numerical oracle).

These run the math of the reference model step by step, in the input dtype:

* RMSNorm with ``eps = finfo(float32).eps`` computed in fp32 (``nn.RMSNorm`` under
  autocast, ``models/layer_helpers.py:113-116``);
* shifted-window attention: cyclic roll, window partition (``models/swin_helpers.py:26-77``),
  QK-RMSNorm, softmax(QK^T * scale + mask) V with the additive -100 latitude-wrap mask
  (``models/swin_helpers.py:322-397``), window reverse and roll back;
* patch embedding as a strided convolution, head + unpatchify
  (``models/swin.py:269-299``), GELU MLP, weighted squared error.

The CUDA kernels are tested against these functions, and CPU runs use them directly.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .geometry import WindowGeometry

EPS32 = float(torch.finfo(torch.float32).eps)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float | None = None) -> torch.Tensor:
    eps = EPS32 if eps is None else eps
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype)


def linear(x, weight, bias=None, residual=None, activation=None):
    y = F.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))
    if activation == "gelu":
        y = F.gelu(y)
    elif activation is not None:
        raise ValueError(f"unknown activation {activation!r}")
    if residual is not None:
        y = y + residual
    return y


def wrap_labels(geom: WindowGeometry, n_rows: int, device) -> torch.Tensor:
    """Region label (0/1) of each local (rolled) token row for the shift mask."""
    rows = torch.arange(n_rows, device=device) + geom.row_offset
    if geom.mask and geom.mask_shift > 0:
        return (rows >= geom.h_global - geom.mask_shift).to(torch.int64)
    return torch.zeros(n_rows, dtype=torch.int64, device=device)


def window_mask(geom: WindowGeometry, H: int, W: int, T: int, device, dtype) -> torch.Tensor:
    """Additive mask of shape (num_windows, T*wa, T*wa)."""
    wh, ww = geom.window
    lab = wrap_labels(geom, H, device)  # (H,)
    lab = lab.view(H // wh, wh, 1).expand(H // wh, wh, ww)  # (nH, wh, ww)
    lab = lab.reshape(H // wh, 1, 1, wh * ww).expand(H // wh, W // ww, T, wh * ww)
    lab = lab.reshape((H // wh) * (W // ww), T * wh * ww)
    diff = lab.unsqueeze(1) != lab.unsqueeze(2)
    m = torch.zeros(diff.shape, dtype=dtype, device=device)
    m.masked_fill_(diff, -100.0)
    return m


def window_partition(x: torch.Tensor, window):
    """(B, T, H, W, ...) -> (B*nW, T*wh*ww, ...)."""
    B, T, H, W = x.shape[:4]
    rest = x.shape[4:]
    wh, ww = window
    x = x.reshape(B, T, H // wh, wh, W // ww, ww, *rest)
    nrest = len(rest)
    perm = (0, 2, 4, 1, 3, 5) + tuple(6 + i for i in range(nrest))
    return x.permute(*perm).reshape(B * (H // wh) * (W // ww), T * wh * ww, *rest)


def window_reverse(x: torch.Tensor, window, B, T, H, W):
    wh, ww = window
    rest = x.shape[2:]
    x = x.reshape(B, H // wh, W // ww, T, wh, ww, *rest)
    nrest = len(rest)
    perm = (0, 3, 1, 4, 2, 5) + tuple(6 + i for i in range(nrest))
    return x.permute(*perm).reshape(B, T, H, W, *rest)


def window_attention(qkv, q_norm_w, k_norm_w, num_heads, head_dim, geom: WindowGeometry,
                     scale: float):
    """qkv: (B, T, H, W, 3*nh*hd) -> (B, T, H, W, nh*hd)."""
    B, T, H, W, _ = qkv.shape
    sh, sw = geom.shift
    x = qkv
    if sh or sw:
        x = torch.roll(x, shifts=(-sh, -sw), dims=(2, 3))
    win = window_partition(x, geom.window)  # (Bw, L, 3C)
    Bw, L, _ = win.shape
    win = win.view(Bw, L, 3, num_heads, head_dim).permute(2, 0, 3, 1, 4)  # 3,Bw,nh,L,hd
    q, k, v = win[0], win[1], win[2]
    q = rms_norm(q, q_norm_w)
    k = rms_norm(k, k_norm_w)
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if geom.mask:
        m = window_mask(geom, H, W, T, qkv.device, torch.float32)  # (nW, L, L)
        nW = m.shape[0]
        s = s.view(Bw // nW, nW, num_heads, L, L) + m.view(1, nW, 1, L, L)
        s = s.view(Bw, num_heads, L, L)
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p.to(v.dtype), v)  # Bw, nh, L, hd
    o = o.transpose(1, 2).reshape(Bw, L, num_heads * head_dim)
    o = window_reverse(o, geom.window, B, T, H, W)
    if sh or sw:
        o = torch.roll(o, shifts=(sh, sw), dims=(2, 3))
    return o.to(qkv.dtype)


def patch_embed(x, weight, bias, patch_size, add=None):
    """x: (N, C, H, W) -> (N, h, w, E) (+ ``add`` broadcast over the leading batch)."""
    y = F.conv2d(x.to(weight.dtype) if not x.is_floating_point() else x, weight.to(x.dtype),
                 None if bias is None else bias.to(x.dtype), stride=patch_size)
    y = y.permute(0, 2, 3, 1)
    if add is not None:
        N = y.shape[0]
        P = add.reshape(-1, *y.shape[1:]).shape[0]
        y = (y.reshape(N // P, P, *y.shape[1:]) + add.reshape(1, P, *y.shape[1:]).to(y.dtype))
        y = y.reshape(N, *y.shape[2:])
    return y.contiguous()


def head_unpatchify(x, weight, patch_size, out_chans):
    """x: (B, T, h, w, E) -> (B, T, C, h*p, w*p)."""
    b, t, h, w, _ = x.shape
    p = patch_size
    y = F.linear(x, weight.to(x.dtype))
    y = y.reshape(b, t, h, w, p, p, out_chans)
    y = torch.einsum("nthwpqc->ntchpwq", y)
    return y.reshape(b, t, out_chans, h * p, w * p)


def weighted_sse(x, y, area_w=None, ch_w=None):
    """sum over all elements of (x - y)^2 * area_w[h, 1] * ch_w[c, 1, 1]."""
    se = (x.float() - y.float()) ** 2
    if area_w is not None:
        se = se * area_w.float()
    if ch_w is not None:
        se = se * ch_w.float()
    return se.sum()


def weighted_se_per_channel(x, y, area_w):
    """sum over (H, W) of area_w * (x - y)^2 -> shape x.shape[:-2]."""
    se = area_w.float() * (x.float() - y.float()) ** 2
    return se.sum(dim=(-1, -2))
