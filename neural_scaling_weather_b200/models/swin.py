"""Flat shifted-window transformer on a lat-lon grid (the weather emulator backbone).

Architecture and parameter layout follow the reference (``models/swin.py:36-323``,
``models/swin_helpers.py:80-459``, ``models/mlp.py:14-95``):

* patch embedding (``Conv2d`` k = s = p) plus a coordinate positional embedding (a second
  patch projection of the (x, y, z, t) coordinate field, on CUDA computed once per weight version) or a
  learned, sp-sharded positional tensor;
* ``depth`` blocks of RMSNorm -> shifted-window multi-head attention with QK-RMSNorm
  -> residual -> RMSNorm -> GELU MLP -> residual; shift 0 on even blocks and half the
  window on odd blocks; an additive -100 mask separates tokens on opposite sides of the
  latitude wrap (longitude is periodic and unmasked);
* a linear head and unpatchify; only the last time step is returned.

The B200 design departs from the reference's data flow, not its math:

* q/k/v are one fused GEMM (the three weights keep their own parameters and names);
* the cyclic shift, window partition and window reverse are index arithmetic inside the
  attention kernel when the spatial dims are not sharded, so no permuted copies exist;
  with spatial sharding the halo roll runs first and the kernel uses the global row
  offset for the mask;
* the mask is computed from row indices inside the kernel instead of a stored tensor;
* the bias, GELU and residual additions are GEMM epilogues.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..parallel import comm
from ..parallel.helpers import offsets
from ..parallel.mappings import roll_forward_reverseroll_backward
from ..utils.checkpoint_io import verified_load
from ..utils.profiler import profile
from .layers import (
    BiasLayer,
    Conv2DLayer,
    LinearLayer,
    NormLayer,
    PatchEmbedLayer,
    _meta,
    trunc_normal_,
)


class WindowMultiHeadAttention(nn.Module):
    """Window attention with QK-RMSNorm; q/k/v column-parallel, proj row-parallel over tp."""

    def __init__(self, dim: int, num_heads: int, window_size: Tuple[int, int]):
        super().__init__()
        if dim % num_heads:
            raise AssertionError("embed dim must be divisible by the number of heads")
        tp = comm.get_size("tp")
        if num_heads % tp or dim % tp:
            raise AssertionError("heads and embed dim must split evenly over tp ranks")
        self.dim, self.num_heads, self.window_size = dim, num_heads, tuple(window_size)
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.num_heads_local = num_heads // tp
        dl = dim // tp
        col = lambda: _meta(["tp", None], ["sp1-sp2"], ["sp1-sp2"])  # noqa: E731
        colb = lambda: _meta(["tp"], ["sp1-sp2"], ["sp1-sp2"])  # noqa: E731
        self.q = LinearLayer(dim, dl, comm_metadata=col())
        self.biasq = BiasLayer(dl, comm_metadata=colb())
        self.k = LinearLayer(dim, dl, comm_metadata=col())
        self.biask = BiasLayer(dl, comm_metadata=colb())
        qk_meta = lambda: _meta([None], ["tp-sp1-sp2"], ["tp-sp1-sp2"])  # noqa: E731
        self.q_norm = NormLayer(self.head_dim, norm_type="rms_norm", comm_metadata=qk_meta())
        self.k_norm = NormLayer(self.head_dim, norm_type="rms_norm", comm_metadata=qk_meta())
        self.v = LinearLayer(dim, dl, comm_metadata=col())
        self.biasv = BiasLayer(dl, comm_metadata=colb())
        self.proj = LinearLayer(dl, dim, comm_metadata=_meta([None, "tp"], ["sp1-sp2"], ["sp1-sp2"]))
        self.biasproj = BiasLayer(dim, comm_metadata=_meta([], ["tp-sp1-sp2"], ["sp1-sp2"]))

    def qkv_params(self):
        """q/k/v weights and biases; the fused GEMM concatenates them along N."""
        return ([self.q.weight, self.k.weight, self.v.weight],
                [self.biasq.bias, self.biask.bias, self.biasv.bias])


class MLP(nn.Module):
    """fc1 (column-parallel) -> exact GELU -> fc2 (row-parallel) with separate biases."""

    def __init__(self, in_features, hidden_features=None, out_features=None,
                 act_layer=nn.GELU, drop: float = 0.0):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        tp = comm.get_size("tp")
        if hidden_features % tp:
            raise AssertionError(f"cannot shard MLP hidden {hidden_features} into {tp} shards")
        hl = hidden_features // tp
        self.fc1 = LinearLayer(in_features, hl, comm_metadata=_meta(["tp", None], ["sp1-sp2"], ["sp1-sp2"]))
        self.bias1 = BiasLayer(hl, comm_metadata=_meta(["tp"], ["sp1-sp2"], ["sp1-sp2"]))
        self.fc2 = LinearLayer(hl, out_features, comm_metadata=_meta([None, "tp"], ["sp1-sp2"], ["sp1-sp2"]))
        self.bias2 = BiasLayer(out_features, comm_metadata=_meta([], ["tp-sp1-sp2"], ["sp1-sp2"]))
        self.drop = drop

    @profile("mlp")
    def forward(self, x, residual: Optional[torch.Tensor] = None):
        tp = comm.get_size("tp")
        if tp == 1 and not (self.drop > 0 and self.training):
            return ops.mlp(x, self.fc1.weight, self.bias1.bias, self.fc2.weight, self.bias2.bias, residual)
        h = ops.linear_colparallel(x, self.fc1.weight, self.bias1.bias, activation="gelu", group="tp")
        if self.drop > 0 and self.training:
            h = F.dropout(h, self.drop, True)
        if tp == 1 and not (self.drop > 0 and self.training):
            return ops.linear(h, self.fc2.weight, self.bias2.bias, residual=residual)
        if not (self.drop > 0 and self.training):  # row-parallel fc2 with the tp all-reduce fused
            return ops.linear_allreduce(h, self.fc2.weight, self.bias2.bias, residual=residual, group="tp")
        y = ops.linear_allreduce(h, self.fc2.weight, self.bias2.bias, group="tp")
        y = F.dropout(y, self.drop, True)
        return y if residual is None else y + residual


class Block(nn.Module):
    def __init__(self, dim, num_heads, feat_size, window_size, temporal_context_window_size,
                 shift_size=(0, 0), mlp_ratio=4.0, drop=0.0, act_layer=nn.GELU,
                 sp1_shapes=None, sp2_shapes=None):
        super().__init__()
        self.dim = dim
        self.feat_size = tuple(feat_size)
        self.window_size = tuple(window_size)
        self.window_area = window_size[0] * window_size[1]
        self.temporal_context_window_size = temporal_context_window_size
        self.shift_size = tuple(shift_size)
        self.sp1_shapes = list(sp1_shapes) if sp1_shapes is not None else [feat_size[0]]
        self.sp2_shapes = list(sp2_shapes) if sp2_shapes is not None else [feat_size[1]]
        h_loc, w_loc = self.feat_size
        if h_loc % window_size[0] or w_loc % window_size[1]:
            raise AssertionError(
                f"local patch grid {self.feat_size} is not divisible by window {window_size}"
            )
        norm_meta = lambda: _meta([None], ["tp-sp1-sp2"], ["sp1-sp2"])  # noqa: E731
        self.norm1 = NormLayer(dim, norm_type="rms_norm", comm_metadata=norm_meta())
        self.attn = WindowMultiHeadAttention(dim, num_heads=num_heads, window_size=window_size)
        self.norm2 = NormLayer(dim, norm_type="rms_norm", comm_metadata=norm_meta())
        self.mlp = MLP(dim, hidden_features=int(dim * mlp_ratio), act_layer=act_layer, drop=drop)
        # global row offset of this rank's shard (patch units), for the wrap mask
        self.row_offset = offsets(self.sp1_shapes)[comm.get_rank("sp1")]
        self.h_global = sum(self.sp1_shapes)

    def attention_geometry(self, index_shift: Tuple[int, int]) -> ops.WindowGeometry:
        sh = self.shift_size[0]
        return ops.WindowGeometry(
            window=self.window_size,
            shift=index_shift,
            mask=any(self.shift_size),
            mask_shift=sh,
            row_offset=self.row_offset,
            h_global=self.h_global,
        )

    def _spatial_sharded(self) -> bool:
        return comm.get_size("sp1") > 1 or comm.get_size("sp2") > 1

    @profile("shifted_wmha")
    def _shifted_window_attn(self, x, skip: Optional[torch.Tensor]):
        """Attention branch; adds ``skip`` inside the proj epilogue when that is exact."""
        attn = self.attn
        roll = self._spatial_sharded() and any(self.shift_size)
        if roll:
            x = roll_forward_reverseroll_backward(
                x, tuple(-s for s in self.shift_size), (-3, -2), ["sp1", "sp2"],
                shapes=(self.sp1_shapes, self.sp2_shapes))
            geom = self.attention_geometry((0, 0))
        else:
            geom = self.attention_geometry(self.shift_size)
        w_qkv, b_qkv = attn.qkv_params()
        qkv = ops.linear_colparallel(x, w_qkv, b_qkv, group="tp")
        o = ops.window_attention(qkv, attn.q_norm.weight, attn.k_norm.weight,
                                 attn.num_heads_local, attn.head_dim, geom, attn.scale)
        tp = comm.get_size("tp")
        if tp == 1 and not roll:
            return ops.linear(o, attn.proj.weight, attn.biasproj.bias, residual=skip)
        # row-parallel proj: the tp all-reduce is fused into the GEMM where the group allows
        if not roll:
            return ops.linear_allreduce(o, attn.proj.weight, attn.biasproj.bias, residual=skip, group="tp")
        y = ops.linear_allreduce(o, attn.proj.weight, attn.biasproj.bias, group="tp")
        y = roll_forward_reverseroll_backward(
            y, self.shift_size, (-3, -2), ["sp1", "sp2"],
            shapes=(self.sp1_shapes, self.sp2_shapes))
        return y if skip is None else y + skip

    def forward(self, x: torch.Tensor, condition: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: (B, T, H, W, C) -> same shape."""
        # each pre-norm and its skip connection come from one node, so the two gradients of
        # the residual stream are summed inside the RMSNorm backward
        h, skip = self._norm_skip(self.norm1, x)
        x = self._shifted_window_attn(h, skip)
        h, skip = self._norm_skip(self.norm2, x)
        return self.mlp(h, residual=skip)

    @staticmethod
    def _norm_skip(norm, x):
        if norm.norm_type == "rms_norm":
            return ops.rms_norm_with_skip(x, norm.weight)
        return norm(x), x


class SwinTransformer(nn.Module):
    """Input (B, T, C_in, H, W) -> output (B, 1, C_out, H', W') for the last time step."""

    @classmethod
    def instantiate_from_cfg(cls, cfg, domain_metadata):
        ws = cfg.model.window_size
        window_size = tuple(ws) if isinstance(ws, (list, tuple)) else (ws, ws)
        n_inv = len(cfg.data.invariants) if cfg.data.invariants else 0
        return cls(
            patch_size=cfg.model.patch_size,
            window_size=window_size,
            depth=cfg.model.depth,
            num_heads=cfg.model.num_heads,
            temporal_context_window_size=cfg.train.temporal_context_window,
            in_chans=domain_metadata["n_channels"] + n_inv,
            out_chans=domain_metadata["n_channels"],
            embed_dim=cfg.model.embed_dim,
            mlp_ratio=cfg.model.mlp_ratio,
            drop_rate=cfg.model.dropout,
            coord_pos_embed=getattr(cfg.model, "coord_pos_embed", True),
            use_transformer_engine=getattr(cfg.parallelism, "use_transformer_engine", True),
            domain_metadata=domain_metadata,
        )

    def __init__(self, temporal_context_window_size=1, window_size=(9, 9), patch_size=16,
                 in_chans=3, out_chans=3, embed_dim=768, depth=12, num_heads=12, mlp_ratio=4.0,
                 drop_rate=0.0, coord_pos_embed=True, domain_metadata=None,
                 use_transformer_engine=True, use_big_skip_conv=False, **kwargs):
        super().__init__()
        if domain_metadata is None:
            raise AssertionError("the data loader must provide domain metadata")
        self.num_features = self.embed_dim = embed_dim
        self.patch_size = patch_size
        self.temporal_context_window_size = temporal_context_window_size
        self.window_size = tuple(window_size)
        self.in_chans, self.out_chans = in_chans, out_chans
        self.drop_rate = drop_rate
        self.coord_pos_embed = coord_pos_embed
        self.domain_metadata = domain_metadata
        self.use_big_skip_conv = use_big_skip_conv
        sp1_shapes, sp2_shapes = domain_metadata["sp_shapes"]
        shared = lambda: _meta([], ["tp-sp1-sp2"], ["sp1-sp2"])  # noqa: E731

        self.patch_embed = PatchEmbedLayer(patch_size, in_chans, embed_dim, sp1_shapes, sp2_shapes,
                                           comm_metadata=shared())
        if coord_pos_embed:
            self._init_coords()
            self.pos_embed = PatchEmbedLayer(patch_size, self.coords.shape[-1], embed_dim,
                                             sp1_shapes, sp2_shapes, comm_metadata=shared())
        else:
            self.pos_embed = nn.Parameter(torch.zeros(
                1, temporal_context_window_size, self.patch_embed.h, self.patch_embed.w, embed_dim))
            trunc_normal_(self.pos_embed, std=0.02)
            self.pos_embed.comm_metadata = _meta([None, None, "sp1", "sp2", None], ["tp"], [])

        self.blocks = nn.ModuleList([
            Block(dim=embed_dim, num_heads=num_heads,
                  feat_size=(self.patch_embed.h, self.patch_embed.w),
                  window_size=self.window_size,
                  temporal_context_window_size=temporal_context_window_size,
                  shift_size=tuple(0 if i % 2 == 0 else w // 2 for w in self.window_size),
                  mlp_ratio=mlp_ratio, drop=drop_rate,
                  sp1_shapes=self.patch_embed.sp1_patch_shapes,
                  sp2_shapes=self.patch_embed.sp2_patch_shapes)
            for i in range(depth)
        ])
        self.out_size = out_chans * patch_size * patch_size
        self.head = LinearLayer(embed_dim, self.out_size, comm_metadata=shared())
        if use_big_skip_conv:
            self.skip_conv = Conv2DLayer(in_chans, out_chans, kernel_size=1, bias=False,
                                         comm_metadata=shared())
        self.apply(self._init_weights)

    def _init_coords(self):
        T = self.temporal_context_window_size
        spatial = self.domain_metadata["coords"]  # (H, W, 3)
        H, W, _ = spatial.shape
        t = torch.linspace(0, 1, T).view(T, 1, 1, 1).expand(T, H, W, 1)
        coords = torch.cat([spatial.unsqueeze(0).expand(T, H, W, -1).float(), t], dim=-1)
        self.register_buffer("coords", coords, persistent=False)  # (T, H, W, 4)
        # the same field channels-first and contiguous: one tensor that the cached projection keys on
        self.register_buffer("coords_nchw", coords.permute(0, 3, 1, 2).contiguous(), persistent=False)

    @staticmethod
    def _init_weights(m):
        if isinstance(m, (nn.Linear, nn.Conv2d, nn.Conv3d)):
            trunc_normal_(m.weight, std=0.02)
            if m.bias is not None:
                nn.init.constant_(m.bias, 0)
        elif isinstance(m, nn.LayerNorm):
            nn.init.constant_(m.bias, 0)
            nn.init.constant_(m.weight, 1.0)
        elif isinstance(m, nn.RMSNorm):
            nn.init.constant_(m.weight, 1.0)

    @profile("embed")
    def prepare_tokens(self, x):
        b, t, c, h, w = x.shape
        if self.coord_pos_embed:
            conv = self.pos_embed.proj.conv
            pos = ops.coord_pos_embed(self.coords_nchw, conv.weight, conv.bias, self.patch_size)  # (T, h', w', E)
        else:
            pos = self.pos_embed[0]
        tok = self.patch_embed.proj.conv
        out = ops.patch_embed(x.reshape(b * t, c, h, w), tok.weight, tok.bias, self.patch_size,
                              add=pos)
        return out.view(b, t, out.shape[1], out.shape[2], self.embed_dim)

    @profile("head")
    def forward_head(self, x):
        return ops.head_unpatchify(x, self.head.weight, self.patch_size, self.out_chans)

    @profile("forward")
    def forward(self, x):
        b, t, c, h, w = x.shape
        skip = x if self.use_big_skip_conv else None
        x = self.prepare_tokens(x)
        for blk in self.blocks:
            x = blk(x)
        x = self.forward_head(x)
        if self.use_big_skip_conv:
            s = self.skip_conv(skip.reshape(b * t, c, h, w)).view(b, t, self.out_chans, h, w)
            x = x + s
        return x[:, -1:]


class TimeStepper(nn.Module):
    """Autoregressive rollout wrapper (``models/helpers.py:9-37`` of the reference)."""

    def __init__(self, cfg, model_handle):
        super().__init__()
        self.model = model_handle
        self.num_rollout_steps = int(cfg.train.num_rollout_steps)
        self.num_invariants = len(cfg.data.invariants) if cfg.data.invariants else 0

    def forward(self, inp):
        preds = []
        x = inp
        c_in = inp.shape[2]
        for step in range(self.num_rollout_steps):
            pred = self.model(x)
            preds.append(pred)
            if step == self.num_rollout_steps - 1:
                break
            n_inv = c_in - pred.shape[2]
            if n_inv != self.num_invariants:
                raise AssertionError("number of invariants does not match")
            if n_inv > 0:
                x = torch.cat([pred.to(inp.dtype), inp[:, -pred.shape[1]:, -n_inv:]], dim=2)
            else:
                x = pred.to(inp.dtype)
        return torch.cat(preds, dim=1)


def get_model(cfg, domain_metadata=None):
    if cfg.model.arch != "swin":
        raise NotImplementedError(f"model type {cfg.model.arch} not implemented")
    return TimeStepper(cfg, SwinTransformer.instantiate_from_cfg(cfg, domain_metadata))


def strip_module_prefix(state_dict):
    from collections import OrderedDict

    return OrderedDict((k[len("module."):] if k.startswith("module.") else k, v)
                       for k, v in state_dict.items())


def load_model(model, checkpoint_file, map_location="cpu"):
    ckpt = verified_load(checkpoint_file, map_location=map_location, weights_only=False)
    state = ckpt["model_state"]
    try:
        model.load_state_dict(state)
    except RuntimeError:
        if not all(k.startswith("module.") for k in state):
            raise
        model.load_state_dict(strip_module_prefix(state))
    return model
