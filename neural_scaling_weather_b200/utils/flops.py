"""Analytic forward FLOP and parameter counts of the Swin stack.

The counting rules are the reference's (``utils/flops_utils.py:15-146``), kept identical
so that "TFLOPs consumed" and MFU figures compare across the two frameworks: patch and
coordinate embeddings as dense projections, attention as qkv + logits + softmax (5 per
element) + attend + projection, MLP with 8 FLOPs per activation element, RMSNorm 3 per
element (x4 per block: two block norms and the q/k norms), and the head.  Training
multiplies the forward count by 3.
"""

from __future__ import annotations

TFLOPS = 1e-12


def attention_flops(batch, seq, embed, heads):
    hd = embed // heads
    qkv = 2 * batch * seq * embed * embed * 3 + batch * seq * embed * 3
    logits = 2 * batch * heads * seq * hd * seq
    softmax = 5 * batch * heads * seq * seq
    attend = 2 * batch * heads * seq * seq * hd
    project = 2 * batch * seq * embed * embed + batch * seq * embed
    return (qkv + logits + softmax + attend + project) * TFLOPS


def mlp_flops(batchseq, embed, hidden):
    fc1 = 2 * batchseq * embed * hidden + batchseq * hidden
    act = 8 * batchseq * hidden
    fc2 = 2 * batchseq * hidden * embed + batchseq * embed
    return (fc1 + act + fc2) * TFLOPS


def patch_embed_flops(batch, h, w, c, patch_size, embed):
    seq = h // patch_size * w // patch_size
    return (2 * batch * h * w * c * embed + batch * seq * embed) * TFLOPS


def rms_norm_flops(size):
    return 3 * size * TFLOPS


def head_flops(batch, h, w, embed, patch_size, out_chans):
    seq = h // patch_size * w // patch_size
    return 2 * batch * seq * embed * out_chans * patch_size * patch_size * TFLOPS


class FlopsCalculator:
    def __init__(self, cfg, h, w, c_in, c_out, batch=None):
        m = cfg.model
        self.wh, self.ww = m.window_size[0], m.window_size[1]
        self.embed, self.heads, self.depth = m.embed_dim, m.num_heads, m.depth
        self.patch_size = m.patch_size
        self.batch = cfg.parallelism.micro_batch_size if batch is None else batch
        self.t = cfg.train.temporal_context_window
        self.seq = self.t * self.wh * self.ww
        self.h, self.w = h, w
        self.h_patch, self.w_patch = h // self.patch_size, w // self.patch_size
        self.num_windows = self.h_patch // self.wh * self.w_patch // self.ww
        self.c_in, self.c_out = c_in, c_out
        self.params_backbone = 0.0

    def flops(self, verbose: bool = False) -> float:
        """Forward TFLOPs of one micro-batch."""
        bt = self.batch * self.t
        patch = patch_embed_flops(bt, self.h, self.w, self.c_in, self.patch_size, self.embed)
        pos = patch_embed_flops(bt, self.h, self.w, 4, self.patch_size, self.embed)
        attn = attention_flops(self.batch * self.num_windows, self.seq, self.embed, self.heads)
        ntok = bt * self.h_patch * self.w_patch
        mlp = mlp_flops(ntok, self.embed, 4 * self.embed)
        norm = rms_norm_flops(ntok * self.embed)
        block = attn + mlp + 4 * norm
        head = head_flops(self.batch, self.h, self.w, self.embed, self.patch_size, self.c_out)
        if verbose:
            print(f"patch {patch} pos {pos} attn {attn} mlp {mlp} norm {norm} block {block} head {head} TFLOP")
        return patch + pos + block * self.depth + head

    def param_count(self) -> float:
        e, p = self.embed, self.patch_size
        patch = e * self.c_in * p * p + e
        pos = e * 4 * p * p + e
        block = e * e * 3 + e * e + e * 4 * e * 2 + e * 4
        head = self.c_out * e * p * p
        self.params_backbone = block * self.depth * 1e-6
        return (patch + pos + block * self.depth + head) * 1e-6
