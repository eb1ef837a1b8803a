"""one.flash_attention: the reference's attention helpers (one/flash_attention.py) over the
B200 engine.

`rotate_half` / `apply_rotary_pos_emb_flash` are the reference's elementwise RoPE helpers
(one/flash_attention.py:20-33), kept as tensor expressions. `flash_attention` computes exact
softmax attention on the engine: the reference's blockwise FlashAttentionFunction (:43-139)
does not rescale across 64-wide blocks and equals exact attention only for N <= 64, and its
exception path (:242-282) computes the exact result; the engine follows the exact result.
"""
from __future__ import annotations

import torch

from .turbo_ops import turbo_flash_attention, turbo_rope_flash_attention


def rotate_half(x):
    x1, x2 = torch.chunk(x, 2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb_flash(q, k, cos, sin, unsqueeze_dim=1):
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


def flash_attention(q, k, v, dropout_p=0.0, causal=False):
    """softmax(q k^T / sqrt(Dh) [+ causal mask]) v; q, k, v [B, H, N, Dh] on CUDA."""
    if dropout_p:
        raise NotImplementedError("the inference engine has no dropout")
    return turbo_flash_attention(q, k, v, causal=causal)


def rope_flash_attention(q, k, v, cos, sin, dropout_p=0.0, causal=False):
    """apply_rotary_pos_emb_flash(q, k, cos, sin) then flash_attention(q, k, v) in one fused
    native call: the isolated RoPE + attention workload. cos, sin [B or 1, N, Dh]."""
    if dropout_p:
        raise NotImplementedError("the inference engine has no dropout")
    return turbo_rope_flash_attention(q, k, v, cos, sin, causal=causal)


class OneFlashAttention(torch.nn.Module):
    """one/flash_attention.py:285-324 (causal); returns (output, None)."""

    def __init__(self, config):
        super().__init__()
        self.num_heads = config.num_attention_heads
        self.head_dim = config.head_dim
        self.causal = True

    def forward(self, q, k, v):
        q = torch.clamp(q, min=-1e4, max=1e4)
        k = torch.clamp(k, min=-1e4, max=1e4)
        return flash_attention(q, k, v, 0.0, self.causal), None
