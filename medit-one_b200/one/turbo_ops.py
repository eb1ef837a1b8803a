"""one.turbo_ops: the reference's turbo entry points (one/turbo_ops.py:96-475), backed by
libone_b200.so. TURBO_MODE is True when the native library loads with every entry point.

There is no CPU fallback: the turbo functions require CUDA tensors and raise otherwise.
"""
from __future__ import annotations

import ctypes
import warnings
from typing import Optional, Tuple

import torch

try:
    from . import _capi as C
    TURBO_MODE = True
except Exception as exc:  # the library is required for every op below
    C = None
    TURBO_MODE = False
    warnings.warn(f"One B200 engine not available ({exc}); turbo ops will raise")


def _need(*ts):
    if not TURBO_MODE:
        raise RuntimeError("libone_b200.so is not built: run `python medit-one_b200/build.py`")
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("the B200 engine has no CPU path: pass CUDA tensors")


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def turbo_flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                          scale_factor: Optional[float] = None) -> torch.Tensor:
    """softmax(q k^T * scale [+ causal mask]) v with an fp32 softmax (one/turbo_ops.py:96-143).
    q [B, H, Nq, Dh], k / v [B, H, Nk, Dh]."""
    _need(q, k, v)
    if scale_factor is None:
        scale_factor = 1.0 / (q.size(-1) ** 0.5)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, Nq, Dh = q.shape
    out = torch.empty_like(q)
    C.check(C.LIB.one_flash_attention(C.ptr(q), C.ptr(k), C.ptr(v), B, H, Nq, k.shape[2], Dh, 1 if causal else 0,
                                      float(scale_factor), C.dtype_code(q.dtype), C.ptr(out), _stream()),
            "one_flash_attention")
    return out


def turbo_rope_flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor,
                               sin: torch.Tensor, causal: bool = True,
                               scale_factor: Optional[float] = None) -> torch.Tensor:
    """apply_rotary_pos_emb_flash(q, k, cos, sin) (one/flash_attention.py:26-33) followed by
    turbo_flash_attention, as one native call. q, k, v [B, H, N, Dh]; cos, sin [B or 1, N, Dh]
    in q's dtype (OneRotaryEmbedding's output)."""
    _need(q, k, v, cos, sin)
    if scale_factor is None:
        scale_factor = 1.0 / (q.size(-1) ** 0.5)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    cos, sin = cos.to(q.dtype).contiguous(), sin.to(q.dtype).contiguous()
    B, H, N, Dh = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape [B, H, N, Dh]")
    cb = cos.shape[0] if cos.dim() == 3 else 1
    if cos.shape[-2:] != (N, Dh) or sin.shape != cos.shape or cb not in (1, B):
        raise ValueError(f"cos / sin must be [B or 1, {N}, {Dh}], got {tuple(cos.shape)}")
    dt = C.dtype_code(q.dtype)
    ws = torch.empty(C.LIB.one_rope_flash_attention_workspace_bytes(B, H, N, Dh, dt), dtype=torch.uint8,
                     device=q.device)
    out = torch.empty_like(q)
    C.check(C.LIB.one_rope_flash_attention(C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(cos), C.ptr(sin), cb, B, H, N, Dh,
                                           1 if causal else 0, float(scale_factor), dt, C.ptr(out), C.ptr(ws),
                                           ws.numel(), _stream()),
            "one_rope_flash_attention")
    return out


def ops_error(clear: bool = True) -> Tuple[int, int]:
    """(code, site) of the standalone ops' device error record (0 = none); synchronises."""
    _need()
    where = ctypes.c_int32(0)
    code = C.LIB.one_ops_error(ctypes.byref(where), 1 if clear else 0)
    return int(code), int(where.value)


def turbo_moe_routing(inputs: torch.Tensor, experts_weights: torch.Tensor, top_k: int) -> torch.Tensor:
    """The reference's turbo_moe_routing (one/turbo_ops.py:146-172) returns its inputs: its
    PyTorch path computes a top-k that it discards. Kept as is. The LinearMoE router itself
    is `one.linear_moe.LinearMoE` / the C ABI `one_moe_routing`."""
    _need(inputs)
    return inputs


def turbo_rotary_embedding(x: torch.Tensor, position_ids: torch.Tensor, inv_freq: torch.Tensor
                           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [B, S, dim] in x's dtype (OneRotaryEmbedding.forward, one/modeling_one.py:159-182)."""
    _need(x, position_ids, inv_freq)
    pos = position_ids.to(torch.int64).contiguous()
    inv = inv_freq.to(torch.float32).contiguous()
    B, S = pos.shape
    dim = 2 * inv.numel()
    cos = torch.empty(B, S, dim, dtype=x.dtype, device=x.device)
    sin = torch.empty_like(cos)
    C.check(C.LIB.one_rotary_embedding(C.ptr(pos), B, S, C.ptr(inv), dim, C.dtype_code(x.dtype), C.ptr(cos), C.ptr(sin),
                                       _stream()), "one_rotary_embedding")
    return cos, sin


def turbo_cumsum_and_normalize(x: torch.Tensor, seq_len: int) -> torch.Tensor:
    """fp32 prefix mean over dim 1 (turbo_cumsum_and_normalize_cpu, one/turbo_ops.py:288-310)."""
    _need(x)
    x = x.contiguous()
    b, s, d = x.shape
    n = min(s, int(seq_len))
    out = torch.empty(b, n, d, dtype=x.dtype, device=x.device)
    C.check(C.LIB.one_cumsum_and_normalize(C.ptr(x), b, s, d, int(seq_len), C.dtype_code(x.dtype), C.ptr(out), _stream()),
            "one_cumsum_and_normalize")
    return out


def turbo_combined_rope_attention(single_x, key, value, cos, sin, lin_q, lin_k, lin_v, compute_sequence_len: int):
    """RoPE + three Dh->H projections + softmax(q*k - max) * v (the model's feature attention,
    one/modeling_one.py:515-547; the reference's own CPU version of this entry point raises
    NameError). Inputs [B, H, T, Dh]; cos/sin [B or 1, T, Dh]; returns [B, H, T, H]."""
    _need(single_x, key, value, cos, sin)
    t = int(compute_sequence_len)
    sx = single_x[:, :, -t:].contiguous()
    ky = key[:, :, -t:].contiguous()
    va = value[:, :, -t:].contiguous()
    if cos.dim() == 4:
        cos, sin = cos[:, 0], sin[:, 0]
    cos = cos[:, -t:].contiguous()
    sin = sin[:, -t:].contiguous()
    B, H, T, Dh = sx.shape
    hout = lin_q.weight.shape[0]
    dt = sx.dtype
    ws = [m.weight.to(dt).contiguous() for m in (lin_q, lin_k, lin_v)]
    bs = [None if m.bias is None else m.bias.to(dt).contiguous() for m in (lin_q, lin_k, lin_v)]
    out = torch.empty(B, H, T, hout, dtype=dt, device=sx.device)
    C.check(C.LIB.one_combined_rope_attention(C.ptr(sx), C.ptr(ky), C.ptr(va), C.ptr(cos.to(dt)), C.ptr(sin.to(dt)),
                                              cos.shape[0], C.ptr(ws[0]), C.ptr(bs[0]), C.ptr(ws[1]), C.ptr(bs[1]),
                                              C.ptr(ws[2]), C.ptr(bs[2]), B, H, T, Dh, hout, C.dtype_code(dt), C.ptr(out),
                                              _stream()), "one_combined_rope_attention")
    return out


class TurboFlashAttention(torch.nn.Module):
    """one/turbo_ops.py:437-475: returns (output, zero attention weights)."""

    def __init__(self, causal=True, dropout=0.0):
        super().__init__()
        self.causal = causal
        self.dropout = dropout

    def forward(self, q, k, v):
        out = turbo_flash_attention(q.contiguous(), k.contiguous(), v.contiguous(), causal=self.causal)
        return out, torch.zeros((q.size(0), q.size(1), q.size(2), k.size(2)), device=q.device, dtype=q.dtype)
