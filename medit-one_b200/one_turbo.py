"""one_turbo: the reference's native-extension module name and its five entry points
(csrc/one_kernels.cpp:128-134, discovered by one/turbo_ops.py:28-93), implemented by the B200
engine (libone_b200.so). Signatures follow the reference's pybind functions.
"""
from __future__ import annotations

import ctypes

import torch

from one import _capi as C
from one import turbo_ops as _t


def flash_attention(q, k, v, causal: bool = True, scale_factor: float = 1.0):
    """csrc/one_kernels.cpp:40-63. The reference's Python wrapper passes 1/sqrt(Dh)."""
    return _t.turbo_flash_attention(q, k, v, causal=causal, scale_factor=scale_factor)


def moe_routing(inputs, experts_weights, top_k: int):
    """csrc/one_kernels.cpp:65-74. The reference gives this entry point no consistent meaning
    (its CUDA and PyTorch paths compute different things); this keeps the PyTorch path's result."""
    return _t.turbo_moe_routing(inputs, experts_weights, top_k)


def rotary_embedding(x, position_ids, inv_freq):
    """csrc/one_kernels.cpp:76-86 -> (cos, sin) [B, S, dim]."""
    return _t.turbo_rotary_embedding(x, position_ids, inv_freq)


def cumsum_and_normalize(x, seq_len: int):
    """csrc/one_kernels.cpp:88-95."""
    return _t.turbo_cumsum_and_normalize(x, seq_len)


def combined_rope_attention(single_x, key, value, cos, sin, lin_q_weight, lin_k_weight, lin_v_weight,
                            compute_sequence_len: int):
    """csrc/one_kernels.cpp:97-125: weights arrive transposed ([Dh, H]) and without biases, as
    one/turbo_ops.py:345-360 passes them."""
    _t._need(single_x, key, value, cos, sin)
    t = int(compute_sequence_len)
    sx = single_x[:, :, -t:].contiguous()
    ky = key[:, :, -t:].contiguous()
    va = value[:, :, -t:].contiguous()
    if cos.dim() == 4:
        cos, sin = cos[:, 0], sin[:, 0]
    dt = sx.dtype
    cos = cos[:, -t:].to(dt).contiguous()
    sin = sin[:, -t:].to(dt).contiguous()
    B, H, T, Dh = sx.shape
    ws = [w.t().to(dt).contiguous() for w in (lin_q_weight, lin_k_weight, lin_v_weight)]
    hout = ws[0].shape[0]
    out = torch.empty(B, H, T, hout, dtype=dt, device=sx.device)
    C.check(C.LIB.one_combined_rope_attention(C.ptr(sx), C.ptr(ky), C.ptr(va), C.ptr(cos), C.ptr(sin), cos.shape[0],
                                              C.ptr(ws[0]), None, C.ptr(ws[1]), None, C.ptr(ws[2]), None, B, H, T, Dh,
                                              hout, C.dtype_code(dt), C.ptr(out),
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "one_combined_rope_attention")
    return out
