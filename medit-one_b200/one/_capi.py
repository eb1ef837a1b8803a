"""ctypes binding of libone_b200.so (include/one_b200.h).

The library is required: importing this module raises if it is missing or does not
export every entry point of the header. There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libone_b200.so")

ONE_OK, ONE_ERR_INVALID, ONE_ERR_CUDA, ONE_ERR_UNSUPPORTED, ONE_ERR_DEVICE = range(5)
ONE_DTYPE_BF16, ONE_DTYPE_F32 = 0, 1

(ONE_W_NORM1, ONE_W_LIN1_W, ONE_W_LIN1_B, ONE_W_LIN2_W, ONE_W_LIN2_B, ONE_W_LIN3_W, ONE_W_LIN3_B,
 ONE_W_LINQ_W, ONE_W_LINQ_B, ONE_W_LINK_W, ONE_W_LINK_B, ONE_W_LINV_W, ONE_W_LINV_B,
 ONE_W_HX_W, ONE_W_HX_B, ONE_W_HX_GATE, ONE_W_HX_EXPERTS, ONE_W_HX_BIAS2,
 ONE_W_CX_W, ONE_W_CX_B, ONE_W_CX_GATE, ONE_W_CX_EXPERTS, ONE_W_CX_BIAS2,
 ONE_W_X_W, ONE_W_X_B, ONE_W_X_GATE, ONE_W_X_EXPERTS, ONE_W_X_BIAS2,
 ONE_W_GATE_UP, ONE_W_GATE_UP_B, ONE_W_DOWN, ONE_W_DOWN_B,
 ONE_W_NORM_W, ONE_W_NORM_B, ONE_W_LAYER_SLOTS) = range(35)
(ONE_G_EMBED, ONE_G_LHS_W, ONE_G_LHS_B, ONE_G_UP_W, ONE_G_UP_B, ONE_G_NORM_W, ONE_G_NORM_B, ONE_G_LM_HEAD,
 ONE_G_SLOTS) = range(9)


class OneConfigC(ctypes.Structure):
    _fields_ = [(n, c_int32) for n in ("vocab_size", "hidden_size", "transformer_dim", "num_hidden_layers",
                                       "num_attention_heads", "head_dim", "intermediate_size", "num_experts",
                                       "top_k", "r", "mlp_bias", "dtype")] + [("rms_norm_eps", c_float),
                                                                              ("rope_theta", c_float),
                                                                              ("use_flash_attention", c_int32)]


# name -> (restype, argtypes); exactly the functions declared in include/one_b200.h
SIGNATURES = {
    "one_abi_version": (c_int, []),
    "one_last_error": (c_char_p, []),
    "one_engine_workspace_bytes": (c_size_t, [POINTER(OneConfigC), c_int32, c_int32, c_int32]),
    "one_engine_create": (c_int, [POINTER(OneConfigC), POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_size_t,
                                  c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int32, POINTER(c_void_p)]),
    "one_engine_destroy": (c_int, [c_void_p]),
    "one_engine_reset": (c_int, [c_void_p, c_int32, c_int32, c_void_p]),
    "one_engine_prefill": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p]),
    "one_engine_step": (c_int, [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "one_engine_capture": (c_int, [c_void_p, c_int32, c_int32, c_void_p]),
    "one_engine_replay": (c_int, [c_void_p, c_void_p]),
    "one_engine_buffer": (c_void_p, [c_void_p, c_char_p]),
    "one_engine_error": (c_int, [c_void_p, POINTER(c_int32), POINTER(c_int32)]),
    "one_engine_step_launches": (c_int32, [c_void_p, c_int32]),
    "one_engine_prefill_launches": (c_int32, [c_void_p, c_int32, c_int32, c_int32]),
    "one_engine_profile_step": (c_int32, [c_void_p, c_int32, c_int32, POINTER(c_float), c_int32, c_void_p]),
    "one_linear_moe_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "one_linear_moe": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "one_linear_moe_noalloc": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "one_moe_routing": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                c_int32, c_void_p, c_void_p, c_void_p]),
    "one_rotary_embedding": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                                     c_void_p]),
    "one_cumsum_and_normalize": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "one_combined_rope_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p,
                                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                            c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "one_flash_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                    c_float, c_int32, c_void_p, c_void_p]),
    "one_rope_flash_attention_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "one_rope_flash_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                         c_int32, c_int32, c_int32, c_float, c_int32, c_void_p, c_void_p, c_size_t,
                                         c_void_p]),
    "one_ops_error": (c_int, [POINTER(c_int32), c_int32]),
    "one_selftest_mean_division": (c_int, [c_void_p, c_int32, c_void_p, c_void_p]),
    "one_sample_tokens": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_float, c_int32, c_float,
                                  ctypes.c_uint64, ctypes.c_uint64, c_void_p, c_void_p]),
}


class OneError(RuntimeError):
    pass


# ONE_B200_ABI_VERSION of include/one_b200.h that the structures above follow
ABI_VERSION = 2


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libone_b200.so not found at {LIB_PATH}; build it with `python medit-one_b200/build.py`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if a declared symbol is missing
        fn.restype = res
        fn.argtypes = args
    if lib.one_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH} has ABI version {lib.one_abi_version()}, this package needs {ABI_VERSION}; "
                          "rebuild it with `python medit-one_b200/build.py`")
    return lib


LIB = _load()


def check(rc: int, what: str = "") -> None:
    if rc != ONE_OK:
        msg = LIB.one_last_error().decode(errors="replace")
        raise OneError(f"{what or 'one_b200'} failed ({rc}): {msg}")


def ptr(t) -> c_void_p:
    """Device (or host) address of a torch tensor, or NULL for None."""
    return c_void_p(0) if t is None else c_void_p(t.data_ptr())


def dtype_code(dt) -> int:
    import torch
    if dt == torch.bfloat16:
        return ONE_DTYPE_BF16
    if dt == torch.float32:
        return ONE_DTYPE_F32
    raise OneError(f"unsupported dtype {dt}: the engine computes in bf16 or fp32")
