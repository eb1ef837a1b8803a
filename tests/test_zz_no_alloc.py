"""one_linear_moe_noalloc: the LinearMoE operator for callers that cannot allocate device
memory (an FFI host holding only the pointers it is handed, or a process whose device memory
belongs to another runtime's pool). Its scratch is a static array in the library; this test
calls it through the C ABI twice in a row and checks each result against one_linear_moe with a
caller-allocated workspace, at the tolerance the other LinearMoE tests use.

Collected last on purpose (file name), so a run that stops at the first failure has already
run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _params(fin, fout, E, r, seed, dt):
    from one.initialization import moe_params
    return {k: v.cuda().contiguous() for k, v in moe_params(fin, fout, E, r, seed, dt).items()}


def _call(fn_name, x, p, k, with_ws, free_bytes=None):
    """One LinearMoE call through the C ABI. With free_bytes (a list), the device's free memory
    (cudaMemGetInfo) is appended before and after the call itself, all buffers being allocated
    before the first reading."""
    from one import _capi as C
    n, fin = x.shape
    fout, E, r = p["weight"].shape[0], p["experts"].numel(), p["gate"].shape[0]
    code = C.dtype_code(x.dtype)
    out = torch.empty(n, fout, dtype=x.dtype, device="cuda")
    idx = torch.empty(n, min(k, E), dtype=torch.int32, device="cuda")
    args = [C.ptr(x), n, fin, fout, C.ptr(p["weight"]), C.ptr(p["bias"]), C.ptr(p["gate"]), C.ptr(p["experts"]),
            C.ptr(p["bias2"]), E, r, k, code, C.ptr(out), C.ptr(idx)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if with_ws:
        wsb = C.LIB.one_linear_moe_workspace_bytes(n, fin, r, code)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        C.check(C.LIB.one_linear_moe(*args, C.ptr(ws), wsb, stream), "one_linear_moe")
    else:
        torch.cuda.synchronize()
        if free_bytes is not None:
            free_bytes.append(torch.cuda.mem_get_info()[0])
        C.check(getattr(C.LIB, fn_name)(*args, stream), fn_name)
        torch.cuda.synchronize()
        if free_bytes is not None:
            free_bytes.append(torch.cuda.mem_get_info()[0])
    torch.cuda.synchronize()
    return out, idx


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_twice(dt):
    tol = dict(rtol=2e-2, atol=2e-2) if dt == torch.bfloat16 else dict(rtol=1e-5, atol=1e-5)
    # The first call on a device is the set-up call: looking the scratch up loads the library's
    # device code on that device (CUDA loads modules lazily), which is when the static scratch
    # takes its device memory. Every later call must leave the device's free memory unchanged.
    p0 = _params(144, 96, 8, 64, 30, dt)
    _call("one_linear_moe_noalloc", torch.randn(8, 144).to(dt).cuda(), p0, 2, with_ws=False)
    for call, (n, fin, fout, seed) in enumerate([(512, 768, 768, 31), (300, 144, 768, 32)]):
        p = _params(fin, fout, 8, 64, seed, dt)
        x = torch.randn(n, fin, generator=torch.Generator().manual_seed(seed)).to(dt).cuda()
        ref, ref_idx = _call(None, x, p, 2, with_ws=True)
        free = []
        got, got_idx = _call("one_linear_moe_noalloc", x, p, 2, with_ws=False, free_bytes=free)
        np.testing.assert_array_equal(got_idx.cpu().numpy(), ref_idx.cpu().numpy(), err_msg=f"call {call}")
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), err_msg=f"call {call}", **tol)
        # the entry point's contract: the call itself takes no device memory (the device's free
        # bytes are unchanged across it; the scratch was reserved by the set-up call above)
        assert free[0] == free[1], f"call {call}: free device memory {free[0]} -> {free[1]}"


def test_noalloc_rejects_oversized_request():
    from one import _capi as C
    fin = 768
    n = (8 * 1024 * 1024) // (2 * fin) + 1  # the clamped copy alone exceeds the scratch
    rc = C.LIB.one_linear_moe_noalloc(None, n, fin, 768, None, None, None, None, None, 8, 64, 2, C.ONE_DTYPE_BF16,
                                      None, None, None)
    assert rc == C.ONE_ERR_INVALID
    assert b"static scratch" in C.LIB.one_last_error()
