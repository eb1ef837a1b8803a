"""GPU parity of the standalone operators (LinearMoE, router, RoPE tables, prefix
mean, feature attention, attention) against the reference goldens and the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import cuda_ok
from test_gpu_engine import DT, assert_close, load

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

CASES = [("d768", 768, 768, 8, 2, 48, 11), ("d144", 144, 768, 8, 2, 96, 12), ("d16", 16, 256, 4, 2, 64, 13),
         ("e64", 144, 256, 64, 2, 64, 14), ("k3", 768, 256, 8, 3, 64, 15), ("e64k1", 144, 256, 64, 1, 64, 16)]


def native_linear_moe(x, p, k):
    import ctypes
    from one import _capi as C
    n, fin = x.shape
    fout = p["weight"].shape[0]
    E = p["experts"].numel()
    r = p["gate"].shape[0]
    dt = C.dtype_code(x.dtype)
    out = torch.empty(n, fout, dtype=x.dtype, device="cuda")
    idx = torch.empty(n, min(k, E), dtype=torch.int32, device="cuda")
    wsb = C.LIB.one_linear_moe_workspace_bytes(n, fin, r, dt)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    pc = {kk: v.cuda().contiguous() for kk, v in p.items()}
    C.check(C.LIB.one_linear_moe(C.ptr(x), n, fin, fout, C.ptr(pc["weight"]), C.ptr(pc["bias"]), C.ptr(pc["gate"]),
                                 C.ptr(pc["experts"]), C.ptr(pc["bias2"]), E, r, k, dt, C.ptr(out), C.ptr(idx), C.ptr(ws),
                                 wsb, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "one_linear_moe")
    torch.cuda.synchronize()
    return out, idx


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_linear_moe_matches_reference(case, dt):
    from one.initialization import moe_params
    g = load("linear_moe.npz")
    tag, fin, fout, E, k, N, seed = case
    p = moe_params(fin, fout, E, 64, seed, DT[dt])
    x = torch.randn(N, fin, generator=torch.Generator().manual_seed(seed + 100)).to(DT[dt]).cuda()
    y, idx = native_linear_moe(x, p, k)
    # router indices: bit-exact, in the reference's order
    np.testing.assert_array_equal(idx.cpu().numpy(), g[f"{tag}_{dt}_idx"])
    assert_close(y.float().cpu().numpy(), g[f"{tag}_{dt}_y"], dt, "LinearMoE output")


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_linear_moe_large_matches_oracle(dt):
    """T=16384 x d=768, 8 experts top-2 (the isolated-layer workload), routing-heavy params."""
    from one.initialization import moe_params
    from oracle import one_oracle as O
    p = moe_params(768, 768, 8, 64, 3, DT[dt])
    x = torch.randn(16384, 768, generator=torch.Generator().manual_seed(3)).to(DT[dt])
    y_ref, idx_ref = O.linear_moe(x, p, 2)
    y, idx = native_linear_moe(x.cuda(), p, 2)
    same = (idx.cpu().long() == idx_ref).all(-1)
    assert same.float().mean().item() == 1.0, f"{(~same).sum().item()} tokens routed differently"
    assert_close(y.float().cpu().numpy(), y_ref.float().numpy(), dt, "LinearMoE output")


def test_linear_moe_all_ties_reference_order():
    """Random-init LinearMoE (bias2 = 0, small experts): every score ties; the reference
    keeps the experts std::nth_element leaves in front."""
    from one.initialization import moe_params
    g = load("linear_moe.npz")
    for E in (4, 8):
        p = moe_params(144, 64, E, 64, 1, torch.bfloat16, experts_std=0.02, bias2_std=0.0)
        x = torch.randn(5, 144).bfloat16().cuda()
        _, idx = native_linear_moe(x, p, 2)
        np.testing.assert_array_equal(idx.cpu().numpy(), g[f"alltie_e{E}_idx"])
