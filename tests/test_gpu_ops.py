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


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_router_clamps_large_inputs_like_reference(dt):
    """Inputs beyond +-1e4 (one/linear_moe.py:53): x.clamp(-1e4, 1e4) of a bf16 tensor gives
    bf16(1e4) = 9984. Through the LinearMoE op, and through the router entry on the unclamped
    input with the reference's gate logits (the router applies the clamp itself)."""
    import ctypes
    import torch.nn.functional as F
    from one import _capi as C
    from one.initialization import moe_params
    from oracle import one_oracle as O
    p = moe_params(144, 64, 8, 64, 7, DT[dt])
    x = (torch.randn(256, 144, generator=torch.Generator().manual_seed(7)) * 8000.0).to(DT[dt])
    assert (x.float().abs() > 1e4).float().mean() > 0.1
    y_ref, idx_ref = O.linear_moe(x, p, 2)
    y, idx = native_linear_moe(x.cuda(), p, 2)
    np.testing.assert_array_equal(idx.cpu().long().numpy(), idx_ref.numpy())
    # outputs ~1e3: the absolute tolerance scales with the largest output (fp32 sums of
    # 144 terms of ~1e2 differ by ~1e-3 between summation orders)
    yr = y_ref.float().numpy()
    tol = {"fp32": 1e-5, "bf16": 2e-2}[dt]
    np.testing.assert_allclose(y.float().cpu().numpy(), yr, rtol=tol, atol=tol * np.abs(yr).max())
    gl = F.linear(x.clamp(-1e4, 1e4), p["gate"]).cuda()
    pc = {kk: v.cuda().contiguous() for kk, v in p.items()}
    xd = x.cuda()
    comb = torch.empty(256, 144, dtype=DT[dt], device="cuda")
    idx2 = torch.empty(256, 2, dtype=torch.int32, device="cuda")
    C.check(C.LIB.one_moe_routing(C.ptr(xd), 256, 144, C.ptr(gl), C.ptr(pc["experts"]), C.ptr(pc["bias2"]), 8, 64, 2,
                                  C.dtype_code(DT[dt]), C.ptr(comb), C.ptr(idx2),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "one_moe_routing")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx2.cpu().long().numpy(), idx_ref.numpy())


def test_prefix_mean_division_is_exact():
    """The prompt path divides the bf16 prefix sums by the position divisors through a
    reciprocal table and one residual correction: identical to the fp32 division for every
    bf16 dividend and every divisor of positions 1..16384."""
    import ctypes
    from one import _capi as C
    from one.engine import prompt_divisors
    div = torch.unique(prompt_divisors(16384, torch.bfloat16)).cuda()
    mism = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    C.check(C.LIB.one_selftest_mean_division(C.ptr(div), div.numel(), C.ptr(mism),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "one_selftest_mean_division")
    assert div.numel() > 500
    assert mism.cpu().tolist() == [0, 0]


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


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_rotary_and_cumsum_match_reference(dt):
    from one import turbo_ops
    g = load("ops.npz")
    from oracle import one_oracle as O
    inv = O.rope_inv_freq(64, 10000.0).cuda()
    x = torch.zeros(1, 300, 64, dtype=DT[dt], device="cuda")
    c, s = turbo_ops.turbo_rotary_embedding(x, torch.arange(0, 300).unsqueeze(0).cuda(), inv)
    assert_close(c.float().cpu().numpy(), g[f"rope_cos_{dt}"], dt, "cos")
    assert_close(s.float().cpu().numpy(), g[f"rope_sin_{dt}"], dt, "sin")
    xs = torch.from_numpy(g[f"cumsum_x_{dt}"]).to(DT[dt]).cuda()
    y = turbo_ops.turbo_cumsum_and_normalize(xs, 50)
    assert_close(y.float().cpu().numpy(), g[f"cumsum_y_{dt}"], dt, "cumsum_and_normalize")


@pytest.mark.parametrize("n", [64, 96])
@pytest.mark.parametrize("dt", ["bf16", "fp32"])
@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_matches_reference(n, dt, causal):
    from one import turbo_ops
    g = load("attention.npz")
    q, k, v = (torch.from_numpy(g[f"{c}_n{n}"]).to(DT[dt]).cuda() for c in "qkv")
    out = turbo_ops.turbo_flash_attention(q, k, v, causal=causal)
    tag = f"n{n}_{dt}_{'c' if causal else 'nc'}"
    assert_close(out.float().cpu().numpy(), g[f"turbo_{tag}"], dt, "attention")


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_combined_rope_attention_matches_oracle(dt):
    from one import turbo_ops
    import one_turbo
    from oracle import one_oracle as O
    gen = torch.Generator().manual_seed(5)
    H, Dh, B, T = 12, 64, 3, 4
    sx, ky, va = (torch.randn(B, H, T, Dh, generator=gen).to(DT[dt]) for _ in range(3))
    lins = [torch.nn.Linear(Dh, H).to(DT[dt]) for _ in range(3)]
    with torch.no_grad():
        for lin in lins:
            lin.weight.copy_(torch.randn(H, Dh, generator=gen) * 0.1)
            lin.bias.copy_(torch.randn(H, generator=gen) * 0.1)
    cos, sin = O.rope_cos_sin(O.rope_inv_freq(Dh, 1e4), torch.arange(7, 7 + T).unsqueeze(0), DT[dt])
    with torch.no_grad():
        ref = O.feature_attention(sx, ky, va, cos, sin, *[(l.weight, l.bias) for l in lins])
    import copy
    with torch.no_grad():
        got = turbo_ops.turbo_combined_rope_attention(sx.cuda(), ky.cuda(), va.cuda(), cos.cuda(), sin.cuda(),
                                                      *[copy.deepcopy(l).cuda() for l in lins], T)
    assert_close(got.float().cpu().numpy(), ref.float().numpy(), dt, "combined rope attention")
    # the legacy one_turbo signature: transposed weights, no biases
    nob = [(l.weight.detach(), None) for l in lins]
    with torch.no_grad():
        ref2 = O.feature_attention(sx, ky, va, cos, sin, *nob)
    with torch.no_grad():
        got2 = one_turbo.combined_rope_attention(sx.cuda(), ky.cuda(), va.cuda(), cos.cuda(), sin.cuda(),
                                                 *[l.weight.t().cuda() for l in lins], T)
    assert_close(got2.float().cpu().numpy(), ref2.float().numpy(), dt, "one_turbo.combined_rope_attention")


def test_linear_moe_module_matches_reference():
    from one.initialization import moe_params
    from one.linear_moe import LinearMoE
    g = load("linear_moe.npz")
    tag, fin, fout, E, k, N, seed = CASES[0]
    p = moe_params(fin, fout, E, 64, seed, torch.bfloat16)
    m = LinearMoE(fin, fout, bias=True, num_experts=E, top_k=k, r=64).to(torch.bfloat16)
    with torch.no_grad():
        m.weight.copy_(p["weight"]); m.bias.copy_(p["bias"]); m.gate.weight.copy_(p["gate"])
        m.experts.copy_(p["experts"]); m.bias2.copy_(p["bias2"])
    m = m.cuda()
    x = torch.randn(N, fin, generator=torch.Generator().manual_seed(seed + 100)).to(torch.bfloat16).cuda()
    y = m(x)
    np.testing.assert_array_equal(m.last_indices.cpu().numpy(), g[f"{tag}_bf16_idx"])
    assert_close(y.float().cpu().numpy(), g[f"{tag}_bf16_y"], "bf16", "LinearMoE module")


def test_causal_lm_api_matches_reference():
    """OneForCausalLM (same parameter names as the reference) loads the seeded state dict and
    reproduces the reference's logits, cached decode and greedy tokens."""
    from one.configuration_one import tiny_config
    from one.initialization import init_state_dict
    from one.modeling_one import OneEngineCache, OneForCausalLM
    g = load("forward_bf16.npz")
    cfg = tiny_config()
    model = OneForCausalLM(cfg)
    sd = init_state_dict(cfg, 0, torch.float32)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and set(missing) <= {"lm_head.weight"}
    model = model.to(torch.bfloat16).cuda()
    out = model(input_ids=torch.from_numpy(g["ids"]).cuda())
    assert_close(out.logits.float().cpu()[..., :512].numpy(), g["logits_slice"], "bf16", "forward logits")
    d = load("decode_bf16.npz")
    cache = OneEngineCache()
    model(input_ids=torch.from_numpy(d["prompt"]).cuda(), past_key_values=cache, use_cache=True)
    gen = torch.from_numpy(d["generated"]).cuda()
    for s in range(gen.shape[1]):
        out = model(input_ids=gen[:, s:s + 1], past_key_values=cache, use_cache=True)
        assert_close(out.logits[:, 0].float().cpu()[:, :512].numpy(), d["logits_slice"][s], "bf16", f"decode {s}")
    seq = model.generate_greedy(torch.from_numpy(d["prompt"]).cuda(), gen.shape[1])
    # each generated token is the oracle's argmax given the same prefix, or a near-tie of it
    from oracle import one_oracle as O
    from parity_util import check_greedy_tokens
    from test_oracle_golden import ocfg
    sd16 = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    excused = check_greedy_tokens(O.RunningDecoder(sd16, ocfg(cfg), torch.bfloat16), torch.from_numpy(d["prompt"]),
                                  seq[:, 12:].cpu(), what="generate_greedy")
    if excused == 0:
        assert (seq[:, 12:].cpu().numpy() == d["generated"]).all()
