"""Pin the CPU oracle to the reference: every golden fixture under tests/golden/
was produced by the reference itself (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from oracle import one_oracle as O
from one.configuration_one import tiny_config
from one.initialization import init_state_dict, moe_params

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def load(name):
    return np.load(os.path.join(G, name))


def ocfg(cfg):
    return O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, transformer_dim=cfg.transformer_dim,
                          num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                          head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                          top_k_experts=cfg.top_k_experts, r=cfg.r,
                          use_flash_attention=bool(getattr(cfg, "use_flash_attention", False)))


def sd_for(dt):
    cfg = tiny_config()
    # the fixtures were made from fp32 weights cast to the model dtype
    sd = {k: v.to(DT[dt]) for k, v in init_state_dict(cfg, 0, torch.float32).items()}
    return cfg, sd


def check_logits(lg, g, exact):
    lg = lg.float()
    if exact:
        np.testing.assert_array_equal(lg[..., :512].numpy(), g["logits_slice"])
    else:
        np.testing.assert_allclose(lg[..., :512].numpy(), g["logits_slice"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(lg.argmax(-1).numpy(), g["logits_argmax"])
    np.testing.assert_allclose(lg.double().sum(-1).numpy(), g["logits_sum"], rtol=1e-4, atol=1e-2)


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_forward_matches_reference(dt):
    g = load(f"forward_{dt}.npz")
    cfg, sd = sd_for(dt)
    res = O.forward(sd, torch.from_numpy(g["ids"]), ocfg(cfg), DT[dt])
    check_logits(res.logits, g, exact=(dt == "bf16"))
    np.testing.assert_allclose(res.hx.float().numpy(), g["hx"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(res.cx.float().numpy(), g["cx"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
@pytest.mark.parametrize("kind", ["cached", "running"])
def test_decode_matches_reference(dt, kind):
    g = load(f"decode_{dt}.npz")
    cfg, sd = sd_for(dt)
    dec = (O.CachedDecoder if kind == "cached" else O.RunningDecoder)(sd, ocfg(cfg), DT[dt])
    gen, lgs, res = O.greedy(dec, torch.from_numpy(g["prompt"]), g["generated"].shape[1], keep_logits=True)
    np.testing.assert_array_equal(gen.numpy(), g["generated"])
    check_logits(torch.stack(lgs, 0), g, exact=(dt == "bf16"))
    np.testing.assert_allclose(res.hx[:, 0].float().numpy(), g["step_hx"][-1], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(res.cx[:, 0].float().numpy(), g["step_cx"][-1], rtol=1e-6, atol=1e-6)


def test_running_sum_equals_cache_cumsum_long():
    """The O(1) running-sum decode equals the reference's O(P) cumsum decode bit for
    bit, across the bf16 divisor's inexact range (P > 256)."""
    cfg = tiny_config(num_hidden_layers=1, vocab_size=512)
    sd = init_state_dict(cfg, 5, torch.bfloat16)
    oc = ocfg(cfg)
    prompt = torch.randint(0, 512, (2, 250), generator=torch.Generator().manual_seed(9))
    a, la, _ = O.greedy(O.CachedDecoder(sd, oc, torch.bfloat16), prompt, 24, keep_logits=True)
    b, lb, _ = O.greedy(O.RunningDecoder(sd, oc, torch.bfloat16), prompt, 24, keep_logits=True)
    assert torch.equal(a, b)
    for x, y in zip(la, lb):
        assert torch.equal(x, y)


CASES = [("d768", 768, 768, 8, 2, 48, 11), ("d144", 144, 768, 8, 2, 96, 12), ("d16", 16, 256, 4, 2, 64, 13),
         ("e64", 144, 256, 64, 2, 64, 14), ("k3", 768, 256, 8, 3, 64, 15), ("e64k1", 144, 256, 64, 1, 64, 16)]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_linear_moe_matches_reference(case, dt):
    g = load("linear_moe.npz")
    tag, fin, fout, E, k, N, seed = case
    p = moe_params(fin, fout, E, 64, seed, DT[dt])
    x = torch.randn(N, fin, generator=torch.Generator().manual_seed(seed + 100)).to(DT[dt])
    y, idx = O.linear_moe(x, p, k)
    np.testing.assert_array_equal(idx.numpy(), g[f"{tag}_{dt}_idx"])
    np.testing.assert_array_equal(y.float().numpy(), g[f"{tag}_{dt}_y"])
    # the restated selection reproduces the reference's indices, in order
    s = O.linear_moe_scores(x, p).float()
    sel = np.array([O.topk_unsorted(row.tolist(), min(k, E)) for row in s])
    np.testing.assert_array_equal(sel, g[f"{tag}_{dt}_idx"])


def test_topk_all_ties_reference_order():
    g = load("linear_moe.npz")
    for E in (4, 8):
        exp = g[f"alltie_e{E}_idx"]
        got = np.array([O.topk_unsorted([0.0] * E, 2) for _ in range(exp.shape[0])])
        np.testing.assert_array_equal(got, exp)


def test_topk_restatement_random_ties():
    gen = torch.Generator().manual_seed(0)
    for E, k in [(4, 2), (8, 2), (8, 1), (8, 3), (16, 2), (64, 2), (64, 1), (128, 2), (5, 4)]:
        s = torch.randint(0, 3, (400, E), generator=gen).float().bfloat16()
        ref = torch.topk(s, k, dim=-1, sorted=False).indices
        got = torch.tensor([O.topk_unsorted(r.float().tolist(), k) for r in s])
        assert torch.equal(ref, got), (E, k)


@pytest.mark.parametrize("n", [64, 96])
@pytest.mark.parametrize("dt", ["fp32", "bf16"])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_matches_reference(n, dt, causal):
    g = load("attention.npz")
    q, k, v = (torch.from_numpy(g[f"{c}_n{n}"]).to(DT[dt]) for c in "qkv")
    tag = f"n{n}_{dt}_{'c' if causal else 'nc'}"
    np.testing.assert_array_equal(O.exact_attention(q, k, v, causal).float().numpy(), g[f"turbo_{tag}"])
    np.testing.assert_array_equal(O.blockwise_flash_attention(q, k, v, causal).float().numpy(), g[f"flash_{tag}"])


@pytest.mark.parametrize("n,dt", [(200, "fp32"), (200, "bf16"), (300, "bf16")])
@pytest.mark.parametrize("causal", [False, True])
def test_rope_attention_matches_reference(n, dt, causal):
    g = load("attention.npz")
    q, k, v = (torch.from_numpy(g[f"r{c}_n{n}"]).to(DT[dt]) for c in "qkv")
    cos, sin = O.rope_cos_sin(O.rope_inv_freq(64, 10000.0), torch.arange(0, n).unsqueeze(0), DT[dt])
    tag = f"n{n}_{dt}_{'c' if causal else 'nc'}"
    np.testing.assert_array_equal(O.rope_exact_attention(q, k, v, cos, sin, causal).float().numpy(), g[f"rope_{tag}"])


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_ops_match_reference(dt):
    g = load("ops.npz")
    inv = O.rope_inv_freq(64, 10000.0)
    c, s = O.rope_cos_sin(inv, torch.arange(0, 300).unsqueeze(0), DT[dt])
    np.testing.assert_array_equal(c.float().numpy(), g[f"rope_cos_{dt}"])
    np.testing.assert_array_equal(s.float().numpy(), g[f"rope_sin_{dt}"])
    x = torch.from_numpy(g[f"cumsum_x_{dt}"]).to(DT[dt])
    np.testing.assert_array_equal(O.cumsum_and_normalize(x, 50).float().numpy(), g[f"cumsum_y_{dt}"])


def test_divisors_match_reference():
    g = load("ops.npz")["div_bf16"]
    got = O.mean_divisors(torch.bfloat16, 5000, 5000).flatten().float().numpy()
    np.testing.assert_array_equal(got, g)
