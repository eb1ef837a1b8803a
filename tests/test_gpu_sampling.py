"""GPU sampling (one_sample_tokens) and OneForCausalLM.generate on the engine.

The kept sets and probabilities are checked against transformers' own logits warpers
(TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper: the sampling branch of
generation/utils.py _get_logits_processor), the draws for determinism and against the warped
softmax's probabilities."""
import math

import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def hf_warp(logits, temperature, top_k, top_p):
    from transformers.generation.logits_process import TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper
    s = logits.float()
    if temperature != 1.0:
        s = TemperatureLogitsWarper(temperature)(None, s)
    if top_k:
        s = TopKLogitsWarper(top_k=top_k, min_tokens_to_keep=1)(None, s)
    if top_p < 1.0:
        s = TopPLogitsWarper(top_p=top_p, min_tokens_to_keep=1)(None, s)
    return s


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_top_k_1_is_argmax(dt):
    from one.engine import sample_tokens
    g = torch.Generator().manual_seed(20)
    lg = torch.randn(64, 32000, generator=g).to(dt)
    got = sample_tokens(lg.cuda(), 0.8, 1, 1.0, seed=5, offset=3).cpu().long()
    kept = hf_warp(lg, 0.8, 1, 1.0) > -math.inf
    assert bool(kept.gather(1, got.view(-1, 1)).all())
    if dt == torch.float32:  # no ties: the single kept token
        assert torch.equal(got, lg.float().argmax(-1))


def test_draws_are_deterministic_per_seed_and_offset():
    from one.engine import sample_tokens
    lg = torch.randn(32, 32000, generator=torch.Generator().manual_seed(21)).cuda()
    a = sample_tokens(lg, 1.0, 0, 1.0, seed=123, offset=7)
    b = sample_tokens(lg, 1.0, 0, 1.0, seed=123, offset=7)
    c = sample_tokens(lg, 1.0, 0, 1.0, seed=123, offset=8)
    assert torch.equal(a, b)
    assert not torch.equal(a, c)


def above_mass(logits, T, k, tok):
    """For each row: the probability mass (float64, after temperature and top-k) of the tokens whose
    score is strictly above the drawn token's. Top-p keeps a token iff this is below top_p."""
    s = hf_warp(logits, T, k, 1.0).double()
    pr = torch.softmax(s, -1)
    st = s.gather(1, tok.view(-1, 1))
    return (pr * (s > st)).sum(-1)


@pytest.mark.parametrize("T,k,p", [(0.7, 50, 0.9), (1.3, 0, 0.5), (1.0, 20, 1.0), (0.5, 0, 0.95)])
def test_draws_stay_in_the_transformers_kept_set(T, k, p):
    """Every draw is a token that transformers' warpers keep. At the top-p boundary transformers
    decides with an fp32 cumulative sum of ~32000 small probabilities (its rounding moves the
    boundary by a few tokens of mass ~1e-6 each); there a draw is also accepted when the exact
    (float64) mass above it is below top_p + 1e-4, which is the rule the kernel computes."""
    from one.engine import sample_tokens
    lg = (2.0 * torch.randn(48, 32000, generator=torch.Generator().manual_seed(22))).to(torch.bfloat16)
    kept = hf_warp(lg, T, k, p) > -math.inf
    kept_k = hf_warp(lg, T, k, 1.0) > -math.inf
    dl = lg.cuda()
    for off in range(40):
        got = sample_tokens(dl, T, k, p, seed=9, offset=off).cpu().long()
        in_hf = kept.gather(1, got.view(-1, 1)).squeeze(1)
        in_k = kept_k.gather(1, got.view(-1, 1)).squeeze(1)
        near = above_mass(lg, T, k, got) < p + 1e-4
        ok = in_hf | (in_k & near)
        assert bool(ok.all()), f"offset {off}: a token outside transformers' kept set"


@pytest.mark.parametrize("T,k,p", [(1.0, 0, 1.0), (0.8, 3, 1.0), (1.2, 0, 0.8)])
def test_draw_frequencies_match_the_warped_softmax(T, k, p):
    """20000 rows of one logits vector (each row its own Philox counter): the frequency of each
    token matches softmax(warped scores) within 5 standard errors."""
    from one.engine import sample_tokens
    V, n = 32000, 20000
    row = torch.full((V,), -30.0)
    row[[7, 1000, 31999, 4242, 12]] = torch.tensor([2.0, 1.5, 1.0, 0.3, -0.5])
    probs = torch.softmax(hf_warp(row.view(1, -1), T, k, p), -1)[0].double()
    got = sample_tokens(row.view(1, -1).expand(n, V).contiguous().cuda(), T, k, p, seed=31, offset=0).cpu().long()
    freq = torch.bincount(got, minlength=V).double() / n
    se = torch.sqrt(probs * (1 - probs) / n) + 1e-4
    bad = (freq - probs).abs() > 5 * se
    assert not bool(bad.any()), [(int(i), float(freq[i]), float(probs[i])) for i in bad.nonzero().flatten()[:5]]


def test_generate_greedy_and_sampling():
    """OneForCausalLM.generate: do_sample=False equals generate_greedy; do_sample=True with a seed
    repeats itself, and with top_k=1 picks the oracle's maximum (or a token tied with it) at
    every step; eos ends sequences with pad."""
    from one.configuration_one import tiny_config
    from one.initialization import init_state_dict
    from one.modeling_one import OneForCausalLM
    from oracle import one_oracle as O
    from parity_util import check_greedy_tokens
    from test_oracle_golden import ocfg
    cfg = tiny_config()
    sd = init_state_dict(cfg, 0, torch.float32)
    model = OneForCausalLM(cfg)
    model.load_state_dict(sd, strict=False)
    model = model.to(torch.bfloat16).cuda()
    ids = torch.randint(1, cfg.vocab_size, (3, 10), generator=torch.Generator().manual_seed(23)).cuda()
    greedy = model.generate(ids, max_new_tokens=12, do_sample=False, temperature=0.7)
    assert greedy.shape == (3, 22)
    assert torch.equal(greedy, model.generate_greedy(ids, 12))
    a = model.generate(ids, max_new_tokens=12, do_sample=True, temperature=0.7, top_p=0.9, seed=4)
    b = model.generate(ids, max_new_tokens=12, do_sample=True, temperature=0.7, top_p=0.9, seed=4)
    assert torch.equal(a, b) and torch.equal(a[:, :10], ids)
    k1 = model.generate(ids, max_new_tokens=12, do_sample=True, top_k=1, seed=5)
    sd16 = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    check_greedy_tokens(O.RunningDecoder(sd16, ocfg(cfg), torch.bfloat16), ids.cpu(), k1[:, 10:].cpu(),
                        what="top_k=1 sampling", ulps=0)
    # eos: the first greedy token of sequence 0 as eos; its later tokens become pad
    eos = int(greedy[0, 10])
    e = model.generate(ids, max_new_tokens=12, do_sample=False, eos_token_id=eos, pad_token_id=0)
    assert int(e[0, 10]) == eos and bool((e[0, 11:] == 0).all())
