"""Parity of the exact configuration bench.py measures: the 140M-class model in bf16
(weights seed 4) at batch 256 after a 128-token prompt (ids seed 4), with the decode kernels
that batch selects (token tiles, split-K counts, the attention/router grid). Checked against
the oracle's running-sum decoder, which restates the reference's cached decode
(one/modeling_one.py:358-387, 857-926) and is pinned to the reference's own outputs.

Tolerances: logits and running means rtol = atol = 2e-2 (bf16); router selections bit-exact
(order included); greedy tokens equal to the oracle's argmax or a near-tie of it
(parity_util). Also a 2048-step decode of the same model with no state drift."""
import pytest
import torch

from conftest import cuda_ok
from parity_util import check_greedy_tokens
from test_gpu_engine import assert_close, make_engine

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

BATCH, PROMPT, SEED = 256, 128, 4


def model():
    from one.configuration_one import config_140m
    from one.initialization import init_state_dict
    cfg = config_140m()
    return cfg, init_state_dict(cfg, SEED, torch.bfloat16)


def test_headline_b256_decode_matches_oracle():
    from oracle import one_oracle as O
    from test_oracle_golden import ocfg
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg, sd = model()
    prompt = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=torch.Generator().manual_seed(SEED))
    forced, greedy = 8, 4
    # the engine exactly as bench.py builds it
    eng = make_engine(cfg, sd, "bf16", max_batch=BATCH, max_tokens=BATCH * PROMPT, hist_cap=64,
                      max_positions=PROMPT + 64)
    eng.prefill(prompt.cuda())
    dec = O.RunningDecoder(sd, ocfg(cfg), torch.bfloat16)
    with torch.no_grad():
        nxt = dec.prefill(prompt, last_only=True).logits[:, -1].argmax(-1)
    # 1) steps fed the oracle's greedy tokens: full logits, last layer's router selections
    for s in range(forced):
        O.ROUTE_LOG = []
        try:
            with torch.no_grad():
                res = dec.step(nxt.view(BATCH, 1))
            log = O.ROUTE_LOG
        finally:
            O.ROUTE_LOG = None
        lg, _ = eng.step(nxt.cuda(), logits=True)
        torch.cuda.synchronize()
        ref = res.logits[:, -1].float()
        assert_close(lg.float().cpu().numpy(), ref.numpy(), "bf16", f"step {s} logits")
        got = eng.router_idx(BATCH).cpu().long()
        for ri, name in enumerate(("hx_moe", "x_moe", "cx_moe")):
            assert torch.equal(got[ri], log[-3 + ri].long()), f"step {s}: last layer {name} selections"
        nxt = ref.argmax(-1)
    P = PROMPT + forced
    st = eng.state()[:, :BATCH].cpu()
    for l in range(cfg.num_hidden_layers):
        assert_close(st[l].numpy() / P, dec.S[l].numpy() / P, "bf16", f"layer {l} running mean")
    assert eng.device_error() == (0, 0)
    # 2) the graph-replayed greedy step bench.py times: its tokens, teacher-forced into a
    #    fresh oracle run over the whole history
    eng.capture(1)
    for _ in range(greedy):
        eng.replay()
    torch.cuda.synchronize()
    assert eng.device_error() == (0, 0)
    hist = eng.history(forced + greedy, BATCH).cpu().T.contiguous()  # inputs of every step
    excused = check_greedy_tokens(O.RunningDecoder(sd, ocfg(cfg), torch.bfloat16), prompt, hist,
                                  what="b256 decode")
    assert excused <= BATCH * (forced + greedy) // 100, f"{excused} near-tie choices"


def test_140m_2048_steps_no_state_drift():
    """2048 single-token steps of the 140M-class model (3 sequences, seeded token stream) against
    the oracle: logits and every layer's running mean at steps 1, 256, 1024 and 2048."""
    from oracle import one_oracle as O
    from test_oracle_golden import ocfg
    torch.set_num_threads(max(1, min(16, torch.get_num_threads())))
    cfg, sd = model()
    B, prompt_len, steps = 3, 16, 2048
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, cfg.vocab_size, (B, prompt_len), generator=g)
    feed = torch.randint(0, cfg.vocab_size, (steps, B), generator=g)
    dec = O.RunningDecoder(sd, ocfg(cfg), torch.bfloat16)
    eng = make_engine(cfg, sd, "bf16", max_batch=B, max_tokens=B * prompt_len, hist_cap=steps + 16,
                      max_positions=prompt_len + steps + 16)
    with torch.no_grad():
        dec.prefill(prompt, last_only=True)
    eng.prefill(prompt.cuda())
    checks = {1, 256, 1024, 2048}
    for s in range(1, steps + 1):
        with torch.no_grad():
            res = dec.step(feed[s - 1].view(B, 1))
        lg, _ = eng.step(feed[s - 1].cuda(), logits=s in checks)
        if s in checks:
            torch.cuda.synchronize()
            assert_close(lg.float().cpu().numpy(), res.logits[:, -1].float().numpy(), "bf16", f"step {s} logits")
            P = prompt_len + s
            st = eng.state()[:, :B].cpu()
            for l in range(cfg.num_hidden_layers):
                assert_close(st[l].numpy() / P, dec.S[l].numpy() / P, "bf16", f"step {s} layer {l} running mean")
    assert eng.counters() == (prompt_len + steps, steps)
    assert eng.device_error() == (0, 0)
