"""Long recurrent decode: 2048 single-token steps carrying the per-layer running state in
HBM, checked against the oracle's running-sum decoder (the reference's cached decode,
one/modeling_one.py:358-387) fed the same seeded token stream. The running mean each layer
consumes and the logits are compared at steps 1, 256, 1024 and 2048: no drift beyond
rtol = atol = 2e-2 in bf16 and 1e-5 in fp32."""
import pytest
import torch

from conftest import cuda_ok
from test_gpu_engine import DT, assert_close, make_engine, tiny_sd

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_2048_steps_no_state_drift(dt):
    from oracle import one_oracle as O
    from test_oracle_golden import ocfg
    torch.set_num_threads(max(1, min(16, torch.get_num_threads())))
    cfg, sd = tiny_sd(dt)
    B, prompt_len, steps = 2, 8, 2048
    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, cfg.vocab_size, (B, prompt_len), generator=g)
    feed = torch.randint(0, cfg.vocab_size, (steps, B), generator=g)
    dec = O.RunningDecoder(sd, ocfg(cfg), DT[dt])
    eng = make_engine(cfg, sd, dt, max_batch=B, max_tokens=B * prompt_len, hist_cap=steps + 16,
                      max_positions=prompt_len + steps + 16)
    with torch.no_grad():
        dec.prefill(prompt)
    eng.prefill(prompt.cuda())
    checks = {1, 256, 1024, 2048}
    for s in range(1, steps + 1):
        with torch.no_grad():
            res = dec.step(feed[s - 1].view(B, 1))
        lg, _ = eng.step(feed[s - 1].cuda(), logits=s in checks)
        if s in checks:
            torch.cuda.synchronize()
            assert_close(lg.float().cpu().numpy(), res.logits[:, -1].float().numpy(), dt, f"step {s} logits")
            P = prompt_len + s  # tokens summed into the state after this step
            st = eng.state()[:, :B].cpu()
            for l in range(cfg.num_hidden_layers):
                assert_close(st[l].numpy() / P, dec.S[l].numpy() / P, dt, f"step {s} layer {l} running mean")
    assert eng.counters() == (prompt_len + steps, steps)
    assert eng.device_error() == (0, 0)
