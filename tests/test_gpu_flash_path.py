"""OneConfig(use_flash_attention=True) on the GPU engine against the oracle's flash branch.

The reference's flash branch (one/modeling_one.py:408-421) under TURBO_MODE runs
TurboFlashAttention(causal=True): turbo_flash_attention's exact causal attention
(one/turbo_ops.py:115-143) over the per-head lin_q / lin_k / lin_v outputs, across the call's
tokens, with head dim = num_attention_heads and scale 1/sqrt(num_attention_heads). Prompt
ingestion therefore attends across each prompt's positions (attn_tok_kernel's q | k | v mode,
then seq_attn_kernel), and a one-token decode call attends to its own token only (o = v in
dec_attn_kernel). Tolerance bf16 rtol = atol = 2e-2; the prompts cross the attention kernel's
64-key and 128-query tiles."""
import numpy as np
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def close(a, b, what, rtol=2e-2, atol=2e-2):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    bad = np.abs(a - b) > atol + rtol * np.abs(b)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance, max |diff| {np.abs(a - b).max():.3g}"


def run(cfg, seed, B, S, steps):
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    from oracle import one_oracle as O
    from test_oracle_golden import ocfg
    cfg.use_flash_attention = True
    sd = init_state_dict(cfg, seed, torch.bfloat16)
    prompt = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(seed))
    oc = ocfg(cfg)
    assert oc.use_flash_attention
    ref = O.forward(sd, prompt, oc, torch.bfloat16)
    gen, lgs, _ = O.greedy(O.RunningDecoder(sd, oc, torch.bfloat16), prompt, steps, keep_logits=True)
    eng = OneEngine(cfg, sd, "cuda", torch.bfloat16, max_batch=B, max_tokens=B * S)
    lg = eng.prefill(prompt.cuda(), logits="all")
    torch.cuda.synchronize()
    assert eng.device_error() == (0, 0)
    close(lg.float().cpu().numpy(), ref.logits.float().numpy(), "prompt logits, every position")
    hx, cx = eng.last_hx_cx(B * S)
    close(hx.float().cpu().view(B, S, -1).numpy(), ref.hx.float().numpy(), "hx")
    close(cx.float().cpu().view(B, S, -1).numpy(), ref.cx.float().numpy(), "cx")
    for s in range(steps):
        out, _ = eng.step(gen[:, s].cuda(), logits=True)
        torch.cuda.synchronize()
        close(out.float().cpu().numpy(), lgs[s].float().numpy(), f"decode step {s} logits")
    assert eng.device_error() == (0, 0)
    # the flag changes the numbers: the feature-attention path gives other logits
    oc.use_flash_attention = False
    other = O.forward(sd, prompt, oc, torch.bfloat16).logits
    assert (other.float() - ref.logits.float()).abs().max() > 0.1


@pytest.mark.parametrize("B,S", [(3, 37), (2, 130)])
def test_flash_path_tiny(B, S):
    from one.configuration_one import tiny_config
    run(tiny_config(), 11, B, S, 3)


def test_flash_path_140m():
    from one.configuration_one import config_140m
    run(config_140m(), 12, 2, 200, 2)
