"""Shared checks of the GPU parity tests.

Greedy tokens are compared by teacher forcing: the oracle is fed the engine's own tokens, and
at every step the engine's choice must be the oracle's argmax, or a near-tie of it: a token
whose oracle logit is within `ulps` units in the last place (of the logits' dtype, at the
maximum) of the oracle's maximum. Logits are rounded to the model dtype, and the engine sums
each logit in a different order than the CPU, so two logits one ulp apart can swap; any other
difference in the choice fails."""
import math

import torch

BF16_TOL = dict(rtol=2e-2, atol=2e-2)


def ulp(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of `dtype` values at |x| (x a float tensor of dtype values)."""
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    e = torch.floor(torch.log2(x.abs().clamp_min(torch.finfo(dtype).tiny)))
    return torch.pow(2.0, e - mant)


def near_tie_ok(logits: torch.Tensor, tok: torch.Tensor, ulps: int = 1):
    """logits [B, V] (oracle, in the model dtype), tok [B] (engine). Returns (ok, excused),
    two [B] bool tensors: ok = argmax or within `ulps` ulps of the maximum; excused = ok but
    not the argmax."""
    lo = logits.float()
    mx, am = lo.max(-1)
    chosen = lo.gather(1, tok.view(-1, 1).long()).squeeze(1)
    exact = tok.long() == am
    near = chosen >= mx - ulps * ulp(mx, logits.dtype)
    return exact | near, near & ~exact


def check_greedy_tokens(decoder, prompt: torch.Tensor, tokens: torch.Tensor, what: str, ulps: int = 1) -> int:
    """decoder: a fresh oracle RunningDecoder. tokens [B, steps]: the engine's greedy inputs,
    tokens[:, 0] being its argmax after the prompt. Returns how many choices were near-ties."""
    B, steps = tokens.shape
    with torch.no_grad():
        logits = decoder.prefill(prompt, last_only=True).logits[:, -1]
        excused = 0
        for s in range(steps):
            tok = tokens[:, s].cpu()
            ok, ex = near_tie_ok(logits, tok, ulps)
            assert bool(ok.all()), (f"{what}: step {s}: {int((~ok).sum())} of {B} tokens are neither the oracle's "
                                    f"argmax nor a near-tie (sequences {(~ok).nonzero().flatten()[:8].tolist()})")
            excused += int(ex.sum())
            logits = decoder.step(tok.view(B, 1)).logits[:, -1]
    return excused
