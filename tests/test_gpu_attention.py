"""GPU parity of the tensor-core attention and the fused RoPE + attention operator.

Small and ragged shapes are checked against the oracle (the reference's exact attention,
pinned by tests/test_oracle_golden.py) and the reference fixtures; the full isolated
workload (Q/K/V [8, 12, 2048, 64] bf16, RoPE base 1e4 on positions 0..2047) against an fp32
PyTorch attention on the GPU over the same rotated inputs. Tolerances: rtol = atol = 2e-2
in bf16, 1e-5 in fp32.
"""
import numpy as np
import pytest
import torch

from conftest import cuda_ok
from test_gpu_engine import DT, assert_close, load

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _no_device_error():
    from one import turbo_ops
    assert turbo_ops.ops_error() == (0, 0)


@pytest.mark.parametrize("n,dt", [(200, "fp32"), (200, "bf16"), (300, "bf16")])
@pytest.mark.parametrize("causal", [False, True])
def test_rope_attention_matches_reference(n, dt, causal):
    from one import turbo_ops
    from oracle import one_oracle as O
    g = load("attention.npz")
    q, k, v = (torch.from_numpy(g[f"r{c}_n{n}"]).to(DT[dt]).cuda() for c in "qkv")
    cos, sin = O.rope_cos_sin(O.rope_inv_freq(64, 10000.0), torch.arange(0, n).unsqueeze(0), DT[dt])
    out = turbo_ops.turbo_rope_flash_attention(q, k, v, cos.cuda(), sin.cuda(), causal=causal)
    tag = f"n{n}_{dt}_{'c' if causal else 'nc'}"
    assert_close(out.float().cpu().numpy(), g[f"rope_{tag}"], dt, "rope attention")
    _no_device_error()


SHAPES = [(1, 2, 128, 128), (1, 1, 200, 333), (2, 3, 256, 256), (1, 2, 1000, 1000), (1, 1, 513, 77), (1, 1, 1, 1),
          (1, 1, 384, 640)]


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
@pytest.mark.parametrize("causal", [False, True])
def test_tensor_core_attention_matches_oracle(shape, causal):
    from one import turbo_ops
    from oracle import one_oracle as O
    b, h, nq, nk = shape
    gen = torch.Generator().manual_seed(nq * 7 + nk)
    q = torch.randn(b, h, nq, 64, generator=gen).bfloat16()
    k = torch.randn(b, h, nk, 64, generator=gen).bfloat16()
    v = torch.randn(b, h, nk, 64, generator=gen).bfloat16()
    ref = O.exact_attention(q, k, v, causal)
    got = turbo_ops.turbo_flash_attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    assert_close(got.float().cpu().numpy(), ref.float().numpy(), "bf16", "attention")
    _no_device_error()


def test_legacy_one_turbo_attention_uses_same_path():
    import one_turbo
    from oracle import one_oracle as O
    gen = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(2, 2, 256, 64, generator=gen).bfloat16() for _ in range(3))
    got = one_turbo.flash_attention(q.cuda(), k.cuda(), v.cuda(), True, 0.125)
    ref = O.exact_attention(q, k, v, True, 0.125)
    assert_close(got.float().cpu().numpy(), ref.float().numpy(), "bf16", "one_turbo.flash_attention")


def _fp32_attention(qr, kr, v, causal):
    """softmax(q k^T / 8 [+ causal mask]) v in fp32 on the GPU, one batch entry at a time."""
    outs = []
    for i in range(qr.shape[0]):
        s = torch.matmul(qr[i].float(), kr[i].float().transpose(-1, -2)) * 0.125
        if causal:
            n = s.shape[-1]
            s.masked_fill_(torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
        outs.append(torch.matmul(torch.softmax(s, dim=-1), v[i].float()))
    return torch.stack(outs)


@pytest.mark.parametrize("causal", [False, True])
def test_isolated_rope_attention_workload(causal):
    """Q/K/V [8, 12, 2048, 64] bf16 ~ N(0, 1) (seed 2), RoPE base 1e4 over positions 0..2047."""
    from one import turbo_ops
    from oracle import one_oracle as O
    B, H, N, D = 8, 12, 2048, 64
    gen = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(B, H, N, D, generator=gen).bfloat16().cuda() for _ in range(3))
    cos, sin = turbo_ops.turbo_rotary_embedding(q, torch.arange(0, N).unsqueeze(0).cuda(),
                                                O.rope_inv_freq(D, 10000.0).cuda())
    got = turbo_ops.turbo_rope_flash_attention(q, k, v, cos, sin, causal=causal)
    qr, kr = O.apply_rope(q, k, cos, sin)  # the reference's bf16 elementwise RoPE, on the GPU
    ref = _fp32_attention(qr, kr, v, causal)
    diff = (got.float() - ref).abs()
    assert torch.isfinite(got.float()).all()
    assert bool((diff <= 2e-2 + 2e-2 * ref.abs()).all()), f"max abs diff {diff.max().item():.3e}"
    _no_device_error()
