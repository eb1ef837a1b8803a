"""Host-side logic that needs no GPU: the running-mean divisor table and the engine's
refusal of OneConfig switches it does not compute."""
import random

import pytest
import torch

from one.configuration_one import tiny_config
from one.engine import OneEngine, check_supported, decode_divisors


def test_decode_divisors_equal_reference_arange_above_4096():
    """The decode step divides the running sum by ``torch.arange(1, P + 1, dtype)[-1] + 1e-10``
    (one/modeling_one.py:379-387). In bf16 the value of that last element depends on how the
    host's arange kernel splits the range into vector chunks and a scalar tail, so the table
    must equal arange at every position, including positions that are not multiples of 16
    and positions above 32768 (config 5 decodes up to P = 36864)."""
    P = 40000
    table = decode_divisors(P, torch.bfloat16)
    rng = random.Random(1234)
    sample = rng.sample(range(4097, P + 1), 2000)
    sample += [p for p in range(32769, P + 1) if p % 256 == 129]  # a tail boundary seen on AVX-512 hosts
    sample += [4097, 4113, 16385, 32767, 32768, 32769, 36864, P]
    for p in sample:
        ref = float((torch.arange(1, p + 1, dtype=torch.bfloat16)[-1:] + 1e-10).float()[0])
        assert float(table[p]) == ref, (p, float(table[p]), ref)
    assert sum(1 for p in sample if p % 16) > 1500


def test_decode_divisors_fp32_are_positions():
    t = decode_divisors(5000, torch.float32)
    assert float(t[0]) == 1.0 and float(t[4097]) == 4097.0


@pytest.mark.parametrize("flag,dtype", [("use_single_token", torch.bfloat16), ("use_flash_attention", torch.float32)])
def test_unsupported_switches_raise(flag, dtype):
    """The engine refuses the switches whose reference path it does not compute (use_single_token;
    use_flash_attention outside bf16), before it touches a device, instead of silently returning
    the default path's numbers."""
    cfg = tiny_config()
    setattr(cfg, flag, True)
    with pytest.raises(NotImplementedError, match=flag):
        check_supported(cfg, dtype)
    with pytest.raises(NotImplementedError, match=flag):
        OneEngine(cfg, {}, "cpu", dtype)


def test_default_switches_accepted():
    check_supported(tiny_config())
    cfg = tiny_config()
    cfg.use_flash_attention = True
    check_supported(cfg, torch.bfloat16)
