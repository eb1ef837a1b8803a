"""Checkpoint round trip of the kept HF API (no GPU): OneForCausalLM.save_pretrained writes a
safetensors checkpoint with the tied lm_head stored once (one/modeling_one.py:846,
README.md:67-68 `from_pretrained` usage), and from_pretrained restores every parameter bit for
bit (the init pass that transformers runs after loading must not redraw loaded weights) with
lm_head tied to the embedding again."""
import os

import pytest
import torch

from one.configuration_one import OneConfig, tiny_config
from one.initialization import init_state_dict, param_specs
from one.modeling_one import OneForCausalLM


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_save_pretrained_round_trip(tmp_path, dtype):
    from safetensors import safe_open
    cfg = tiny_config()
    model = OneForCausalLM(cfg)
    sd = init_state_dict(cfg, 0, torch.float32)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and set(missing) <= {"lm_head.weight"}
    model = model.to(dtype)
    model.save_pretrained(str(tmp_path))
    with safe_open(os.path.join(str(tmp_path), "model.safetensors"), "pt") as f:
        keys = set(f.keys())
    assert "model.embed_tokens.weight" in keys and "lm_head.weight" not in keys  # tied: stored once
    back = OneForCausalLM.from_pretrained(str(tmp_path))
    assert back.dtype == dtype
    assert back.lm_head.weight.data_ptr() == back.model.embed_tokens.weight.data_ptr()
    a, b = model.state_dict(), back.state_dict()
    assert set(a) == set(b)
    diff = [k for k in a if not torch.equal(a[k], b[k])]
    assert not diff, f"parameters changed by the round trip: {diff[:5]}"
    for name, shape in param_specs(cfg):
        assert tuple(b[name].shape) == tuple(shape)
    assert isinstance(back.config, OneConfig)
    for field in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads", "head_dim",
                  "intermediate_size", "num_experts", "top_k_experts", "r", "use_flash_attention"):
        assert getattr(back.config, field) == getattr(cfg, field), field


def test_reference_state_dict_loads_strictly():
    """A state dict with the reference's parameter names (one/modeling_one.py:209-316, 593-660)
    loads into OneForCausalLM with nothing missing or unexpected."""
    cfg = tiny_config()
    sd = init_state_dict(cfg, 1, torch.float32)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    model = OneForCausalLM(cfg)
    model.load_state_dict(sd, strict=True)
    assert torch.equal(model.lm_head.weight, sd["model.embed_tokens.weight"])
