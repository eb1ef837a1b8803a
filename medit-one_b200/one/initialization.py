"""Parameter inventory and a deterministic random init for MedIT One models.

``param_specs`` lists the parameters of the reference ``OneForCausalLM`` in its
``named_parameters()`` order (one/modeling_one.py:209-316, 614-663, 845-855;
one/linear_moe.py:23-38), with the tied ``lm_head.weight`` folded into
``model.embed_tokens.weight``.

``init_state_dict`` is the seeded init used for every random-init workload:
one ``torch.Generator`` seeded once; walking the list in order, each bias and
``bias2`` is zero, each norm weight is one, and every other tensor (linear
weights, the embedding, LinearMoE ``experts`` and ``gate``) is drawn from
N(0, 0.02) in fp32; the result is cast to the model dtype. Loading the same
state dict into the reference model and into this engine makes the two runs
share weights bit for bit.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch


def param_specs(cfg) -> List[Tuple[str, Tuple[int, ...]]]:
    D = cfg.transformer_dim
    H, Dh = cfg.num_attention_heads, cfg.head_dim
    HD = H * Dh
    HH = H * H
    I = cfg.intermediate_size
    specs: List[Tuple[str, Tuple[int, ...]]] = [("model.embed_tokens.weight", (cfg.vocab_size, cfg.hidden_size))]
    use_moe = cfg.num_experts is not None and cfg.num_experts > 0
    for i in range(cfg.num_hidden_layers):
        p = f"model.decoder_layers.{i}."
        specs += [
            (p + "norm1.weight", (D,)),
            (p + "lin1.weight", (HD, D)), (p + "lin1.bias", (HD,)),
            (p + "lin2.weight", (HD, D)), (p + "lin2.bias", (HD,)),
            (p + "lin3.weight", (HD, D)), (p + "lin3.bias", (HD,)),
            (p + "lin_q.weight", (H, Dh)), (p + "lin_q.bias", (H,)),
            (p + "lin_k.weight", (H, Dh)), (p + "lin_k.bias", (H,)),
            (p + "lin_v.weight", (H, Dh)), (p + "lin_v.bias", (H,)),
            (p + "gate1.weight", (HD, D)), (p + "gate1.bias", (HD,)),
        ]
        for name, fin in (("hx_moe", HH), ("cx_moe", D), ("x_moe", HH)):
            specs += [(p + f"{name}.weight", (D, fin)), (p + f"{name}.bias", (D,))]
            if use_moe:
                E = cfg.num_experts
                specs += [(p + f"{name}.experts", (E,)), (p + f"{name}.bias2", (E, fin)),
                          (p + f"{name}.gate.weight", (cfg.r, fin))]
        specs += [
            (p + "mlp.gate_proj.weight", (I, D)),
            (p + "mlp.up_proj.weight", (I, D)),
            (p + "mlp.down_proj.weight", (D, I)),
            (p + "norm.weight", (D,)), (p + "norm.bias", (D,)),
        ]
        if cfg.mlp_bias:
            specs += [(p + "mlp.gate_proj.bias", (I,)), (p + "mlp.up_proj.bias", (I,)),
                      (p + "mlp.down_proj.bias", (D,))]
    specs += [
        ("model.lhs_norm.weight", (D,)), ("model.lhs_norm.bias", (D,)),
        ("model.up_scaler.weight", (cfg.hidden_size, D)), ("model.up_scaler.bias", (cfg.hidden_size,)),
        ("model.norm.weight", (cfg.hidden_size,)), ("model.norm.bias", (cfg.hidden_size,)),
    ]
    return specs


def _kind(name: str) -> str:
    leaf = name.rsplit(".", 1)[-1]
    if leaf in ("bias", "bias2"):
        return "zero"
    if "norm" in name.rsplit(".", 2)[-2] and leaf == "weight":
        return "one"
    return "normal"


def init_state_dict(cfg, seed: int, dtype: torch.dtype = torch.bfloat16, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Seeded random init (see module docstring). CPU tensors of ``dtype``."""
    g = torch.Generator().manual_seed(seed)
    sd: Dict[str, torch.Tensor] = {}
    for name, shape in param_specs(cfg):
        kind = _kind(name)
        if kind == "zero":
            t = torch.zeros(shape)
        elif kind == "one":
            t = torch.ones(shape)
        else:
            t = torch.empty(shape).normal_(0.0, std, generator=g)
        sd[name] = t.to(dtype)
    return sd


def moe_params(fin: int, fout: int, num_experts: int, r: int, seed: int, dtype: torch.dtype,
               w_std: float = 0.02, experts_std: float = 3.0, bias_std: float = 0.05,
               bias2_std: float = 0.05) -> Dict[str, torch.Tensor]:
    """Seeded LinearMoE parameters that exercise routing: ``experts`` large enough
    that ``1 + silu(score)`` leaves 1.0 in bf16, and nonzero ``bias2`` so the
    per-expert scores differ (one/linear_moe.py:32-38)."""
    g = torch.Generator().manual_seed(seed)
    n = lambda *s, sd: torch.empty(s).normal_(0.0, sd, generator=g)
    p = {
        "weight": n(fout, fin, sd=w_std),
        "bias": n(fout, sd=bias_std),
        "gate": n(r, fin, sd=0.2),
        "experts": n(num_experts, sd=experts_std),
        "bias2": n(num_experts, fin, sd=bias2_std),
    }
    return {k: v.to(dtype) for k, v in p.items()}
