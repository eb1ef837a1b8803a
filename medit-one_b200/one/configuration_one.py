"""OneConfig: the MedIT One model configuration (same fields and defaults as the
reference's one/configuration_one.py:24-56).

The reference declares the config as a ``@dataclass`` over
``transformers.PretrainedConfig``, which transformers 5 no longer accepts; this
class keeps every field name, default and meaning and stores them the classic
way, so ``OneConfig(**kwargs)``, ``to_dict`` / ``from_dict`` and
``save_pretrained`` / ``from_pretrained`` all work on the installed stack.
"""
from __future__ import annotations

from typing import Optional

from transformers import PretrainedConfig

_FIELDS = dict(
    vocab_size=28886,
    num_hidden_layers=32,
    hidden_size=1024,
    transformer_dim=512,
    intermediate_size=4096,
    conv_filters=4,
    num_attention_heads=32,
    scale_factor=4,
    dropout=0.02,
    lstm_dropout=0.01,
    conv_activation="silu",
    rms_norm_eps=1e-6,
    use_cache=False,
    with_hx=True,
    head_dim=32,
    max_model_length=32768,
    lm_head_embedding=False,
    num_of_tokens_to_predict=1,
    rope_theta=10000.0,
    rope_scaling=None,
    max_position_embeddings=32768,
    hidden_act="gelu",
    mlp_bias=False,
    use_flash_attention=False,
    use_single_token=False,
    num_experts=None,
    top_k_experts=2,
    r=64,
)


class OneConfig(PretrainedConfig):
    model_type = "one"

    def __init__(self, pad_token_id: int = 0, tie_word_embeddings: bool = True, **kwargs):
        for name, default in _FIELDS.items():
            setattr(self, name, kwargs.pop(name, default))
        if self.rope_scaling is not None and "type" in self.rope_scaling:
            self.rope_scaling["rope_type"] = self.rope_scaling["type"]
        super().__init__(pad_token_id=pad_token_id, tie_word_embeddings=tie_word_embeddings, **kwargs)

    # The reference reads these through PretrainedConfig in transformers 4.x.
    @property
    def use_moe(self) -> bool:
        return self.num_experts is not None and self.num_experts > 0

    def to_dict(self):
        d = super().to_dict()
        for name in _FIELDS:
            d[name] = getattr(self, name)
        return d


def tiny_config(**over) -> OneConfig:
    """The tiny CPU-runnable configuration: vocab 32000, hidden 256, 2 layers,
    4 heads of 64, 4 experts top-2, FFN 1024."""
    kw = dict(vocab_size=32000, hidden_size=256, transformer_dim=256, num_hidden_layers=2,
              num_attention_heads=4, head_dim=64, intermediate_size=1024, num_experts=4,
              top_k_experts=2, r=64, use_flash_attention=False)
    kw.update(over)
    return OneConfig(**kw)


def config_140m(**over) -> OneConfig:
    """The 140M-class configuration: vocab 32000, hidden 768, 12 layers, 12 heads
    of 64, 8 experts top-2, FFN 3072."""
    kw = dict(vocab_size=32000, hidden_size=768, transformer_dim=768, num_hidden_layers=12,
              num_attention_heads=12, head_dim=64, intermediate_size=3072, num_experts=8,
              top_k_experts=2, r=64, use_flash_attention=False)
    kw.update(over)
    return OneConfig(**kw)
