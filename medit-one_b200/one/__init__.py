"""MedIT One on B200 (sm_100a): the reference's Python API (OneConfig, OneForCausalLM,
one.turbo_ops, LinearMoE, flash_attention) over a native CUDA engine.

Submodules that need the native library (engine, turbo_ops, modeling_one, ...) load
it on import and raise if it is missing; ``configuration_one`` and
``initialization`` do not need it.
"""
from .configuration_one import OneConfig  # noqa: F401

__all__ = ["OneConfig", "OneForCausalLM", "OneModel", "OneEngine"]


def __getattr__(name):
    if name in ("OneForCausalLM", "OneModel"):
        from . import modeling_one
        return getattr(modeling_one, name)
    if name == "OneEngine":
        from .engine import OneEngine
        return OneEngine
    raise AttributeError(name)
