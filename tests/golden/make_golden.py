"""Generate the golden fixtures in this directory by running the MedIT One
reference itself (its PyTorch CPU path) on seeded inputs.

Usage:  python tests/golden/make_golden.py /path/to/reference
        (or set ONE_REFERENCE_DIR to the reference source tree)

The reference targets transformers 4.x; on the installed transformers 5.5 it
needs three patches, applied here before any model is built and without editing
the reference:
  1. ``ROPE_INIT_FUNCTIONS["default"]`` (removed in v5; used at
     one/modeling_one.py:117-121) is restored as the standard default init
     ``inv_freq = 1 / theta ** (arange(0, d, 2) / d)``, scaling 1.0;
  2. ``OneConfig.__post_init__`` is routed to the base class (the reference's
     takes no kwargs, one/configuration_one.py:63-66);
  3. ``OneForCausalLM._tied_weights_keys`` becomes the v5 dict form
     (one/modeling_one.py:846).
Weights come from ``one.initialization.init_state_dict`` of this repository
(loaded into the reference model), so the engine's tests can rebuild them from
the seed alone. Outputs are small slices and statistics, not whole logits.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ONE_REFERENCE_DIR")
if not REF or not os.path.isdir(os.path.join(REF, "one")):
    sys.exit("usage: make_golden.py /path/to/reference (the MedIT One source tree, holding one/)")


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


init_mod = _load("one_b200_initialization", os.path.join(REPO, "medit-one_b200", "one", "initialization.py"))

sys.path.insert(0, REF)
from transformers import PreTrainedConfig  # noqa: E402
from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS  # noqa: E402


def _default_rope(config, device=None, **kw):
    dim = config.head_dim
    inv = 1.0 / (config.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(device=device, dtype=torch.float) / dim))
    return inv, 1.0


ROPE_INIT_FUNCTIONS.setdefault("default", _default_rope)
from one import configuration_one, flash_attention, linear_moe, modeling_one, turbo_ops  # noqa: E402

configuration_one.OneConfig.__post_init__ = lambda self, **kw: PreTrainedConfig.__post_init__(self, **kw)
modeling_one.OneForCausalLM._tied_weights_keys = {"lm_head.weight": "model.embed_tokens.weight"}

TINY = dict(vocab_size=32000, hidden_size=256, transformer_dim=256, num_hidden_layers=2, num_attention_heads=4,
            head_dim=64, intermediate_size=1024, num_experts=4, top_k_experts=2, r=64, use_flash_attention=False)


def build(dtype, seed=0, **over):
    kw = dict(TINY)
    kw.update(over)
    cfg = configuration_one.OneConfig(**kw)
    m = modeling_one.OneForCausalLM(cfg).eval()
    sd = init_mod.init_state_dict(cfg, seed, torch.float32)
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert set(missing) <= {"lm_head.weight"}, missing
    assert m.lm_head.weight.data_ptr() == m.model.embed_tokens.weight.data_ptr()
    return m.to(dtype), cfg


def last_layer_hook(m, store):
    def hook(mod, args, out):
        store["hx"], store["cx"] = out[1][0].detach().float().clone(), out[1][1].detach().float().clone()
    return m.model.decoder_layers[-1].register_forward_hook(hook)


def f32(t):
    return t.detach().float().numpy()


def logits_stats(lg):
    lg = lg.detach().float()
    return dict(logits_slice=f32(lg[..., :512]), logits_argmax=lg.argmax(-1).numpy(),
                logits_sum=lg.double().sum(-1).numpy(), logits_absmax=lg.abs().amax(-1).numpy())


def gen_forward():
    ids = torch.randint(0, 32000, (2, 64), generator=torch.Generator().manual_seed(1))
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        m, cfg = build(dt)
        store = {}
        h = last_layer_hook(m, store)
        with torch.no_grad():
            out = m(input_ids=ids, use_cache=False)
        h.remove()
        np.savez_compressed(os.path.join(HERE, f"forward_{name}.npz"), ids=ids.numpy(), hx=f32(store["hx"]),
                            cx=f32(store["cx"]), **logits_stats(out.logits))
        print("forward", name, out.logits.shape)


def gen_decode():
    from transformers.cache_utils import DynamicCache
    ids = torch.randint(0, 32000, (3, 12), generator=torch.Generator().manual_seed(7))
    steps = 10
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        m, cfg = build(dt)
        store = {}
        h = last_layer_hook(m, store)
        cache = DynamicCache()
        with torch.no_grad():
            out = m(input_ids=ids, past_key_values=cache, use_cache=True)
            nxt = out.logits[:, -1].argmax(-1)
            gen, lgs, hxs, cxs = [], [], [], []
            for _ in range(steps):
                gen.append(nxt)
                out = m(input_ids=nxt[:, None], past_key_values=cache, use_cache=True)
                lgs.append(out.logits[:, 0].float())
                hxs.append(store["hx"][:, 0])
                cxs.append(store["cx"][:, 0])
                nxt = out.logits[:, -1].argmax(-1)
        h.remove()
        lg = torch.stack(lgs, 0)
        np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"), prompt=ids.numpy(),
                            generated=torch.stack(gen, 1).numpy(), step_hx=f32(torch.stack(hxs, 0)),
                            step_cx=f32(torch.stack(cxs, 0)), **logits_stats(lg))
        print("decode", name, lg.shape)


def gen_linear_moe():
    out = {}
    cases = [("d768", 768, 768, 8, 2, 48, 11), ("d144", 144, 768, 8, 2, 96, 12), ("d16", 16, 256, 4, 2, 64, 13),
             ("e64", 144, 256, 64, 2, 64, 14), ("k3", 768, 256, 8, 3, 64, 15), ("e64k1", 144, 256, 64, 1, 64, 16)]
    for tag, fin, fout, E, k, N, seed in cases:
        for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            p = init_mod.moe_params(fin, fout, E, 64, seed, dt)
            mod = linear_moe.LinearMoE(fin, fout, bias=True, num_experts=E, top_k=k, r=64).to(dt)
            with torch.no_grad():
                mod.weight.copy_(p["weight"]); mod.bias.copy_(p["bias"]); mod.gate.weight.copy_(p["gate"])
                mod.experts.copy_(p["experts"]); mod.bias2.copy_(p["bias2"])
            x = torch.randn(N, fin, generator=torch.Generator().manual_seed(seed + 100)).to(dt)
            # capture the reference's top-k indices through torch.topk
            captured = {}
            orig_topk = torch.topk

            def spy(*a, **kw):
                r = orig_topk(*a, **kw)
                captured["idx"] = r.indices.clone()
                return r
            torch.topk = spy
            try:
                with torch.no_grad():
                    y = mod(x)
            finally:
                torch.topk = orig_topk
            out[f"{tag}_{name}_y"] = f32(y)
            out[f"{tag}_{name}_idx"] = captured["idx"].numpy().astype(np.int16)
    # the degenerate init of random-init models: all expert scores tie
    for E in (4, 8):
        s = torch.zeros(5, E, dtype=torch.bfloat16)
        out[f"alltie_e{E}_idx"] = torch.topk(s, 2, dim=-1, sorted=False).indices.numpy().astype(np.int16)
    np.savez_compressed(os.path.join(HERE, "linear_moe.npz"), **out)
    print("linear_moe", len(out))


def gen_attention():
    out = {}
    g = torch.Generator().manual_seed(2)
    for N in (64, 96):
        q, k, v = (torch.randn(1, 2, N, 64, generator=g) for _ in range(3))
        for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            qq, kk, vv = q.to(dt), k.to(dt), v.to(dt)
            for causal in (False, True):
                tag = f"n{N}_{name}_{'c' if causal else 'nc'}"
                out[f"turbo_{tag}"] = f32(turbo_ops.turbo_flash_attention(qq, kk, vv, causal=causal))
                out[f"flash_{tag}"] = f32(flash_attention.FlashAttentionFunction.apply(qq, kk, vv, 0.0, causal))
        out[f"q_n{N}"], out[f"k_n{N}"], out[f"v_n{N}"] = f32(q), f32(k), f32(v)
    # RoPE + attention across several 128-key tiles with a ragged end: the reference's
    # rotary embedding (turbo_rotary_embedding_cpu), apply_rotary_pos_emb_flash and the exact
    # PyTorch path of turbo_flash_attention, in that order.
    g = torch.Generator().manual_seed(21)
    inv = _default_rope(configuration_one.OneConfig(**TINY))[0]
    for N, dts in ((200, ("fp32", "bf16")), (300, ("bf16",))):
        q, k, v = (torch.randn(1, 2, N, 64, generator=g) for _ in range(3))
        pos = torch.arange(0, N).unsqueeze(0)
        for name in dts:
            dt = torch.float32 if name == "fp32" else torch.bfloat16
            qq, kk, vv = q.to(dt), k.to(dt), v.to(dt)
            c, s = turbo_ops.turbo_rotary_embedding_cpu(qq, pos, inv)
            qr, kr = flash_attention.apply_rotary_pos_emb_flash(qq, kk, c, s)
            for causal in (False, True):
                tag = f"n{N}_{name}_{'c' if causal else 'nc'}"
                out[f"rope_{tag}"] = f32(turbo_ops.turbo_flash_attention(qr, kr, vv, causal=causal))
        out[f"rq_n{N}"], out[f"rk_n{N}"], out[f"rv_n{N}"] = f32(q), f32(k), f32(v)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)
    print("attention", len(out))


def gen_ops():
    out = {}
    g = torch.Generator().manual_seed(3)
    inv = _default_rope(configuration_one.OneConfig(**TINY))[0]
    pos = torch.arange(0, 300).unsqueeze(0)
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        x = torch.randn(1, 300, 64, generator=g).to(dt)
        c, s = turbo_ops.turbo_rotary_embedding_cpu(x, pos, inv)
        out[f"rope_cos_{name}"], out[f"rope_sin_{name}"] = f32(c), f32(s)
        xs = torch.randn(2, 50, 32, generator=g).to(dt)
        out[f"cumsum_x_{name}"] = f32(xs)
        out[f"cumsum_y_{name}"] = f32(turbo_ops.turbo_cumsum_and_normalize_cpu(xs, 50, dt))
        # turbo_combined_rope_attention_cpu (one/turbo_ops.py:382-434) raises NameError in the
        # reference (rotate_half is not imported there); the model's in-line feature attention it
        # restates (one/modeling_one.py:515-547) is pinned through the forward/decode fixtures.
    # the reference's running-mean divisors in bf16 (one/modeling_one.py:379-387)
    out["div_bf16"] = torch.arange(1, 5001, dtype=torch.bfloat16).float().numpy()
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)
    print("ops", len(out))


if __name__ == "__main__":
    torch.set_num_threads(8)
    gen_forward()
    gen_decode()
    gen_linear_moe()
    gen_attention()
    gen_ops()
