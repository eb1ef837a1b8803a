"""OneForCausalLM / OneModel with the reference's module tree and parameter names
(one/modeling_one.py:55-944), so reference checkpoints and state dicts load unchanged.

The forward pass runs on the B200 engine (one.engine.OneEngine, libone_b200.so): a call
without a cache ingests the prompt (prefix-mean semantics of a cache-free forward,
:671-826); with a `OneEngineCache` the first call ingests the prompt and every later
single-token call is one decode step that carries the per-layer running state in HBM
(the reference's DynamicCache history reduced to an O(1) running sum). There is no CPU path.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import nn
from transformers import PreTrainedModel
from transformers.generation import GenerationMixin
from transformers.modeling_outputs import BaseModelOutputWithPast, CausalLMOutputWithPast

from .configuration_one import OneConfig
from .linear_moe import LinearMoE


try:  # transformers >= 5: init helpers that skip parameters loaded from a checkpoint
    from transformers import initialization as _init
except ImportError:  # transformers 4.x initialises only missing parameters itself
    _init = nn.init


class OneRMSNorm(nn.Module):
    """Parameters of one/modeling_one.py:55-70."""

    def __init__(self, dim: int, bias: bool = False, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim)) if bias else 0

    def extra_repr(self):
        return f"{tuple(self.weight.shape)}, eps={self.eps}"


class OneMLP(nn.Module):
    """Parameters of one/modeling_one.py:188-206."""

    def __init__(self, config):
        super().__init__()
        self.hidden_size = config.transformer_dim
        self.intermediate_size = config.intermediate_size
        self.gate_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=config.mlp_bias)
        self.up_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=config.mlp_bias)
        self.down_proj = nn.Linear(self.intermediate_size, self.hidden_size, bias=config.mlp_bias)


class One(nn.Module):
    """The per-layer block's parameters (one/modeling_one.py:209-316). Its computation runs
    inside the engine's layer kernels."""

    def __init__(self, config: OneConfig, dropout: float = 0.1, layer_idx: int = 0, with_hx: bool = True):
        super().__init__()
        self.hidden_size = config.transformer_dim
        self.num_attention_heads = config.num_attention_heads
        self.head_dim = config.head_dim
        self.layer_idx = layer_idx
        self.scaled_dim = self.num_attention_heads * self.head_dim
        self.norm1 = OneRMSNorm(self.hidden_size)
        self.lin1 = nn.Linear(self.hidden_size, self.scaled_dim)
        self.lin2 = nn.Linear(self.hidden_size, self.scaled_dim)
        self.lin3 = nn.Linear(self.hidden_size, self.scaled_dim)
        self.attention_scale = 1.0 / math.sqrt(self.head_dim)
        self.lin_q = nn.Linear(self.head_dim, self.num_attention_heads)
        self.lin_k = nn.Linear(self.head_dim, self.num_attention_heads)
        self.lin_v = nn.Linear(self.head_dim, self.num_attention_heads)
        self.gate1 = nn.Linear(self.hidden_size, self.scaled_dim)
        HH = self.num_attention_heads * self.num_attention_heads
        if config.num_experts is not None and config.num_experts > 0:
            kw = dict(bias=True, num_experts=config.num_experts, top_k=config.top_k_experts, r=config.r)
            self.hx_moe = LinearMoE(HH, self.hidden_size, **kw)
            self.cx_moe = LinearMoE(self.hidden_size, self.hidden_size, **kw)
            self.x_moe = LinearMoE(HH, self.hidden_size, **kw)
        else:
            self.hx_moe = nn.Linear(HH, self.hidden_size, bias=True)
            self.cx_moe = nn.Linear(self.hidden_size, self.hidden_size, bias=True)
            self.x_moe = nn.Linear(HH, self.hidden_size, bias=True)
        self.mlp = OneMLP(config)
        self.norm = OneRMSNorm(self.hidden_size, bias=True, eps=1e-6)
        for module in self.modules():
            if isinstance(module, nn.Linear) and not isinstance(module, LinearMoE):
                module.weight.data.normal_(mean=0.0, std=0.01)
                if module.bias is not None:
                    module.bias.data.zero_()

    def forward(self, *args, **kwargs):
        raise RuntimeError("One layers run inside the B200 engine; call OneForCausalLM / OneModel")


class OnePreTrainedModel(PreTrainedModel):
    config_class = OneConfig
    base_model_prefix = "model"
    supports_gradient_checkpointing = False
    _no_split_modules = ["One"]

    def _init_weights(self, module):
        # from_pretrained calls this after loading the checkpoint: the transformers init helpers
        # leave parameters that the checkpoint provided (_is_hf_initialized) untouched
        if isinstance(module, nn.Linear) and not isinstance(module, LinearMoE):
            _init.normal_(module.weight, mean=0.0, std=0.01)
            if module.bias is not None:
                _init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            _init.normal_(module.weight, mean=0.0, std=0.01)
            if module.padding_idx is not None and not getattr(module.weight, "_is_hf_initialized", False):
                with torch.no_grad():
                    module.weight[module.padding_idx].zero_()


class OneEngineCache:
    """Decode state of a batch of sequences: the engine's running sums and position. Plays the
    role of the reference's DynamicCache (one/modeling_one.py:358-365) with O(1) memory."""

    def __init__(self):
        self.seen_tokens = 0

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.seen_tokens


class OneModel(OnePreTrainedModel):
    def __init__(self, config: OneConfig):
        super().__init__(config)
        self.padding_idx = config.pad_token_id
        self.vocab_size = config.vocab_size
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, padding_idx=config.pad_token_id)
        self.decoder_layers = nn.ModuleList(
            [One(config, dropout=config.lstm_dropout, layer_idx=i, with_hx=config.with_hx)
             for i in range(config.num_hidden_layers)])
        self.lhs_norm = OneRMSNorm(config.transformer_dim, bias=True, eps=config.rms_norm_eps)
        self.up_scaler = nn.Linear(config.transformer_dim, config.hidden_size, bias=True)
        self.norm = OneRMSNorm(config.hidden_size, bias=True, eps=config.rms_norm_eps)
        self.post_init()

    def get_input_embeddings(self):
        return self.embed_tokens

    def set_input_embeddings(self, value):
        self.embed_tokens = value


class OneForCausalLM(OnePreTrainedModel, GenerationMixin):
    _tied_weights_keys = {"lm_head.weight": "model.embed_tokens.weight"}

    def __init__(self, config: OneConfig):
        super().__init__(config)
        self.model = OneModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.post_init()
        self._engine = None
        self._engine_key = None

    def get_input_embeddings(self):
        return self.model.embed_tokens

    def set_input_embeddings(self, value):
        self.model.embed_tokens = value

    def get_output_embeddings(self):
        return self.lm_head

    def set_output_embeddings(self, new_embeddings):
        self.lm_head = new_embeddings

    # ------------------------------------------------------------------ engine
    def engine(self, max_batch: int = 256, max_tokens: Optional[int] = None, max_positions: int = 8192):
        """The OneEngine over this model's current parameters. Reused while its capacity
        covers the request; otherwise rebuilt (which drops any decode state)."""
        from .engine import OneEngine
        p = self.model.embed_tokens.weight
        if not p.is_cuda:
            raise RuntimeError("OneForCausalLM runs on the B200 engine: move the model to CUDA")
        max_tokens = max_tokens or max_batch
        e = self._engine
        if (e is None or e.device != p.device or e.dtype != p.dtype or e.max_batch < max_batch
                or e.max_tokens < max_tokens or e.max_positions < max_positions):
            sd = {k: v for k, v in self.state_dict().items()}
            sd.setdefault("lm_head.weight", self.lm_head.weight)
            self._engine = OneEngine(self.config, sd, p.device, p.dtype, max_batch=max_batch,
                                     max_tokens=max(max_tokens, 4096), max_positions=max_positions)
        return self._engine

    def refresh_engine(self):
        """Drop the engine so the next call repacks the (changed) parameters."""
        self._engine = None

    @torch.no_grad()
    def forward(self, input_ids: torch.LongTensor = None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, labels=None, use_cache: Optional[bool] = None,
                output_attentions=None, output_hidden_states=None, return_dict: Optional[bool] = None,
                cache_position=None, **kwargs):
        if input_ids is None:
            raise ValueError("the engine takes input_ids")
        B, S = input_ids.shape
        cache = past_key_values
        if use_cache and cache is None:
            cache = OneEngineCache()
        if cache is None or cache.seen_tokens == 0:
            eng = self.engine(max_batch=B, max_tokens=B * S)
        else:
            eng = self._engine
            if eng is None or eng.batch != B:
                raise RuntimeError("this cache's sequences are not the engine's current batch")
        if cache is None or cache.seen_tokens == 0:
            logits = eng.prefill(input_ids, logits="all")
            if cache is not None:
                cache.seen_tokens = S
        else:
            if S != 1:
                raise NotImplementedError("continuing a cached sequence takes one token per call")
            lg, _ = eng.step(input_ids[:, 0], logits=True, next_ids=False)
            logits = lg.unsqueeze(1)
            cache.seen_tokens += 1
        loss = None
        if labels is not None:
            loss = self.loss_function(logits=logits.float(), labels=labels, vocab_size=self.config.vocab_size)
        if return_dict is False:
            out = (logits, cache)
            return ((loss,) + out) if loss is not None else out
        return CausalLMOutputWithPast(loss=loss, logits=logits, past_key_values=cache)

    @torch.no_grad()
    def generate(self, input_ids: Optional[torch.LongTensor] = None, generation_config=None, max_length=None,
                 max_new_tokens=None, do_sample=None, temperature=None, top_k=None, top_p=None, eos_token_id=None,
                 pad_token_id=None, seed: Optional[int] = None, attention_mask=None, **kwargs) -> torch.LongTensor:
        """GenerationMixin.generate for greedy search and multinomial sampling, run on the engine
        (the reference's documented use, README.md:73, model.generate(input_ids, max_length=50,
        temperature=0.7), goes through transformers' generation loop, one/modeling_one.py:845).

        Arguments resolve as transformers resolves them: explicit argument, else the model's
        generation_config, else the default (do_sample False, temperature 1, no top-k, top_p 1,
        max_length 20). do_sample=False is greedy search whatever the temperature (the
        argmax fused into lm_head, steps replayed from a captured graph); do_sample=True warps
        each step's logits (temperature, top-k, top-p) and draws one token per sequence on the
        GPU (one_sample_tokens). Once a sequence emits eos_token_id its later tokens are
        pad_token_id (eos when pad is unset), and generation stops when every sequence has
        finished. `seed` fixes the draws (default: drawn from torch's global generator).
        Returns [B, S + new tokens]. Beam search, constraints and streaming are not supported."""
        unsupported = {k: v for k, v in kwargs.items()
                       if v is not None and not (k in ("num_beams", "num_return_sequences") and v == 1)
                       and k not in ("use_cache", "return_dict_in_generate", "output_scores", "output_logits")}
        if unsupported or kwargs.get("return_dict_in_generate") or kwargs.get("output_scores"):
            raise NotImplementedError(f"generate() on the B200 engine does not support {sorted(unsupported or kwargs)}")
        gc = generation_config if generation_config is not None else getattr(self, "generation_config", None)

        def pick(v, name, default):
            if v is not None:
                return v
            g = getattr(gc, name, None) if gc is not None else None
            return g if g is not None else default

        do_sample = bool(pick(do_sample, "do_sample", False))
        temperature = float(pick(temperature, "temperature", 1.0))
        top_k = int(pick(top_k, "top_k", 0) or 0)
        top_p = float(pick(top_p, "top_p", 1.0))
        eos = pick(eos_token_id, "eos_token_id", None)
        if isinstance(eos, (list, tuple)):
            if len(eos) > 1:
                raise NotImplementedError("one eos_token_id")
            eos = eos[0] if eos else None
        pad = pick(pad_token_id, "pad_token_id", None)
        if pad is None:
            pad = eos
        if input_ids is None:
            raise ValueError("generate() needs input_ids")
        B, S = input_ids.shape
        if max_new_tokens is None:
            max_new_tokens = int(pick(max_length, "max_length", 20)) - S
        if max_new_tokens <= 0:
            return input_ids
        if do_sample and not temperature > 0:
            raise ValueError("do_sample=True needs temperature > 0")
        eng = self.engine(max_batch=B, max_tokens=max(B * S, B), max_positions=S + max_new_tokens + 16)
        if not do_sample:
            if eng.hist_cap < max_new_tokens:
                raise ValueError(f"max_new_tokens > engine history capacity ({eng.hist_cap})")
            eng.prefill(input_ids)
            for _ in range(max_new_tokens):
                eng.step(None, next_ids=False)
            new = eng.history(max_new_tokens, B).t().to(torch.long)
        else:
            from .engine import sample_tokens
            if seed is None:
                seed = int(torch.randint(0, 2 ** 62, (1,)).item())
            lg = eng.prefill(input_ids, logits="last")
            buf = torch.empty(B, self.config.vocab_size, dtype=lg.dtype, device=lg.device)
            toks = torch.empty(max_new_tokens, B, dtype=torch.int32, device=lg.device)
            for i in range(max_new_tokens):
                sample_tokens(lg, temperature, top_k, top_p, seed, i, out=toks[i])
                if i + 1 < max_new_tokens:
                    lg, _ = eng.step(toks[i], logits=True, next_ids=False, out=buf)
            new = toks.t().to(torch.long)
        if eos is not None:
            # tokens after a sequence's first eos become pad; stop once all have finished
            hit = new == int(eos)
            after = (hit.cumsum(1) - hit.long()) > 0
            new = torch.where(after, torch.full_like(new, int(pad)), new)
            done = hit.cumsum(1) > 0
            all_done = done.all(0)
            if bool(all_done.any()):
                new = new[:, : int(all_done.nonzero()[0]) + 1]
        return torch.cat([input_ids.to(new.device), new], dim=1)

    @torch.no_grad()
    def generate_greedy(self, input_ids: torch.LongTensor, max_new_tokens: int) -> torch.LongTensor:
        """Greedy decode on the engine: prompt ingestion, then max_new_tokens single-token steps
        with the argmax fed back on the device. Returns [B, S + max_new_tokens]."""
        B, S = input_ids.shape
        eng = self.engine(max_batch=B, max_tokens=max(B * S, B), max_positions=S + max_new_tokens + 16)
        if eng.hist_cap < max_new_tokens:
            raise ValueError(f"max_new_tokens > engine history capacity ({eng.hist_cap})")
        eng.prefill(input_ids)
        for _ in range(max_new_tokens):
            eng.step(None, next_ids=False)
        # history[i] holds the token fed at step i: the argmax of the previous logits
        new = eng.history(max_new_tokens, B).t().to(torch.long)
        return torch.cat([input_ids.to(new.device), new], dim=1)
