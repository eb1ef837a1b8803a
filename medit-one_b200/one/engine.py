"""OneEngine: the B200 decode engine behind OneForCausalLM.

Owns the packed device weights, one workspace allocation, the RoPE frequency table
and the running-mean divisor table, and drives libone_b200.so through its C ABI
(include/one_b200.h). All memory is allocated here, once, through torch; the library
itself never allocates.

Decode keeps the model's only cross-token information — per layer, the running sum of
``norm1(hidden)`` (one/modeling_one.py:358-387) — as an fp32 array
``state [L, batch, D]`` resident in HBM; one step reads it, adds the new token and
writes it back.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import _capi as C
from .initialization import param_specs


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """Default RoPE frequencies (one/modeling_one.py:117-122): 1 / theta^(2i/d), fp32."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float) / head_dim))


def arange_last(n: int, dtype: torch.dtype) -> float:
    """``torch.arange(1, n + 1, dtype=dtype)[-1] + 1e-10`` evaluated in ``dtype``, as a float.

    The reference divides the running sum by this value (one/modeling_one.py:379-387).
    In bf16, CPU ``arange`` fills vector lanes as ``bf16(base) + lane``, so some values
    above 256 differ from ``bf16(n)``; calling ``arange`` itself reproduces them.
    """
    return float((torch.arange(1, n + 1, dtype=dtype)[-1:] + 1e-10).float()[0])


def decode_divisors(max_pos: int, dtype: torch.dtype) -> torch.Tensor:
    """Divisor of the decode step at each position P = tokens already seen (0 .. max_pos).

    With a cache, the reference's kv_seq is P + 1 and is reduced to P for a single new
    token (one/modeling_one.py:371-374), except for P = 0 where it stays 1.
    """
    out = torch.empty(max_pos + 1, dtype=torch.float32)
    if dtype == torch.float32:
        out[0] = 1.0
        out[1:] = torch.arange(1, max_pos + 1, dtype=torch.float32)
        return out
    # Every entry comes from arange itself: which positions differ from dtype(P) depends on
    # the host CPU's vector width and on where arange's scalar tail starts (on one AVX-512
    # host, P = 32897, 33153, ... (129 mod 256) give dtype(P) - 256), so no position is
    # inferred. ~50 us per entry.
    out[0] = arange_last(1, dtype)
    for p in range(1, max_pos + 1):
        out[p] = arange_last(p, dtype)
    return out


def prompt_divisors(seq_len: int, dtype: torch.dtype) -> torch.Tensor:
    """Divisors of a prompt of seq_len tokens read with an empty cache (:379-387)."""
    return (torch.arange(1, seq_len + 1, dtype=dtype) + 1e-10).float()


def check_supported(config, dtype=torch.bfloat16) -> None:
    """Raise NotImplementedError for OneConfig switches whose reference behaviour the engine
    does not compute, instead of silently running the default path.

    * ``use_single_token=True`` computes the attention of each sequence's last position only
      and broadcasts it over the sequence (one/modeling_one.py:338, 550-568): not built.
    * ``use_flash_attention=True`` replaces the feature-level softmax with causal attention
      across the call's tokens (one/modeling_one.py:408-421, TurboFlashAttention in
      one/turbo_ops.py:437-475): built for bf16 models (the engine refuses other shapes).
    """
    if getattr(config, "use_single_token", False):
        raise NotImplementedError("OneConfig.use_single_token=True is not supported by the B200 engine")
    if getattr(config, "use_flash_attention", False) and dtype != torch.bfloat16:
        raise NotImplementedError("OneConfig.use_flash_attention=True is built for bf16 models only")


class OneEngine:
    def __init__(self, config, state_dict: Dict[str, torch.Tensor], device="cuda", dtype=torch.bfloat16,
                 max_batch: int = 256, max_tokens: Optional[int] = None, hist_cap: int = 4096,
                 max_positions: int = 8192):
        check_supported(config, dtype)
        if not torch.cuda.is_available():
            raise C.OneError("OneEngine needs a CUDA device (B200, sm_100a)")
        self.cfg = config
        self.device = torch.device(device)
        self.dtype = dtype
        self.max_batch = int(max_batch)
        self.max_tokens = int(max_tokens or max_batch)
        self.hist_cap = int(hist_cap)
        self.max_positions = int(max_positions)
        D = config.transformer_dim
        self.D = D
        L = config.num_hidden_layers
        use_moe = config.num_experts is not None and config.num_experts > 0

        self.c = C.OneConfigC(
            vocab_size=config.vocab_size, hidden_size=config.hidden_size, transformer_dim=D,
            num_hidden_layers=L, num_attention_heads=config.num_attention_heads, head_dim=config.head_dim,
            intermediate_size=config.intermediate_size, num_experts=config.num_experts if use_moe else 0,
            top_k=min(config.top_k_experts, config.num_experts) if use_moe else 0, r=config.r if use_moe else 0,
            mlp_bias=1 if config.mlp_bias else 0, dtype=C.dtype_code(dtype),
            rms_norm_eps=config.rms_norm_eps, rope_theta=config.rope_theta,
            use_flash_attention=1 if getattr(config, "use_flash_attention", False) else 0)

        # ---- weights, packed to the engine's layout (device tensors owned here)
        self._keep = []

        def dev(t):
            t = t.detach().to(device=self.device, dtype=dtype).contiguous()
            self._keep.append(t)
            return t

        sd = state_dict
        need = {n for n, _ in param_specs(config)}
        missing = sorted(n for n in need if n not in sd and ".gate1." not in n)
        if missing:
            raise C.OneError(f"state dict lacks {missing[:5]}{'...' if len(missing) > 5 else ''}")
        g = [None] * C.ONE_G_SLOTS
        g[C.ONE_G_EMBED] = dev(sd["model.embed_tokens.weight"])
        g[C.ONE_G_LHS_W] = dev(sd["model.lhs_norm.weight"])
        g[C.ONE_G_LHS_B] = dev(sd["model.lhs_norm.bias"])
        g[C.ONE_G_UP_W] = dev(sd["model.up_scaler.weight"])
        g[C.ONE_G_UP_B] = dev(sd["model.up_scaler.bias"])
        g[C.ONE_G_NORM_W] = dev(sd["model.norm.weight"])
        g[C.ONE_G_NORM_B] = dev(sd["model.norm.bias"])
        lm = sd.get("lm_head.weight")
        g[C.ONE_G_LM_HEAD] = g[C.ONE_G_EMBED] if lm is None or lm.data_ptr() == sd["model.embed_tokens.weight"].data_ptr() \
            else dev(lm)
        self.global_ptrs = (ctypes.c_void_p * C.ONE_G_SLOTS)(*[t.data_ptr() for t in g])

        lw = [0] * (L * C.ONE_W_LAYER_SLOTS)
        for l in range(L):
            p = f"model.decoder_layers.{l}."
            base = l * C.ONE_W_LAYER_SLOTS

            def put(slot, name):
                lw[base + slot] = dev(sd[p + name]).data_ptr()

            put(C.ONE_W_NORM1, "norm1.weight")
            for slot_w, slot_b, nm in ((C.ONE_W_LIN1_W, C.ONE_W_LIN1_B, "lin1"), (C.ONE_W_LIN2_W, C.ONE_W_LIN2_B, "lin2"),
                                       (C.ONE_W_LIN3_W, C.ONE_W_LIN3_B, "lin3"), (C.ONE_W_LINQ_W, C.ONE_W_LINQ_B, "lin_q"),
                                       (C.ONE_W_LINK_W, C.ONE_W_LINK_B, "lin_k"), (C.ONE_W_LINV_W, C.ONE_W_LINV_B, "lin_v")):
                put(slot_w, nm + ".weight")
                put(slot_b, nm + ".bias")
            for nm, sw, sb, sg, se, s2 in (
                    ("hx_moe", C.ONE_W_HX_W, C.ONE_W_HX_B, C.ONE_W_HX_GATE, C.ONE_W_HX_EXPERTS, C.ONE_W_HX_BIAS2),
                    ("cx_moe", C.ONE_W_CX_W, C.ONE_W_CX_B, C.ONE_W_CX_GATE, C.ONE_W_CX_EXPERTS, C.ONE_W_CX_BIAS2),
                    ("x_moe", C.ONE_W_X_W, C.ONE_W_X_B, C.ONE_W_X_GATE, C.ONE_W_X_EXPERTS, C.ONE_W_X_BIAS2)):
                put(sw, nm + ".weight")
                put(sb, nm + ".bias")
                if use_moe:
                    put(sg, nm + ".gate.weight")
                    put(se, nm + ".experts")
                    put(s2, nm + ".bias2")
            gate = sd[p + "mlp.gate_proj.weight"]
            up = sd[p + "mlp.up_proj.weight"]
            lw[base + C.ONE_W_GATE_UP] = dev(torch.stack([gate, up], 1).reshape(-1, gate.shape[1])).data_ptr()
            if config.mlp_bias:
                lw[base + C.ONE_W_GATE_UP_B] = dev(torch.stack([sd[p + "mlp.gate_proj.bias"],
                                                               sd[p + "mlp.up_proj.bias"]], 1).reshape(-1)).data_ptr()
                put(C.ONE_W_DOWN_B, "mlp.down_proj.bias")
            put(C.ONE_W_DOWN, "mlp.down_proj.weight")
            put(C.ONE_W_NORM_W, "norm.weight")
            put(C.ONE_W_NORM_B, "norm.bias")
        self.layer_ptrs = (ctypes.c_void_p * len(lw))(*lw)

        # ---- tables
        self.inv_freq = rope_inv_freq(config.head_dim, config.rope_theta).to(self.device)
        self.div = decode_divisors(self.max_positions, dtype).to(self.device)

        # ---- workspace (1024-byte aligned)
        nbytes = C.LIB.one_engine_workspace_bytes(ctypes.byref(self.c), self.max_tokens, self.max_batch, self.hist_cap)
        self._ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device=self.device)
        base = self._ws.data_ptr()
        self._ws_ptr = (base + 1023) & ~1023
        self._ws_bytes = nbytes
        h = ctypes.c_void_p()
        C.check(C.LIB.one_engine_create(ctypes.byref(self.c), self.global_ptrs, self.layer_ptrs,
                                        ctypes.c_void_p(self._ws_ptr), nbytes, self.max_tokens, self.max_batch,
                                        self.hist_cap, C.ptr(self.inv_freq), C.ptr(self.div), self.div.numel(),
                                        ctypes.byref(h)), "one_engine_create")
        self.h = h
        self._ids_buf = torch.zeros(self.max_tokens, dtype=torch.int32, device=self.device)
        self._next_buf = torch.zeros(self.max_batch, dtype=torch.int32, device=self.device)
        self.batch = 0

    # ------------------------------------------------------------------ helpers
    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value:
            try:
                C.LIB.one_engine_destroy(h)
            except Exception:
                pass
            self.h = None

    @staticmethod
    def _stream():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _view(self, name: str, shape, dtype) -> torch.Tensor:
        addr = C.LIB.one_engine_buffer(self.h, name.encode())
        if not addr:
            raise C.OneError(f"no engine buffer {name}")
        off = addr - self._ws.data_ptr()
        n = 1
        for s in shape:
            n *= s
        es = torch.tensor([], dtype=dtype).element_size()
        return self._ws[off:off + n * es].view(dtype).view(*shape)

    def state(self) -> torch.Tensor:
        """fp32 running sums [L, max_batch, D] (live view)."""
        return self._view("state", (self.cfg.num_hidden_layers, self.max_batch, self.D), torch.float32)

    def counters(self) -> Tuple[int, int]:
        c = self._view("counters", (2,), torch.int32).cpu()
        return int(c[0]), int(c[1])

    def history(self, steps: int, batch: Optional[int] = None) -> torch.Tensor:
        b = batch or self.batch
        return self._view("history", (self.hist_cap, b), torch.int32)[:steps]

    def last_hx_cx(self, T: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return (self._view("hx", (self.max_tokens if self.max_tokens > self.max_batch else self.max_batch, self.D),
                           self.dtype)[:T],
                self._view("cx", (max(self.max_tokens, self.max_batch), self.D), self.dtype)[:T])

    def router_idx(self, T: int) -> torch.Tensor:
        k = self.c.top_k
        return self._view("router_idx", (3 * T * k,), torch.int32).view(3, T, k)

    def device_error(self) -> Tuple[int, int]:
        code, where = ctypes.c_int32(), ctypes.c_int32()
        C.LIB.one_engine_error(self.h, ctypes.byref(code), ctypes.byref(where))
        return code.value, where.value

    def profile_step(self, reps: int = 20, batch: Optional[int] = None):
        """Mean microseconds of each launch of one decode step (CUDA events, warm caches)."""
        n = 256
        buf = (ctypes.c_float * n)()
        m = C.LIB.one_engine_profile_step(self.h, batch or self.batch, reps, buf, n, self._stream())
        if m < 0:
            raise C.OneError("one_engine_profile_step failed: " + C.LIB.one_last_error().decode())
        return [float(buf[i]) for i in range(m)]

    def step_launches(self, batch: Optional[int] = None) -> int:
        return int(C.LIB.one_engine_step_launches(self.h, batch or self.batch))

    def prefill_launches(self, batch: int, seq_len: int, logits: str = "none") -> int:
        """Kernels one prefill(ids [batch, seq_len], logits) launches: per layer row_pre, prefix-mean
        scan, GEMM A, attention (+ gate GEMM and three router launches on the prompt path), GEMM C,
        gate/up, down; the RoPE table; the final row_pre, up_scaler, norm, lm_head; the counter update."""
        mode = {"none": 0, "last": 1, "all": 2}[logits]
        return int(C.LIB.one_engine_prefill_launches(self.h, batch, seq_len, mode))

    # ------------------------------------------------------------------ API
    def reset(self, batch: int, pos: int = 0) -> None:
        C.check(C.LIB.one_engine_reset(self.h, batch, pos, self._stream()), "one_engine_reset")
        self.batch = batch

    def prefill(self, ids: torch.Tensor, logits: str = "none") -> Optional[torch.Tensor]:
        """Ingest prompts ids [B, S] (fresh sequences). logits: "none" | "last" | "all"."""
        B, S = ids.shape
        self.reset(B, 0)
        ids32 = ids.to(device=self.device, dtype=torch.int32).contiguous().view(-1)
        div = prompt_divisors(S, self.dtype).to(self.device)
        mode = {"none": 0, "last": 1, "all": 2}[logits]
        out = None
        if mode == 1:
            out = torch.empty(B, self.cfg.vocab_size, dtype=self.dtype, device=self.device)
        elif mode == 2:
            out = torch.empty(B * S, self.cfg.vocab_size, dtype=self.dtype, device=self.device)
        C.check(C.LIB.one_engine_prefill(self.h, C.ptr(ids32), B, S, C.ptr(div), mode, C.ptr(out), self._stream()),
                "one_engine_prefill")
        self._keep_step = (ids32, div)
        if mode == 2:
            out = out.view(B, S, -1)
        return out

    def step(self, ids: Optional[torch.Tensor] = None, logits: bool = False, next_ids: bool = True,
             out: Optional[torch.Tensor] = None):
        """One decode step for the current batch. ids [B] (None = greedy from the previous
        argmax). Returns (logits [B, V] or None, next_ids [B] int32 or None). `out`: a [B, V]
        model-dtype buffer the logits are written to (reused across steps, one captured graph)."""
        B = self.batch
        idp = None
        if ids is not None:
            self._ids_buf[:B].copy_(ids.view(-1).to(torch.int32), non_blocking=True)
            idp = self._ids_buf
        lg = None
        if logits:
            lg = out if out is not None else torch.empty(B, self.cfg.vocab_size, dtype=self.dtype, device=self.device)
        nx = self._next_buf if next_ids else None
        C.check(C.LIB.one_engine_step(self.h, B, C.ptr(idp), C.ptr(lg), C.ptr(nx), self._stream()), "one_engine_step")
        return lg, (nx[:B] if nx is not None else None)

    def capture(self, steps: int, batch: Optional[int] = None) -> None:
        C.check(C.LIB.one_engine_capture(self.h, batch or self.batch, steps, self._stream()), "one_engine_capture")

    def replay(self) -> None:
        C.check(C.LIB.one_engine_replay(self.h, self._stream()), "one_engine_replay")


def sample_tokens(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                  seed: int = 0, offset: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One token per row of logits [B, V] (CUDA, bf16 or fp32) drawn on the GPU
    (one_sample_tokens): scores / temperature, top-k, top-p, one draw from the softmax of the
    kept scores, as transformers' sampling loop warps its logits. The draw of row b depends on
    (seed, offset, b) only. Returns int32 [B] on the logits' device."""
    if logits.dim() != 2 or not logits.is_cuda:
        raise C.OneError("sample_tokens takes CUDA logits [batch, vocab]")
    B, V = logits.shape
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    C.check(C.LIB.one_sample_tokens(C.ptr(logits), B, V, logits.stride(0), C.dtype_code(logits.dtype), float(temperature),
                                    int(top_k or 0), float(1.0 if top_p is None else top_p),
                                    ctypes.c_uint64(seed & (2 ** 64 - 1)), ctypes.c_uint64(offset & (2 ** 64 - 1)),
                                    C.ptr(out), ctypes.c_void_p(torch.cuda.current_stream(logits.device).cuda_stream)),
            "one_sample_tokens")
    return out
