"""CPU oracle: a restatement of the MedIT One reference path in plain PyTorch (CPU).

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA engine: the
GPU parity tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` call it. The product package never imports it.

Every function restates the reference algorithm with the same torch operations
in the same order, so that its rounding points (bf16 after every op, fp32
softmax / RMSNorm statistics) are the reference's. Citations are
``path:line`` into the MedIT One reference repository.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself (imported
from its source tree with three transformers-5 compatibility patches) on seeded
inputs and commits the outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against them.

Two restatements here are the specification the CUDA kernels follow:
  * ``topk_unsorted`` — the CPU ``torch.topk(..., sorted=False)`` selection
    (libstdc++ ``std::nth_element`` / ``std::partial_sort`` with a value-only
    comparator), which decides the reference's router ties
    (one/linear_moe.py:84);
  * the O(1) running-sum decode (``RunningDecoder``), equal to the reference's
    O(P) cache-concatenate-and-cumsum (one/modeling_one.py:358-387).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor


# --------------------------------------------------------------------------- config
@dataclass
class OracleConfig:
    """The OneConfig fields the decode path reads (one/configuration_one.py:24-56)."""

    vocab_size: int = 32000
    hidden_size: int = 768
    transformer_dim: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    head_dim: int = 64
    intermediate_size: int = 3072
    num_experts: Optional[int] = 8
    top_k_experts: int = 2
    r: int = 64
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    hidden_act: str = "gelu"
    mlp_bias: bool = False
    # use_flash_attention with the reference's turbo semantics (see flash_path_attention)
    use_flash_attention: bool = False

    @property
    def use_moe(self) -> bool:
        return self.num_experts is not None and self.num_experts > 0


# --------------------------------------------------------------------------- top-k
def _gt(a, b) -> bool:
    # comparator of torch's CPU top-k for largest=True: NaN first, then '>'
    an, bn = math.isnan(a[0]), math.isnan(b[0])
    return (an and not bn) or (a[0] > b[0])


def _insertion_sort(q, lo, hi):
    for i in range(lo + 1, hi):
        if _gt(q[i], q[lo]):
            v = q[i]
            q[lo + 1:i + 1] = q[lo:i]
            q[lo] = v
        else:
            v = q[i]
            j = i
            nx = j - 1
            while _gt(v, q[nx]):
                q[j] = q[nx]
                j = nx
                nx -= 1
            q[j] = v


def _move_median_to_first(q, r, a, b, c):
    if _gt(q[a], q[b]):
        if _gt(q[b], q[c]):
            q[r], q[b] = q[b], q[r]
        elif _gt(q[a], q[c]):
            q[r], q[c] = q[c], q[r]
        else:
            q[r], q[a] = q[a], q[r]
    elif _gt(q[a], q[c]):
        q[r], q[a] = q[a], q[r]
    elif _gt(q[b], q[c]):
        q[r], q[c] = q[c], q[r]
    else:
        q[r], q[b] = q[b], q[r]


def _unguarded_partition(q, first, last, pivot):
    while True:
        while _gt(q[first], q[pivot]):
            first += 1
        last -= 1
        while _gt(q[pivot], q[last]):
            last -= 1
        if not (first < last):
            return first
        q[first], q[last] = q[last], q[first]
        first += 1


def _adjust_heap(q, first, hole, length, val):
    top = hole
    second = hole
    while second < (length - 1) // 2:
        second = 2 * (second + 1)
        if _gt(q[first + second], q[first + second - 1]):
            second -= 1
        q[first + hole] = q[first + second]
        hole = second
    if (length & 1) == 0 and second == (length - 2) // 2:
        second = 2 * (second + 1)
        q[first + hole] = q[first + second - 1]
        hole = second - 1
    parent = (hole - 1) // 2
    while hole > top and _gt(q[first + parent], val):
        q[first + hole] = q[first + parent]
        hole = parent
        parent = (hole - 1) // 2
    q[first + hole] = val


def _make_heap(q, first, middle):
    length = middle - first
    if length < 2:
        return
    parent = (length - 2) // 2
    while True:
        _adjust_heap(q, first, parent, length, q[first + parent])
        if parent == 0:
            return
        parent -= 1


def _heap_select(q, first, middle, last):
    _make_heap(q, first, middle)
    for i in range(middle, last):
        if _gt(q[i], q[first]):
            v = q[i]
            q[i] = q[first]
            _adjust_heap(q, first, 0, middle - first, v)


def _sort_heap(q, first, last):
    while last - first > 1:
        last -= 1
        v = q[last]
        q[last] = q[first]
        _adjust_heap(q, first, 0, last - first, v)


def _nth_element(q, nth):
    first, last = 0, len(q)
    if first == last or nth == last:
        return
    depth = 2 * int(math.floor(math.log2(last - first)))
    while last - first > 3:
        if depth == 0:
            _heap_select(q, first, nth + 1, last)
            q[first], q[nth] = q[nth], q[first]
            return
        depth -= 1
        mid = first + (last - first) // 2
        _move_median_to_first(q, first, first + 1, mid, last - 1)
        cut = _unguarded_partition(q, first + 1, last, first)
        if cut <= nth:
            first = cut
        else:
            last = cut
    _insertion_sort(q, first, last)


def topk_unsorted(values: List[float], k: int) -> List[int]:
    """Indices chosen by CPU ``torch.topk(v, k, largest=True, sorted=False)``, in its order.

    torch's CPU top-k fills a queue of (value, index) pairs and runs
    ``std::partial_sort`` when ``k * 64 <= n`` and ``std::nth_element``
    otherwise, with a comparator that looks at values only; libstdc++'s
    introselect then decides which of several equal scores are kept. This is
    a step-for-step restatement of that selection, the rule the reference's
    router ties follow (one/linear_moe.py:83-84).
    """
    q = [(float(v), i) for i, v in enumerate(values)]
    n = len(q)
    if k == 0:
        return []
    if k * 64 <= n:
        _heap_select(q, 0, k, n)
        _sort_heap(q, 0, k)
    else:
        _nth_element(q, k - 1)
    return [i for _, i in q[:k]]


# --------------------------------------------------------------------------- primitives
def rmsnorm(x: Tensor, weight: Tensor, bias: Optional[Tensor], eps: float) -> Tensor:
    """OneRMSNorm.forward (one/modeling_one.py:62-67): fp32 statistics, cast, then affine."""
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    out = weight * h.to(dt)
    if bias is not None:
        out = out + bias
    return out


def rope_inv_freq(head_dim: int, theta: float) -> Tensor:
    """Default RoPE init (transformers ``_compute_default_rope_parameters``), used at
    one/modeling_one.py:117-121: ``1 / theta ** (arange(0, d, 2) / d)`` in fp32."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float) / head_dim))


def rope_cos_sin(inv_freq: Tensor, position_ids: Tensor, dtype: torch.dtype) -> Tuple[Tensor, Tensor]:
    """OneRotaryEmbedding.forward (one/modeling_one.py:159-182); position_ids [bs, S]."""
    inv_freq_expanded = inv_freq[None, :, None].float().expand(position_ids.shape[0], -1, 1)
    position_ids_expanded = position_ids[:, None, :].float()
    freqs = (inv_freq_expanded.float() @ position_ids_expanded.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: Tensor) -> Tensor:
    """one/flash_attention.py:20-23."""
    x1, x2 = torch.chunk(x, 2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor, unsqueeze_dim: int = 1):
    """apply_rotary_pos_emb_flash (one/flash_attention.py:26-33)."""
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


def gelu(x: Tensor) -> Tensor:
    """ACT2FN["gelu"] (transformers GELUActivation): exact erf GELU."""
    return F.gelu(x)


def linear_moe(x: Tensor, p: Dict[str, Tensor], top_k: int) -> Tuple[Tensor, Tensor]:
    """LinearMoE.forward (one/linear_moe.py:46-99). Returns (output, top-k indices [N, k]).

    ``p`` holds ``weight [out,in]``, ``bias [out]``, ``gate [r,in]``,
    ``experts [E]`` and ``bias2 [E,in]``.
    """
    orig_shape = x.shape
    if x.dim() > 2:
        x = x.reshape(-1, x.size(-1))
    x = x.clamp(-1e4, 1e4)                                             # :53
    gate = F.softmax(F.linear(x, p["gate"]), dim=-1)                   # :56
    E = p["experts"].numel()
    experts = p["experts"].clamp(-10.0, 10.0).view(1, 1, E)            # :59
    experts_weight = gate.unsqueeze(-1) * experts                      # :61
    expert_scores = experts_weight.mean(dim=1).clamp(-10, 10)          # :64-66
    contribution = (1.0 + F.silu(expert_scores)).unsqueeze(-1)         # :68
    x_biased = x.unsqueeze(1).expand(-1, E, -1) * contribution + p["bias2"].unsqueeze(0)  # :71-77
    scores = x_biased.sum(dim=-1)                                      # :80
    k = min(top_k, E, scores.size(-1))
    _, indices = torch.topk(scores, k, dim=-1, sorted=False)           # :83-84
    gathered = torch.gather(x_biased, 1, indices.unsqueeze(-1).expand(-1, -1, x.size(-1)))
    result = F.linear(gathered.mean(dim=1), p["weight"], p.get("bias"))  # :87-93
    if len(orig_shape) > 2:
        result = result.view(orig_shape[0], orig_shape[1], -1)
    return result, indices


def linear_moe_scores(x: Tensor, p: Dict[str, Tensor]) -> Tensor:
    """The routing scores ``x_biased.sum(-1)`` of one/linear_moe.py:53-80, [N, E]."""
    x = x.reshape(-1, x.size(-1)).clamp(-1e4, 1e4)
    gate = F.softmax(F.linear(x, p["gate"]), dim=-1)
    E = p["experts"].numel()
    experts = p["experts"].clamp(-10.0, 10.0).view(1, 1, E)
    contribution = (1.0 + F.silu((gate.unsqueeze(-1) * experts).mean(dim=1).clamp(-10, 10))).unsqueeze(-1)
    return (x.unsqueeze(1).expand(-1, E, -1) * contribution + p["bias2"].unsqueeze(0)).sum(dim=-1)


def feature_attention(single_x: Tensor, key: Tensor, value: Tensor, cos: Tensor, sin: Tensor,
                      lq: Tuple[Tensor, Tensor], lk: Tuple[Tensor, Tensor], lv: Tuple[Tensor, Tensor]) -> Tensor:
    """The model's per-head feature attention (one/modeling_one.py:512-547), equal to
    turbo_combined_rope_attention_cpu (one/turbo_ops.py:382-434).

    single_x/key/value: [b, H, t, Dh] (single_x already scaled); returns [b, H, t, H].
    """
    xr, kr = apply_rope(single_x, key, cos, sin)
    q = F.linear(xr, *lq)
    k = F.linear(kr, *lk)
    v = F.linear(value, *lv)
    logits = q * k
    logits = logits - torch.max(logits, dim=-1, keepdim=True)[0]
    w = torch.softmax(logits, dim=-1, dtype=torch.float32).to(dtype=q.dtype)
    if torch.isnan(w).any():
        w = w.masked_fill(torch.isnan(w), 1.0 / w.size(-1))
    return w * v


def flash_path_attention(single_x: Tensor, key: Tensor, value: Tensor, cos: Tensor, sin: Tensor,
                         lq: Tuple[Tensor, Tensor], lk: Tuple[Tensor, Tensor], lv: Tuple[Tensor, Tensor]) -> Tensor:
    """The model's use_flash_attention branch (one/modeling_one.py:408-421) under TURBO_MODE, where
    ``self.flash_attention`` is ``TurboFlashAttention(causal=True)`` (:298-300,
    one/turbo_ops.py:437-475), i.e. turbo_flash_attention's exact causal attention with the
    default scale 1/sqrt(q.size(-1)) (one/turbo_ops.py:115-143) across the call's tokens.

    single_x/key/value: [b, H, t, Dh] (single_x already scaled); returns [b, H, t, H].

    Without TURBO_MODE the reference takes ``OneFlashAttention`` instead, whose call unpacks
    ``flash_attention()``'s single tensor into two names (one/flash_attention.py:311): that
    raises for a batch other than 2 and the layer falls back to the feature attention (:422-448),
    and for a batch of 2 the unpacked 3-d result then fails in the rearrange (:550). The turbo
    semantics are the only ones the flag has for every batch, and the engine follows them.
    """
    xr, kr = apply_rope(single_x, key, cos, sin)
    q = F.linear(xr, *lq)
    k = F.linear(kr, *lk)
    v = F.linear(value, *lv)
    return exact_attention(q, k, v, True)


def exact_attention(q: Tensor, k: Tensor, v: Tensor, causal: bool, scale: Optional[float] = None) -> Tensor:
    """turbo_flash_attention's PyTorch path (one/turbo_ops.py:115-143): exact softmax
    attention in the input dtype with an fp32 softmax."""
    if scale is None:
        scale = 1.0 / (q.size(-1) ** 0.5)
    q = q * scale
    scores = torch.matmul(q, k.transpose(-1, -2))
    if causal:
        mask = torch.triu(torch.ones(scores.shape[-2], scores.shape[-1], dtype=torch.bool), diagonal=1)
        scores.masked_fill_(mask, float("-inf"))
    w = torch.softmax(scores, dim=-1, dtype=torch.float32).to(dtype=q.dtype)
    return torch.matmul(w, v)


def rope_exact_attention(q: Tensor, k: Tensor, v: Tensor, cos: Tensor, sin: Tensor, causal: bool,
                         scale: Optional[float] = None) -> Tensor:
    """The isolated RoPE + attention workload: apply_rotary_pos_emb_flash
    (one/flash_attention.py:26-33) on q and k, then turbo_flash_attention's exact PyTorch
    path (one/turbo_ops.py:115-143)."""
    qr, kr = apply_rope(q, k, cos, sin)
    return exact_attention(qr, kr, v, causal, scale)


def exact_attention_fp32(q: Tensor, k: Tensor, v: Tensor, causal: bool, scale: Optional[float] = None) -> Tensor:
    """flash_attention()'s fp32 fallback (one/flash_attention.py:242-282): the whole
    attention in fp32, cast back to the input dtype at the end."""
    qf, kf, vf = q.float(), k.float(), v.float()
    if scale is None:
        scale = 1.0 / math.sqrt(qf.size(-1))
    attn = torch.matmul(qf * scale, kf.transpose(-1, -2))
    if causal:
        n = q.size(2)
        attn = attn.masked_fill(torch.triu(torch.ones(n, n), diagonal=1).bool()[None, None], float("-inf"))
    attn = torch.exp(attn - torch.max(attn, dim=-1, keepdim=True)[0])
    attn = attn / (torch.sum(attn, dim=-1, keepdim=True) + 1e-10)
    out = torch.matmul(attn, vf).to(q.dtype)
    return torch.nan_to_num(out, nan=0.0, posinf=0.0, neginf=0.0)


def blockwise_flash_attention(q: Tensor, k: Tensor, v: Tensor, causal: bool) -> Tensor:
    """FlashAttentionFunction.forward (one/flash_attention.py:43-139): 64x64 blocks,
    per-block max without cross-block rescaling, +1e-10 per exponent."""
    B, H, N, D = q.shape
    q = q * (1.0 / math.sqrt(D))
    o = torch.zeros_like(q)
    l = torch.zeros((B, H, N, 1), dtype=q.dtype)
    for m0 in range(0, N, 64):
        m1 = min(m0 + 64, N)
        for n0 in range(0, N, 64):
            n1 = min(n0 + 64, N)
            if causal and m0 > n1:
                continue
            s = torch.matmul(q[:, :, m0:m1], k[:, :, n0:n1].transpose(-1, -2))
            if causal:
                mask = torch.arange(m0, m1)[:, None] >= torch.arange(n0, n1)[None, :]
                s = s.masked_fill(~mask.view(1, 1, m1 - m0, n1 - n0), float("-inf"))
            s = s.float()
            e = torch.exp(s - torch.max(s, dim=-1, keepdim=True)[0]) + 1e-10
            e = e.to(q.dtype)
            l[:, :, m0:m1] += torch.sum(e, dim=-1, keepdim=True)
            o[:, :, m0:m1] += torch.matmul(e, v[:, :, n0:n1])
    o = o / l.clamp(min=1e-10)
    return torch.nan_to_num(o, nan=0.0, posinf=0.0, neginf=0.0)


def cumsum_and_normalize(x: Tensor, seq_len: int) -> Tensor:
    """turbo_cumsum_and_normalize_cpu (one/turbo_ops.py:288-310): fp32 prefix mean."""
    dt = x.dtype
    xf = x.to(torch.float32) if dt != torch.float32 else x
    res = torch.cumsum(xf, dim=1) / (torch.arange(1, seq_len + 1, dtype=torch.float32).view(1, -1, 1) + 1e-8)
    return res.to(dt) if dt != torch.float32 else res


def rotary_embedding(x: Tensor, position_ids: Tensor, inv_freq: Tensor) -> Tuple[Tensor, Tensor]:
    """turbo_rotary_embedding_cpu (one/turbo_ops.py:219-250)."""
    return rope_cos_sin(inv_freq, position_ids, x.dtype)


def mean_divisors(dtype: torch.dtype, kv_seq: int, s: int) -> Tensor:
    """The running-mean divisors of one/modeling_one.py:379-387 for the last ``s``
    tokens: ``arange(1, kv_seq + 1, dtype)[-s:] + 1e-10`` (note: bf16 ``arange``
    rounds per vector lane, not per value)."""
    seq_range = torch.arange(1, kv_seq + 1, dtype=dtype).view(1, -1, 1)
    return seq_range[:, -s:, :] + 1e-10


# --------------------------------------------------------------------------- parameters
def layer_params(sd: Dict[str, Tensor], i: int, cfg: OracleConfig) -> Dict[str, object]:
    pre = f"model.decoder_layers.{i}."
    g = lambda n: sd[pre + n]
    lp = {
        "norm1": g("norm1.weight"),
        "lin1": (g("lin1.weight"), g("lin1.bias")),
        "lin2": (g("lin2.weight"), g("lin2.bias")),
        "lin3": (g("lin3.weight"), g("lin3.bias")),
        "lin_q": (g("lin_q.weight"), g("lin_q.bias")),
        "lin_k": (g("lin_k.weight"), g("lin_k.bias")),
        "lin_v": (g("lin_v.weight"), g("lin_v.bias")),
        "mlp_gate": g("mlp.gate_proj.weight"),
        "mlp_up": g("mlp.up_proj.weight"),
        "mlp_down": g("mlp.down_proj.weight"),
        "norm": (g("norm.weight"), g("norm.bias")),
    }
    for name in ("hx_moe", "cx_moe", "x_moe"):
        d = {"weight": g(f"{name}.weight"), "bias": g(f"{name}.bias")}
        if cfg.use_moe:
            d.update(gate=g(f"{name}.gate.weight"), experts=g(f"{name}.experts"), bias2=g(f"{name}.bias2"))
        lp[name] = d
    return lp


# When a list, every routed LinearMoE call appends its top-k indices [tokens, k] (per layer:
# hx_moe, x_moe, cx_moe), for tests that compare the engine's expert selections.
ROUTE_LOG: Optional[List[Tensor]] = None


def _moe(x: Tensor, p: Dict[str, Tensor], cfg: OracleConfig) -> Tensor:
    if cfg.use_moe:
        y, idx = linear_moe(x, p, cfg.top_k_experts)
        if ROUTE_LOG is not None:
            ROUTE_LOG.append(idx.reshape(-1, idx.shape[-1]))
        return y
    return F.linear(x, p["weight"], p["bias"])


# --------------------------------------------------------------------------- one layer
def one_layer(h: Tensor, hx: Tensor, cx: Tensor, lp: Dict[str, object], cos: Tensor, sin: Tensor,
              mean_fn, cfg: OracleConfig):
    """One.forward (one/modeling_one.py:325-590); the attention is the feature attention, or with
    ``cfg.use_flash_attention`` the causal attention across the call's tokens (:408-421).

    ``mean_fn(norm_x)`` returns the running mean ``hidden_state_sum`` (:358-387);
    the caller owns the history / running sum. Returns (output, hx, cx, norm_x).
    """
    b, s, _ = h.shape
    H, Dh = cfg.num_attention_heads, cfg.head_dim
    norm_x = rmsnorm(h, lp["norm1"], None, 1e-6)                                      # :340
    value = F.linear(cx, *lp["lin3"]).view(b, s, H, Dh).permute(0, 2, 1, 3)           # :343-346
    mean = mean_fn(norm_x)                                                            # :358-387
    single_x = F.linear(norm_x, *lp["lin1"]).view(b, s, H, Dh).permute(0, 2, 1, 3)    # :390,394-399
    key = F.linear(hx, *lp["lin2"]).view(b, s, H, Dh).permute(0, 2, 1, 3)             # :391,400-402
    single_x = single_x * (1.0 / math.sqrt(Dh))                                       # :405
    if cfg.use_flash_attention:
        o = flash_path_attention(single_x, key, value, cos, sin, lp["lin_q"], lp["lin_k"], lp["lin_v"])  # :408-421
    else:
        o = feature_attention(single_x, key, value, cos, sin, lp["lin_q"], lp["lin_k"], lp["lin_v"])  # :515-547
    o = o.permute(0, 2, 1, 3).reshape(b, s, H * H)                                    # :550-556
    hx_m = torch.clamp(_moe(o, lp["hx_moe"], cfg), min=-100, max=100)                 # :559
    x_m = torch.clamp(_moe(o, lp["x_moe"], cfg), min=-100, max=100)                   # :560
    hx = rmsnorm(hx + hx_m, *lp["norm"], 1e-6)                                        # :563-564
    cx = _moe(cx, lp["cx_moe"], cfg)                                                  # :565
    out = mean * x_m                                                                  # :568
    mlp = F.linear(gelu(F.linear(out, lp["mlp_gate"])) * F.linear(out, lp["mlp_up"]), lp["mlp_down"])  # :205-206
    out = rmsnorm(out + mlp, *lp["norm"], 1e-6)                                       # :571-573
    return out, hx, cx, norm_x


def _final(sd: Dict[str, Tensor], h: Tensor, cfg: OracleConfig) -> Tensor:
    """OneModel final norms (one/modeling_one.py:801-803) and lm_head (:902)."""
    h = rmsnorm(h, sd["model.lhs_norm.weight"], sd["model.lhs_norm.bias"], cfg.rms_norm_eps)
    h = F.linear(h, sd["model.up_scaler.weight"], sd["model.up_scaler.bias"])
    h = rmsnorm(h, sd["model.norm.weight"], sd["model.norm.bias"], cfg.rms_norm_eps)
    return F.linear(h, sd.get("lm_head.weight", sd["model.embed_tokens.weight"]))


def _embed(sd: Dict[str, Tensor], ids: Tensor, cfg: OracleConfig) -> Tensor:
    """Embedding + AdaptiveAvgPool1d (one/modeling_one.py:728, 741)."""
    e = F.embedding(ids, sd["model.embed_tokens.weight"])
    if cfg.transformer_dim != cfg.hidden_size:
        e = F.adaptive_avg_pool1d(e, cfg.transformer_dim)
    return e


# --------------------------------------------------------------------------- model drivers
@dataclass
class ForwardResult:
    logits: Tensor
    hx: Tensor
    cx: Tensor
    norm_x: List[Tensor] = field(default_factory=list)


def forward(sd: Dict[str, Tensor], ids: Tensor, cfg: OracleConfig, dtype: torch.dtype,
            history: Optional[List[Tensor]] = None, last_only: bool = False) -> ForwardResult:
    """OneForCausalLM.forward (one/modeling_one.py:671-826, 857-926) over ``ids [b, s]``.

    ``history`` is the per-layer DynamicCache content (norm_x of earlier tokens,
    [b, P, D] each) or None for a cache-free forward. It is extended in place,
    exactly as ``past_key_value.update`` does (:358-365).
    Returns the logits (of the last position only when ``last_only``; the other outputs are
    unchanged), the last layer's (hx, cx) and the per-layer norm_x.
    """
    b, s = ids.shape
    P = 0 if history is None or len(history) == 0 else history[0].shape[1]
    h = _embed(sd, ids, cfg)
    pos = torch.arange(P, P + s).unsqueeze(0)                                          # :731-738
    cos, sin = rope_cos_sin(rope_inv_freq(cfg.head_dim, cfg.rope_theta), pos, h.dtype)  # :743
    hx = torch.ones((b, s, cfg.transformer_dim), dtype=h.dtype)                        # :748-752
    cx = h.clone()                                                                     # :753
    norms = []
    for i in range(cfg.num_hidden_layers):
        lp = layer_params(sd, i, cfg)

        def mean_fn(norm_x, i=i):
            if history is not None:
                if len(history) <= i:
                    history.append(norm_x)
                else:
                    history[i] = torch.cat([history[i], norm_x], dim=1)
                full = history[i]
            else:
                full = norm_x
            kv_seq = full.shape[1]
            if s < kv_seq:                                                             # :373-374
                kv_seq -= 1
            csum = torch.cumsum(full, dim=1)[:, -s:, :]                                # :376
            return csum / mean_divisors(h.dtype, kv_seq, s)                            # :379-387

        out, hx, cx, norm_x = one_layer(h, hx, cx, lp, cos, sin, mean_fn, cfg)
        norms.append(norm_x)
        h = h + out                                                                    # :793
    return ForwardResult(_final(sd, h[:, -1:] if last_only else h, cfg), hx, cx, norms)


class RunningDecoder:
    """O(1)-state equivalent of the reference's cached decode.

    The reference appends every token's ``norm_x`` to a per-layer cache and
    re-runs ``cumsum`` over it each step (one/modeling_one.py:358-387). CPU
    ``cumsum`` accumulates sequentially in fp32 (bf16 inputs included), so a
    per-layer fp32 running sum ``S_l`` updated in token order holds exactly the
    cumsum's last element before its final cast. Each step then divides
    ``S_l.to(dtype)`` by the same ``arange``-derived divisor.
    """

    def __init__(self, sd: Dict[str, Tensor], cfg: OracleConfig, dtype: torch.dtype):
        self.sd, self.cfg, self.dtype = sd, cfg, dtype
        self.S: Optional[List[Tensor]] = None
        self.P = 0
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta)
        self.layers = [layer_params(sd, i, cfg) for i in range(cfg.num_hidden_layers)]

    def prefill(self, ids: Tensor, last_only: bool = False) -> ForwardResult:
        res = forward(self.sd, ids, self.cfg, self.dtype, history=None, last_only=last_only)
        self.S = []
        for nx in res.norm_x:
            acc = torch.zeros(nx.shape[0], nx.shape[2], dtype=torch.float32)
            for t in range(nx.shape[1]):
                acc = acc + nx[:, t].float()
            self.S.append(acc)
        self.P = ids.shape[1]
        return res

    def step(self, ids: Tensor) -> ForwardResult:
        """One single-token decode step, ids [b, 1]."""
        cfg, dt = self.cfg, self.dtype
        b = ids.shape[0]
        if self.S is None:
            self.S = [torch.zeros(b, cfg.transformer_dim) for _ in range(cfg.num_hidden_layers)]
        P = self.P
        h = _embed(self.sd, ids, cfg)
        cos, sin = rope_cos_sin(self.inv_freq, torch.tensor([[P]]), h.dtype)
        hx = torch.ones((b, 1, cfg.transformer_dim), dtype=h.dtype)
        cx = h.clone()
        div = mean_divisors(dt, P if P > 0 else 1, 1)
        norms = []
        for i, lp in enumerate(self.layers):
            def mean_fn(norm_x, i=i):
                self.S[i] = self.S[i] + norm_x[:, 0].float()
                return self.S[i].to(dt).unsqueeze(1) / div
            out, hx, cx, norm_x = one_layer(h, hx, cx, lp, cos, sin, mean_fn, cfg)
            norms.append(norm_x)
            h = h + out
        self.P += 1
        return ForwardResult(_final(self.sd, h, cfg), hx, cx, norms)


class CachedDecoder:
    """The reference's own decode: per-layer norm_x history, cumsum over it each step
    (one/modeling_one.py:358-387). O(P) per step; the CPU baseline this engine replaces."""

    def __init__(self, sd: Dict[str, Tensor], cfg: OracleConfig, dtype: torch.dtype):
        self.sd, self.cfg, self.dtype = sd, cfg, dtype
        self.history: List[Tensor] = []

    def prefill(self, ids: Tensor) -> ForwardResult:
        return forward(self.sd, ids, self.cfg, self.dtype, history=self.history)

    def step(self, ids: Tensor) -> ForwardResult:
        return forward(self.sd, ids, self.cfg, self.dtype, history=self.history)


def greedy(decoder, prompt: Tensor, steps: int, keep_logits: bool = False):
    """Prefill ``prompt`` then ``steps`` greedy single-token steps (argmax, first max)."""
    res = decoder.prefill(prompt)
    nxt = torch.argmax(res.logits[:, -1, :], dim=-1)
    out_ids, logits = [], []
    for _ in range(steps):
        out_ids.append(nxt)
        res = decoder.step(nxt.unsqueeze(1))
        if keep_logits:
            logits.append(res.logits[:, 0])
        nxt = torch.argmax(res.logits[:, -1, :], dim=-1)
    return torch.stack(out_ids, 1), logits, res
