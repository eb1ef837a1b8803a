"""Decode throughput of the 140M-class MedIT One model in bf16 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--workload decode|attention|linear_moe|prefill]

Workload (per GPU, weak scaling): 256 sequences, prompt of 128 tokens (ids uniform in
[0, 32000), seed 4 + rank), then greedy single-token decode steps carrying the
per-layer running state in HBM. A "step" is one decode step of all 256 sequences.
Weights are random-init (N(0, 0.02), seed 4); there is no dataset.

`value` is tokens/s over all GPUs: N * 256 * K / (max over ranks of the device time of
K graph-replayed steps). `e2e` is the same metric through the public API
(OneEngine.step) with the step's input ids copied from pinned host memory and the
next ids read back to the host every step. The roofline is the whole decode step
(the path's unit of work): algorithmic HBM bytes per step / step time.

--impl reference times the reference algorithm on the host CPU (the oracle's
restatement of one/modeling_one.py's cached decode: per-layer history concatenated
and cumsum-ed every step) on the same model and a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "medit-one_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

BATCH = 256
PROMPT = 128
SEED = 4
METRIC = "decode tok/s (140M-class bf16, B=256 per GPU)"


# DRAM bytes measured by ncu (read + write) for the bench workloads' dominant kernels, per launch:
# one graph-replayed decode step of the 140M bf16 model at 256 sequences (the 76 launches summed,
# caches left warm: 304.3 MB read + 44.8 MB written) and one non-causal [8, 12, 2048, 64]
# attention launch (103.7 MB; algorithmic q, k, v, out = 100.7 MB).
STEP_DRAM_BYTES = {256: 349.05e6}
ATTN_DRAM_BYTES = 103.7e6

def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def step_bytes(cfg, batch: int) -> dict:
    """Algorithmic HBM bytes of one decode step: every weight the step reads once, the
    fp32 running state read and written once per layer, token ids and the argmax."""
    from one.initialization import param_specs
    w = 0
    for name, shape in param_specs(cfg):
        if ".gate1." in name:
            continue  # One.gate1 is never used by the forward pass
        n = 1
        for s in shape:
            n *= s
        if name == "model.embed_tokens.weight":
            emb_rows = batch * cfg.hidden_size * 2  # gathered rows
            lm = n * 2  # the tied lm_head reads the whole table
            w += emb_rows + lm
            continue
        w += n * 2
    state = 2 * cfg.num_hidden_layers * batch * cfg.transformer_dim * 4
    io = batch * (4 + 8)
    flops = 0
    for name, shape in param_specs(cfg):
        if ".gate1." in name or len(shape) != 2 or name == "model.embed_tokens.weight":
            continue
        if name.endswith(("lin_q.weight", "lin_k.weight", "lin_v.weight")):
            flops += 2 * batch * cfg.num_attention_heads * shape[0] * shape[1]
        else:
            flops += 2 * batch * shape[0] * shape[1]
    flops += 2 * batch * cfg.vocab_size * cfg.hidden_size
    return {"weights": w, "state": state, "io": io, "total": w + state + io, "flops": flops}


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, idx: int):
        self.idx = idx
        self.proc = None
        # raw samples: kept in $ONE_CLOCKS_DIR when it is set (the JSON line carries the summary)
        d = os.environ.get("ONE_CLOCKS_DIR")
        self.path = os.path.join(d, f"clocks_rank{idx}.csv") if d and os.path.isdir(d) else \
            f"/tmp/one_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        except Exception:
            rows = []
        mhz, mx, reasons = [], None, set()
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                mhz.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, v in (("hw_slowdown", r[5]), ("hw_thermal_slowdown", r[6]), ("sw_thermal_slowdown", r[7]),
                            ("sw_power_cap", r[8])):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# The stated decode workload: 2048 steps after a 128-token prompt. The reference's cached decode
# re-runs a cumsum over the whole history each step (one/modeling_one.py:358-387), so its step
# time grows with the context; its rate over the workload is sampled at the first, middle and last
# context and combined with Simpson's weights (exact for a step time linear in the context).
DECODE_STEPS = 2048
CPU_CONTEXTS = (PROMPT, PROMPT + DECODE_STEPS // 2, PROMPT + DECODE_STEPS - 1)
CPU_WEIGHTS = (1.0 / 6.0, 4.0 / 6.0, 1.0 / 6.0)


def cpu_reference(cfg, steps: int, warmup: int, batch: int, contexts=CPU_CONTEXTS) -> dict:
    """The reference's cached decode on the host CPU: per-layer norm_x history of `context`
    tokens (seeded random bf16, as left by a prompt), one new token per step, timed at each of
    `contexts`; the value is the rate over the whole 2048-step run (Simpson-weighted mean step
    time over the sampled contexts)."""
    from one.initialization import init_state_dict
    from oracle import one_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    oc = O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, transformer_dim=cfg.transformer_dim,
                        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                        head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                        top_k_experts=cfg.top_k_experts, r=cfg.r)
    per_step, total = [], 0.0
    for context in contexts:
        dec = O.CachedDecoder(sd, oc, torch.bfloat16)
        g = torch.Generator().manual_seed(SEED)
        dec.history = [torch.randn(batch, context, cfg.transformer_dim, generator=g).bfloat16()
                       for _ in range(cfg.num_hidden_layers)]
        ids = torch.randint(0, cfg.vocab_size, (batch, 1), generator=g)
        with torch.no_grad():
            for _ in range(warmup):
                ids = dec.step(ids).logits[:, -1].argmax(-1, keepdim=True)
            t0 = time.perf_counter()
            for _ in range(steps):
                ids = dec.step(ids).logits[:, -1].argmax(-1, keepdim=True)
            dt = time.perf_counter() - t0
        per_step.append(dt / steps)
        total += dt
        del dec
    w = CPU_WEIGHTS if len(contexts) == 3 else tuple(1.0 / len(contexts) for _ in contexts)
    mean_step = sum(wi * ti for wi, ti in zip(w, per_step))
    # the same ops with the O(1) running sum in place of the history cumsum (the engine's
    # algorithm on the CPU): context-independent
    run = O.RunningDecoder(sd, oc, torch.bfloat16)
    g = torch.Generator().manual_seed(SEED)
    run.S = [torch.randn(batch, cfg.transformer_dim, generator=g) for _ in range(cfg.num_hidden_layers)]
    run.P = contexts[0]
    ids = torch.randint(0, cfg.vocab_size, (batch, 1), generator=g)
    with torch.no_grad():
        ids = run.step(ids).logits[:, -1].argmax(-1, keepdim=True)
        t0 = time.perf_counter()
        for _ in range(steps):
            ids = run.step(ids).logits[:, -1].argmax(-1, keepdim=True)
        o1 = (time.perf_counter() - t0) / steps
    return {"value": batch / mean_step, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} decode steps of {batch} sequences at each context {list(contexts)} "
                      f"({warmup} untimed each; step s {[round(t, 3) for t in per_step]}), Simpson-weighted over the "
                      f"{DECODE_STEPS}-step run; oracle restatement of the reference's cached decode, bf16",
            "o1_tok_s": batch / o1,
            "seconds": total, "step_seconds": per_step, "contexts": list(contexts)}


def run_reference(args, ws, rank):
    from one.configuration_one import config_140m
    if rank != 0:
        return
    cfg = config_140m()
    # bounded sample: a CPU step of 256 sequences takes ~0.2 s at context 128 and a few seconds at
    # context 2175 on the host; three timed steps per sampled context at most
    steps = max(1, min(args.steps, 3))
    warmup = max(0, min(args.warmup, 1))
    r = cpu_reference(cfg, steps, warmup, BATCH)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 1000.0 * BATCH / r["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, uniform ids)",
            "config": {"workload": f"140M-class One, bf16, greedy decode of 256 sequences, {DECODE_STEPS} steps after a "
                                   f"{PROMPT}-token prompt (step time sampled at contexts {list(CPU_CONTEXTS)})",
                       "batch": BATCH, "prompt": PROMPT},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "o1_tok_s")},
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_native(args, ws, rank, local):
    from one import distributed as Dd
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    steps, warmup = args.steps, args.warmup
    strong = args.global_batch is not None
    if strong:
        # fixed global batch, split by sequence: rank r decodes its contiguous shard of one
        # seeded prompt set
        G = args.global_batch
        first, bl = Dd.shard(G, ws, rank)
        g = torch.Generator().manual_seed(SEED)
        prompt = torch.randint(0, cfg.vocab_size, (G, PROMPT), generator=g)[first:first + bl]
    else:
        G, bl = BATCH * ws, BATCH
        g = torch.Generator().manual_seed(SEED + rank)
        prompt = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=g)
    eng = OneEngine(cfg, sd, f"cuda:{local}", torch.bfloat16, max_batch=bl, max_tokens=bl * PROMPT,
                    hist_cap=2 * (steps + warmup) + 64, max_positions=PROMPT + 2 * (steps + warmup) + 4096)
    del sd
    eng.prefill(prompt.cuda())
    eng.capture(1)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        eng.replay()
    torch.cuda.synchronize()
    barrier(ws)
    # The timed region: the K graph-replayed steps, then the run's only collective, the NCCL
    # all-gather of every rank's generated tokens of those steps to every rank.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(steps):
            eng.replay()
        tokens = Dd.gather_tokens(eng.history(warmup + steps, bl)[warmup:].t().contiguous(), G)
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize()
    barrier(ws)
    assert tokens.shape == (G, steps)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ws, ms)
    code = eng.device_error()
    if code != (0, 0):
        raise RuntimeError(f"device error {code}")
    value = G * steps / (ms_max / 1000.0)
    # the gather alone, for the record (same collective, same sizes)
    gather_ms = None
    if ws > 1:
        torch.cuda.synchronize()
        barrier(ws)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        Dd.gather_tokens(eng.history(warmup + steps, bl)[warmup:].t().contiguous(), G)
        g1.record(stream)
        g1.synchronize()
        gather_ms = max_over_ranks(ws, g0.elapsed_time(g1))

    # e2e through the public step API: pinned host ids in, next ids out, every step; the
    # run's tokens all-gathered at the end (inside the timed region)
    ids_host = torch.randint(0, cfg.vocab_size, (bl,), dtype=torch.int32, generator=g).pin_memory()
    out_host = torch.empty(bl, dtype=torch.int32).pin_memory()
    ids_dev = torch.empty(bl, dtype=torch.int32, device=f"cuda:{local}")
    for _ in range(max(warmup, 2)):
        ids_dev.copy_(ids_host, non_blocking=True)
        _, nx = eng.step(ids_dev)
        out_host.copy_(nx, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    done = eng.counters()[1]
    barrier(ws)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e_start.record(stream)
    for _ in range(steps):
        ids_dev.copy_(ids_host, non_blocking=True)
        _, nx = eng.step(ids_dev)
        out_host.copy_(nx, non_blocking=True)
        stream.synchronize()
        ids_host.copy_(out_host)
    e_tokens = Dd.gather_tokens(eng.history(done + steps, bl)[done:].t().contiguous(), G)
    e_end.record(stream)
    e_end.synchronize()
    assert e_tokens.shape == (G, steps)
    e_ms = max_over_ranks(ws, e_start.elapsed_time(e_end))
    e2e = G * steps / (e_ms / 1000.0)

    hbm, tf, tf_sus, src = peaks()
    sb = step_bytes(cfg, bl)
    t_step = ms_max / 1000.0 / steps
    achieved = sb["total"] / t_step / 1e9
    launches = eng.step_launches(bl)
    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC if not strong else f"decode tok/s (140M-class bf16, global batch {G})",
            "value": value, "unit": "tok/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
            "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights N(0,0.02) seed 4, uniform prompt ids)",
            "config": {"workload": "140M-class One (vocab 32000, hidden 768, 12 layers, 12 heads, 8 experts top-2, "
                                   "FFN 3072), bf16 greedy decode after a 128-token prompt",
                       "batch_per_gpu": bl, "global_batch": G, "prompt": PROMPT,
                       "parallelism": f"sequence-sharded dp{ws}, no collective on the step path; one NCCL "
                                      f"all-gather of the generated tokens per timed run, inside the timed region",
                       "gather_ms": gather_ms,
                       "l2": "inputs larger than L2 (285 MB of weights streamed per step)"},
            "roofline": {"bound": "hbm", "kernel": f"decode step ({launches} launches, CUDA graph)",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": src, "traffic": STEP_DRAM_BYTES.get(bl),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum summed over the "
                                           "76 launches of one decode step (--cache-control none, serialized)",
                         "algorithmic_bytes_per_step": sb["total"],
                         "tflops_achieved": sb["flops"] / t_step / 1e12,
                         "tensor_frac_sustained": sb["flops"] / t_step / 1e12 / tf_sus},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": bl * 4, "d2h_bytes_per_step": bl * 4},
            "gpu_launches": launches * steps + (1 if ws > 1 else 0),
            "clocks": clocks,
        }
        if ws == 1 and not args.no_cpu_baseline:
            r = cpu_reference(cfg, 2, 1, BATCH)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "o1_tok_s")}
        print(json.dumps(line), flush=True)


ATT_SHAPE = (8, 12, 2048, 64)
ATT_METRIC = "fused RoPE + attention TFLOP/s (Q/K/V [8,12,2048,64] bf16, causal + non-causal)"


def attention_flops(b, h, n, d, causal):
    """Algorithmic FLOPs of softmax(q k^T) v: 2 matmuls of 2*n*n_keys*d per head; under the
    causal mask each query row sees row+1 keys."""
    keys = n * (n + 1) / 2 if causal else n * n
    return 4.0 * b * h * d * keys


def attention_inputs(device):
    from one import turbo_ops
    from one.engine import rope_inv_freq
    B, H, N, D = ATT_SHAPE
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(B, H, N, D, generator=g).bfloat16() for _ in range(3))
    pos = torch.arange(0, N).unsqueeze(0)
    if device == "cpu":
        return q, k, v, pos
    q, k, v = q.to(device), k.to(device), v.to(device)
    cos, sin = turbo_ops.turbo_rotary_embedding(q, pos.to(device), rope_inv_freq(D, 10000.0).to(device))
    return q, k, v, cos, sin


def attention_cpu(heads: int) -> dict:
    """The reference's RoPE + exact attention (oracle restatement) on the host CPU for a
    bounded sample of `heads` (batch, head) pairs of the workload, causal and non-causal."""
    from oracle import one_oracle as O
    B, H, N, D = ATT_SHAPE
    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v, pos = attention_inputs("cpu")
    cos, sin = O.rope_cos_sin(O.rope_inv_freq(D, 10000.0), pos, torch.bfloat16)
    qs, ks, vs = (x.reshape(B * H, N, D)[:heads].unsqueeze(0) for x in (q, k, v))
    O.rope_exact_attention(qs[:, :1], ks[:, :1], vs[:, :1], cos, sin, False)  # warm-up
    t0 = time.perf_counter()
    for causal in (False, True):
        for h0 in range(0, heads, 8):  # 8 heads at a time bounds the score matrices' memory
            O.rope_exact_attention(qs[:, h0:h0 + 8], ks[:, h0:h0 + 8], vs[:, h0:h0 + 8], cos, sin, causal)
    dt = time.perf_counter() - t0
    fl = sum(attention_flops(1, heads, N, D, c) for c in (False, True))
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{heads} of {B * H} (batch, head) pairs, causal and non-causal, oracle restatement of "
                      f"apply_rotary_pos_emb_flash + turbo_flash_attention's exact path in bf16", "seconds": dt}


def run_attention(args, ws, rank, local):
    """One step = the fused RoPE + attention op on the whole workload, non-causal then causal."""
    import ctypes
    from one import _capi as C, turbo_ops
    B, H, N, D = ATT_SHAPE
    dev = f"cuda:{local}"
    q, k, v, cos, sin = attention_inputs(dev)
    out = torch.empty_like(q)
    ws_buf = torch.empty(C.LIB.one_rope_flash_attention_workspace_bytes(B, H, N, D, 0), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    st = ctypes.c_void_p(stream.cuda_stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > L2: inputs are 75 MB

    def op(causal):
        C.check(C.LIB.one_rope_flash_attention(C.ptr(q), C.ptr(k), C.ptr(v), C.ptr(cos), C.ptr(sin), 1, B, H, N, D,
                                               1 if causal else 0, 0.125, 0, C.ptr(out), C.ptr(ws_buf),
                                               ws_buf.numel(), st), "one_rope_flash_attention")

    for _ in range(args.warmup):
        op(False)
        op(True)
    torch.cuda.synchronize()
    barrier(ws)
    per = {False: 0.0, True: 0.0}
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(2 * args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            for c, causal in enumerate((False, True)):
                flush.zero_()
                e0, e1 = ev[2 * i + c]
                e0.record(stream)
                op(causal)
                e1.record(stream)
        torch.cuda.synchronize()
    for i in range(args.steps):
        for c, causal in enumerate((False, True)):
            per[causal] += ev[2 * i + c][0].elapsed_time(ev[2 * i + c][1])
    barrier(ws)
    ms = max_over_ranks(ws, per[False] + per[True])
    fl_step = attention_flops(B, H, N, D, False) + attention_flops(B, H, N, D, True)
    value = ws * fl_step * args.steps / (ms / 1000.0) / 1e12
    if turbo_ops.ops_error() != (0, 0):
        raise RuntimeError("device error in the attention kernels")

    # e2e through the public API: host q/k/v/cos/sin in, host output back, every step
    hq, hk, hv, hc, hs = (x.cpu().pin_memory() for x in (q, k, v, cos, sin))
    for _ in range(2):
        turbo_ops.turbo_rope_flash_attention(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True),
                                             hv.to(dev, non_blocking=True), hc.to(dev, non_blocking=True),
                                             hs.to(dev, non_blocking=True), causal=False).cpu()
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for causal in (False, True):
            o = turbo_ops.turbo_rope_flash_attention(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True),
                                                     hv.to(dev, non_blocking=True), hc.to(dev, non_blocking=True),
                                                     hs.to(dev, non_blocking=True), causal=causal)
            o.cpu()
    e1.record(stream)
    e1.synchronize()
    e_ms = max_over_ranks(ws, e0.elapsed_time(e1))
    e2e = ws * fl_step * args.steps / (e_ms / 1000.0) / 1e12
    h2d = 2 * sum(x.numel() * x.element_size() for x in (hq, hk, hv, hc, hs))
    d2h = 2 * out.numel() * out.element_size()

    _, tf, _, src = peaks()
    clocks = clk.summary()
    if rank == 0:
        line = {"metric": ATT_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (Q/K/V ~ N(0,1) seed 2, RoPE base 1e4)",
                "config": {"workload": "isolated fused RoPE + flash attention, Q/K/V [8, 12, 2048, 64] bf16, "
                                       "scale 1/8, one non-causal and one causal call per step",
                           "us_noncausal": 1000 * per[False] / args.steps, "us_causal": 1000 * per[True] / args.steps,
                           "l2": "256 MB buffer written between timed calls (inputs 75 MB < L2)"},
                "roofline": {"bound": "tensor", "kernel": "flash_attn_tc_kernel + rope_qk_kernel",
                             "achieved": value / ws, "peak": tf, "unit": "TFLOP/s", "frac": value / ws / tf,
                             "peak_source": src, "traffic": ATTN_DRAM_BYTES,
                             "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one non-causal "
                                               "flash_attn_tc_kernel launch (L2 flushed first)"},
                "e2e": {"value": e2e, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "gpu_launches": 4 * args.steps, "clocks": clocks}
        if ws == 1 and not args.no_cpu_baseline:
            r = attention_cpu(96)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)


def run_attention_reference(args):
    r = attention_cpu(96)
    line = {"impl": "reference", "metric": ATT_METRIC, "value": r["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 1, "ms_per_step": 1000 * r["seconds"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (Q/K/V ~ N(0,1) seed 2, RoPE base 1e4)",
            "config": {"workload": "isolated fused RoPE + flash attention, Q/K/V [8, 12, 2048, 64] bf16"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PF_B, PF_S, PF_SEED = 64, 4096, 5
PF_METRIC = "prefill tok/s (140M-class bf16, 4096-token prompts, 64 sequences per call)"


def gemm_flops_per_token(cfg) -> float:
    """2 x the weights a token's forward multiplies (lm_head excluded: prefill returns no logits)."""
    return step_bytes(cfg, 1)["flops"] - 2.0 * cfg.vocab_size * cfg.hidden_size


def prefill_cpu(cfg, seqs: int, length: int) -> dict:
    """The reference forward (oracle restatement of one/modeling_one.py:671-826) on the host
    CPU for a bounded sample of the prompts."""
    from one.initialization import init_state_dict
    from oracle import one_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    oc = O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, transformer_dim=cfg.transformer_dim,
                        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                        head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                        top_k_experts=cfg.top_k_experts, r=cfg.r)
    g = torch.Generator().manual_seed(PF_SEED)
    ids = torch.randint(0, cfg.vocab_size, (seqs, length), generator=g)
    with torch.no_grad():
        O.forward(sd, ids[:, :16], oc, torch.bfloat16)  # warm-up
        t0 = time.perf_counter()
        O.forward(sd, ids, oc, torch.bfloat16)
        dt = time.perf_counter() - t0
    return {"value": seqs * length / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "seconds": dt, "sample": f"{seqs} prompts x {length} tokens (oracle restatement of the reference's "
                                     f"forward, bf16)"}


def run_prefill(args, ws, rank, local):
    """One step = prefill of 64 prompts of 4096 tokens (the per-GPU share of the 4096 x 4096 prompt
    set is 512 prompts: 8 steps); then the decode rate at batch 64 from that state."""
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    dev = f"cuda:{local}"
    dsteps = 200
    eng = OneEngine(cfg, init_state_dict(cfg, SEED, torch.bfloat16), dev, torch.bfloat16, max_batch=PF_B,
                    max_tokens=PF_B * PF_S, hist_cap=dsteps + 64, max_positions=PF_S + dsteps + 64)
    g = torch.Generator().manual_seed(PF_SEED + rank)
    ids = torch.randint(0, cfg.vocab_size, (PF_B, PF_S), generator=g)
    ids_dev = ids.to(dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        eng.prefill(ids_dev)
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            eng.prefill(ids_dev)
        e1.record(stream)
        e1.synchronize()
    ms = max_over_ranks(ws, e0.elapsed_time(e1))
    if eng.device_error() != (0, 0):
        raise RuntimeError(f"device error {eng.device_error()}")
    tokens = PF_B * PF_S
    value = ws * tokens * args.steps / (ms / 1000.0)
    fl = gemm_flops_per_token(cfg) * tokens
    # decode at batch 64 from the prefilled state (positions 4096 ..)
    eng.capture(1)
    for _ in range(5):
        eng.replay()
    torch.cuda.synchronize()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(dsteps):
        eng.replay()
    d1.record(stream)
    d1.synchronize()
    dec_ms = d0.elapsed_time(d1) / dsteps
    # e2e through the public API: prompt ids from pinned host memory in, each prompt's next token out
    hids = ids.pin_memory()
    barrier(ws)
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for _ in range(args.steps):
        lg = eng.prefill(hids.to(dev, non_blocking=True), logits="last")
        nxt = lg.argmax(-1).to(torch.int32).cpu()
    x1.record(stream)
    x1.synchronize()
    e_ms = max_over_ranks(ws, x0.elapsed_time(x1))
    e2e = ws * tokens * args.steps / (e_ms / 1000.0)
    assert nxt.shape[0] == PF_B
    _, _, tf_sus, src = peaks()
    t_step = ms / 1000.0 / args.steps
    clocks = clk.summary()
    if rank == 0:
        line = {"metric": PF_METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights N(0,0.02) seed 4, prompt ids uniform, seed 5 + rank)",
                "config": {"workload": "140M-class One bf16 prompt ingestion, 64 prompts x 4096 tokens per call "
                                       "(the per-GPU 512-prompt share of 4096 x 4096 is 8 calls), then greedy "
                                       "decode at batch 64",
                           "decode_b64_ms_per_step": dec_ms, "decode_b64_tok_s": ws * PF_B / (dec_ms / 1000.0),
                           "l2": "inputs larger than L2 (weights 285 MB, activations GBs)"},
                "roofline": {"bound": "tensor", "kernel": "prefill (tcgen05 GEMMs + row kernels)",
                             "achieved": fl / t_step / 1e12, "peak": tf_sus, "unit": "TFLOP/s",
                             "frac": fl / t_step / 1e12 / tf_sus, "peak_source": src + " (sustained)",
                             "traffic": None, "flops_per_token": gemm_flops_per_token(cfg)},
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": tokens * 8, "d2h_bytes_per_step": PF_B * 4},
                "gpu_launches": args.steps * eng.prefill_launches(PF_B, PF_S), "clocks": clocks}
        if ws == 1 and not args.no_cpu_baseline:
            r = prefill_cpu(cfg, 8, 1024)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)


def run_prefill_reference(args):
    from one.configuration_one import config_140m
    r = prefill_cpu(config_140m(), 8, 1024)
    line = {"impl": "reference", "metric": PF_METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 1, "ms_per_step": 1000 * r["seconds"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, uniform prompt ids)",
            "config": {"workload": "140M-class One bf16 prompt ingestion"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


C5_PROMPTS, C5_LEN, C5_CALL, C5_DECODE, C5_DEC_B = 4096, 4096, 64, 32768, 64
C5_METRIC = "config 5: prompt ingestion tok/s (4096 prompts x 4096 tokens over the GPUs) and decode tok/s (batch 64)"


def run_config5(args, ws, rank, local):
    """The stated prompt-ingestion + long-decode workload at its full size: 4096 prompts of 4096
    tokens (ids uniform, seed 5) split evenly over the GPUs and ingested 64 prompts per call,
    then 32768 greedy decode steps of the last call's 64 sequences on every GPU (positions
    4096 .. 36863), each step a CUDA-graph replay. Checks: the device error record stays clear,
    and the last-position logits of two of the prompts match the oracle's forward over the
    whole 4096-token prompt (bf16 tolerance 2e-2). The ingestion and the decode are each timed
    with CUDA events, max over ranks."""
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    dev = f"cuda:{local}"
    prompts = args.c5_prompts // ws
    calls = max(1, prompts // C5_CALL)
    dsteps = args.c5_steps
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    eng = OneEngine(cfg, sd, dev, torch.bfloat16, max_batch=C5_CALL, max_tokens=C5_CALL * C5_LEN,
                    hist_cap=dsteps + 16, max_positions=C5_LEN + dsteps + 16)
    g = torch.Generator().manual_seed(PF_SEED)
    all_ids = torch.randint(0, cfg.vocab_size, (args.c5_prompts, C5_LEN), generator=g)
    mine = all_ids[rank * prompts:(rank + 1) * prompts]
    stream = torch.cuda.current_stream()
    eng.prefill(mine[:C5_CALL, :64].to(dev))  # warm-up (kernel attributes, tables)
    torch.cuda.synchronize()
    barrier(ws)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        p0.record(stream)
        for c in range(calls):
            lg = eng.prefill(mine[c * C5_CALL:(c + 1) * C5_CALL].to(dev, non_blocking=True), logits="last")
        p1.record(stream)
        p1.synchronize()
        pf_ms = max_over_ranks(ws, p0.elapsed_time(p1))
        if eng.device_error() != (0, 0):
            raise RuntimeError(f"device error after prompt ingestion {eng.device_error()}")
        # the last call's prompts 0 and 63 against the oracle over the whole prompt
        checked = 0
        if rank == 0:
            from oracle import one_oracle as O
            oc = O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                                transformer_dim=cfg.transformer_dim, num_hidden_layers=cfg.num_hidden_layers,
                                num_attention_heads=cfg.num_attention_heads, head_dim=cfg.head_dim,
                                intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                                top_k_experts=cfg.top_k_experts, r=cfg.r)
            last = mine[(calls - 1) * C5_CALL:calls * C5_CALL]
            rows = [0, C5_CALL - 1]
            torch.set_num_threads(os.cpu_count() or 1)
            with torch.no_grad():
                ref = O.forward(sd, last[rows], oc, torch.bfloat16, last_only=True).logits[:, -1].float()
            got = lg.view(C5_CALL, -1)[rows].float().cpu()
            bad = (got - ref).abs() > 2e-2 + 2e-2 * ref.abs()
            if bool(bad.any()):
                raise RuntimeError(f"last-position logits differ from the oracle at {int(bad.sum())} entries")
            checked = len(rows)
        # decode: 32768 steps of the last call's sequences
        eng.capture(1)
        eng.replay()
        torch.cuda.synchronize()
        barrier(ws)
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(dsteps - 1):
            eng.replay()
        d1.record(stream)
        d1.synchronize()
        dec_ms = max_over_ranks(ws, d0.elapsed_time(d1))
    if eng.device_error() != (0, 0):
        raise RuntimeError(f"device error after decode {eng.device_error()}")
    hist = eng.history(dsteps, C5_CALL)
    assert int(hist.min()) >= 0 and int(hist.max()) < cfg.vocab_size
    if rank == 0:
        tokens = ws * calls * C5_CALL * C5_LEN
        line = {"metric": C5_METRIC, "value": tokens / (pf_ms / 1000.0), "unit": "tok/s", "n_gpus": ws,
                "steps": calls, "warmup": 1, "ms_per_step": pf_ms / calls, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights N(0,0.02) seed 4, prompt ids uniform seed 5)",
                "config": {"workload": f"140M-class One bf16: {ws * calls * C5_CALL} prompts x {C5_LEN} tokens "
                                       f"({calls} calls of {C5_CALL} per GPU), then {dsteps} decode steps at batch "
                                       f"{C5_CALL} per GPU (positions {C5_LEN} .. {C5_LEN + dsteps - 1})",
                           "prefill_s": pf_ms / 1000.0, "decode_steps": dsteps,
                           "decode_ms_per_step": dec_ms / (dsteps - 1),
                           "decode_tok_s": ws * C5_CALL * (dsteps - 1) / (dec_ms / 1000.0),
                           "oracle_checked_prompts": checked},
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)


MOE_T, MOE_D, MOE_E, MOE_K, MOE_R = 16384, 768, 8, 2, 64
MOE_METRIC = "LinearMoE TFLOP/s (16384 x 768 bf16, 8 experts top-2, r 64, 768 -> 768)"


def moe_inputs():
    """x ~ N(0, 1) seed 3; LinearMoE(768, 768, 8 experts, top-2, r 64) with the random-init rule
    (weights, gate and experts N(0, 0.02), biases and bias2 zero)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(MOE_T, MOE_D, generator=g).bfloat16()
    n = lambda *shape: torch.empty(shape).normal_(0.0, 0.02, generator=g).bfloat16()
    p = {"weight": n(MOE_D, MOE_D), "bias": torch.zeros(MOE_D).bfloat16(), "gate": n(MOE_R, MOE_D),
         "experts": n(MOE_E), "bias2": torch.zeros(MOE_E, MOE_D).bfloat16()}
    return x, p


def moe_flops(tokens):
    """gate (D -> r) and shared Linear (D -> D) GEMMs: 2 * tokens * D * (D + r)."""
    return 2.0 * tokens * MOE_D * (MOE_D + MOE_R)


def moe_cpu(tokens: int) -> dict:
    from oracle import one_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    x, p = moe_inputs()
    xs = x[:tokens]
    O.linear_moe(xs[:64], p, MOE_K)  # warm-up
    t0 = time.perf_counter()
    O.linear_moe(xs, p, MOE_K)
    dt = time.perf_counter() - t0
    return {"value": moe_flops(tokens) / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds": dt,
            "sample": f"{tokens} of {MOE_T} tokens, oracle restatement of LinearMoE.forward in bf16"}


def run_linear_moe(args, ws, rank, local):
    """One step = the LinearMoE operator (clamp, gate GEMM, router: softmax, expert factors,
    exact expert sums, top-k, combine; shared Linear) on all 16384 tokens."""
    import ctypes
    from one import _capi as C, turbo_ops
    dev = f"cuda:{local}"
    x, p = moe_inputs()
    x = x.to(dev)
    pc = {k: v.to(dev).contiguous() for k, v in p.items()}
    out = torch.empty(MOE_T, MOE_D, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(MOE_T, MOE_K, dtype=torch.int32, device=dev)
    wsb = C.LIB.one_linear_moe_workspace_bytes(MOE_T, MOE_D, MOE_R, 0)
    wsp = torch.empty(wsb, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    st = ctypes.c_void_p(stream.cuda_stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # x + out = 50 MB < L2

    def op(xin, o):
        C.check(C.LIB.one_linear_moe(C.ptr(xin), MOE_T, MOE_D, MOE_D, C.ptr(pc["weight"]), C.ptr(pc["bias"]),
                                     C.ptr(pc["gate"]), C.ptr(pc["experts"]), C.ptr(pc["bias2"]), MOE_E, MOE_R, MOE_K,
                                     0, C.ptr(o), C.ptr(idx), C.ptr(wsp), wsb, st), "one_linear_moe")

    for _ in range(args.warmup):
        op(x, out)
    torch.cuda.synchronize()
    barrier(ws)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            op(x, out)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(ws, sum(a.elapsed_time(b) for a, b in ev))
    value = ws * moe_flops(MOE_T) * args.steps / (ms / 1000.0) / 1e12
    code = turbo_ops.ops_error()
    if code != (0, 0):
        raise RuntimeError(f"device error {code}")
    # e2e through the C ABI with host buffers: x in, y and the top-k indices out, every step
    hx = x.cpu().pin_memory()
    hy = torch.empty(MOE_T, MOE_D, dtype=torch.bfloat16).pin_memory()
    hi = torch.empty(MOE_T, MOE_K, dtype=torch.int32).pin_memory()
    xd = torch.empty_like(x)
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xd.copy_(hx, non_blocking=True)
        op(xd, out)
        hy.copy_(out, non_blocking=True)
        hi.copy_(idx, non_blocking=True)
    e1.record(stream)
    e1.synchronize()
    e_ms = max_over_ranks(ws, e0.elapsed_time(e1))
    e2e = ws * moe_flops(MOE_T) * args.steps / (e_ms / 1000.0) / 1e12
    _, tf, _, src = peaks()
    clocks = clk.summary()
    if rank == 0:
        line = {"metric": MOE_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (x ~ N(0,1) seed 3; weights, gate, experts N(0,0.02); biases zero)",
                "config": {"workload": "isolated LinearMoE(768, 768, num_experts=8, top_k=2, r=64) on 16384 tokens",
                           "tokens_per_s": ws * MOE_T * args.steps / (ms / 1000.0),
                           "l2": "256 MB buffer written between timed calls (x + y = 50 MB < L2)"},
                "roofline": {"bound": "tensor", "kernel": "one_linear_moe (clamp, gate GEMM, router, shared GEMM)",
                             "achieved": value / ws, "peak": tf, "unit": "TFLOP/s", "frac": value / ws / tf,
                             "peak_source": src, "traffic": None,
                             "algorithmic_bytes": 2 * MOE_T * MOE_D * 2 + (MOE_D + MOE_R) * MOE_D * 2},
                "e2e": {"value": e2e, "unit": "TFLOP/s", "h2d_bytes_per_step": MOE_T * MOE_D * 2,
                        "d2h_bytes_per_step": MOE_T * (MOE_D * 2 + MOE_K * 4)},
                "gpu_launches": 4 * args.steps, "clocks": clocks}
        if ws == 1 and not args.no_cpu_baseline:
            r = moe_cpu(MOE_T)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)


def run_linear_moe_reference(args):
    r = moe_cpu(MOE_T)
    line = {"impl": "reference", "metric": MOE_METRIC, "value": r["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 1, "ms_per_step": 1000 * r["seconds"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (x ~ N(0,1) seed 3)",
            "config": {"workload": "isolated LinearMoE(768, 768, num_experts=8, top_k=2, r=64) on 16384 tokens"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_case(args):
    """Small fixed case for ncu captures: 140M engine at batch 256, a 16-token prompt, then
    three graph-replayed decode steps (launch order: prompt kernels, then 76 per step)."""
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    eng = OneEngine(cfg, init_state_dict(cfg, SEED, torch.bfloat16), "cuda", torch.bfloat16, max_batch=BATCH,
                    max_tokens=BATCH * 16)
    g = torch.Generator().manual_seed(SEED)
    eng.prefill(torch.randint(0, cfg.vocab_size, (BATCH, 16), generator=g).cuda())
    eng.capture(1)
    for _ in range(3):
        eng.replay()
    torch.cuda.synchronize()
    if eng.device_error() != (0, 0):
        raise RuntimeError(f"device error {eng.device_error()}")
    print(json.dumps({"profile_case": "ok", "launches_per_step": eng.step_launches(BATCH),
                      "prefill_launches": eng.prefill_launches(BATCH, 16)}))


def profile_prefill(args):
    """Small fixed prompt-ingestion case for ncu captures: 140M engine, one call of 20 prompts of
    4096 tokens, the smallest prompt set whose GEMMs take the persistent path (>= 2 tiles per SM).
    Launch order per layer: row_pre, scan, GEMM A, attention, gate GEMM, 3 routers, x_moe GEMM,
    gate/up GEMM, down GEMM (persistent GEMMs 0..4 of layer 0)."""
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    b, s = 20, 4096
    eng = OneEngine(cfg, init_state_dict(cfg, SEED, torch.bfloat16), "cuda", torch.bfloat16, max_batch=b,
                    max_tokens=b * s)
    g = torch.Generator().manual_seed(PF_SEED)
    eng.prefill(torch.randint(0, cfg.vocab_size, (b, s), generator=g).cuda())
    torch.cuda.synchronize()
    if eng.device_error() != (0, 0):
        raise RuntimeError(f"device error {eng.device_error()}")
    print(json.dumps({"profile_prefill": "ok", "tokens": b * s, "launches": eng.prefill_launches(b, s)}))


def profile_flash(args):
    """Small fixed case for ncu captures of the use_flash_attention path: the 140M model with the
    flag set, one prompt-ingestion call of 4 prompts x 2048 tokens (launch order per layer: row_pre,
    scan, GEMM A, q | k | v per token, the causal sequence attention, ...)."""
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    cfg.use_flash_attention = True
    b, s = 4, 2048
    eng = OneEngine(cfg, init_state_dict(cfg, SEED, torch.bfloat16), "cuda", torch.bfloat16, max_batch=b,
                    max_tokens=b * s)
    g = torch.Generator().manual_seed(PF_SEED)
    eng.prefill(torch.randint(0, cfg.vocab_size, (b, s), generator=g).cuda())
    torch.cuda.synchronize()
    if eng.device_error() != (0, 0):
        raise RuntimeError(f"device error {eng.device_error()}")
    print(json.dumps({"profile_flash": "ok", "tokens": b * s, "launches": eng.prefill_launches(b, s)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="decode: fixed global batch split over the GPUs (strong scaling); default 256 per GPU")
    ap.add_argument("--profile-case", action="store_true", help="run the small ncu case and exit")
    ap.add_argument("--profile-prefill", action="store_true", help="run the small prompt-ingestion ncu case and exit")
    ap.add_argument("--profile-flash", action="store_true",
                    help="run the small use_flash_attention prompt-ingestion ncu case and exit")
    ap.add_argument("--workload", default="decode", choices=["decode", "attention", "linear_moe", "prefill", "config5"],
                    help="decode: the 140M decode step (default); attention: the isolated RoPE + attention op; "
                         "linear_moe: the isolated LinearMoE op on 16384 tokens; prefill: 64 x 4096-token prompts; "
                         "config5: 4096 x 4096 prompts over the GPUs, then 32768 decode steps at batch 64")
    ap.add_argument("--c5-prompts", type=int, default=C5_PROMPTS, help="config5: prompts over all GPUs")
    ap.add_argument("--c5-steps", type=int, default=C5_DECODE, help="config5: decode steps")
    args = ap.parse_args()
    if args.profile_prefill:
        profile_prefill(args)
        return
    if args.profile_flash:
        profile_flash(args)
        return
    if args.profile_case:
        profile_case(args)
        return
    if args.impl == "reference":
        # rank 0 alone times the host-CPU reference; other ranks exit without work
        if int(os.environ.get("RANK", "0")) == 0:
            if args.workload == "attention":
                run_attention_reference(args)
            elif args.workload == "linear_moe":
                run_linear_moe_reference(args)
            elif args.workload == "prefill":
                run_prefill_reference(args)
            else:
                run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), 0)
        return
    ws, rank, local = dist_init()
    try:
        if args.workload == "attention":
            run_attention(args, ws, rank, local)
        elif args.workload == "linear_moe":
            run_linear_moe(args, ws, rank, local)
        elif args.workload == "prefill":
            run_prefill(args, ws, rank, local)
        elif args.workload == "config5":
            run_config5(args, ws, rank, local)
        else:
            run_native(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
