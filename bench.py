"""Decode throughput of the 140M-class MedIT One model in bf16 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

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
        self.path = os.path.join(REPO, "gpurun_out", f"clocks_rank{idx}.csv") if os.path.isdir(
            os.path.join(REPO, "gpurun_out")) else f"/tmp/one_clocks_{os.getpid()}.csv"

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


def cpu_reference(cfg, steps: int, warmup: int, batch: int, context: int) -> dict:
    """The reference's cached decode on the host CPU: per-layer norm_x history of `context`
    tokens (seeded random bf16, as left by a prompt), one new token per step."""
    from one.initialization import init_state_dict
    from oracle import one_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    oc = O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, transformer_dim=cfg.transformer_dim,
                        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                        head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                        top_k_experts=cfg.top_k_experts, r=cfg.r)
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
    return {"value": batch * steps / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} decode steps of {batch} sequences at context {context}..{context + warmup + steps} "
                      f"(oracle restatement of the reference's cached decode, bf16, {warmup} untimed)",
            "seconds": dt}


def run_reference(args, ws, rank):
    from one.configuration_one import config_140m
    if rank != 0:
        return
    cfg = config_140m()
    # bounded sample: each CPU step of 256 sequences takes ~0.5 s; cap the run
    steps = max(1, min(args.steps, 8))
    warmup = max(0, min(args.warmup, 2))
    r = cpu_reference(cfg, steps, warmup, BATCH, PROMPT)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 1000 * r["seconds"] / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, uniform ids)",
            "config": {"workload": "140M-class One, bf16, greedy decode, 256 sequences, context 128", "batch": BATCH,
                       "prompt": PROMPT},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_native(args, ws, rank, local):
    from one.configuration_one import config_140m
    from one.engine import OneEngine
    from one.initialization import init_state_dict
    cfg = config_140m()
    sd = init_state_dict(cfg, SEED, torch.bfloat16)
    steps, warmup = args.steps, args.warmup
    eng = OneEngine(cfg, sd, f"cuda:{local}", torch.bfloat16, max_batch=BATCH, max_tokens=BATCH * PROMPT,
                    hist_cap=max(steps + warmup + 64, 256), max_positions=PROMPT + 2 * (steps + warmup) + 4096)
    del sd
    g = torch.Generator().manual_seed(SEED + rank)
    prompt = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=g)
    eng.prefill(prompt.cuda())
    eng.capture(1)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        eng.replay()
    torch.cuda.synchronize()
    barrier(ws)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(steps):
            eng.replay()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize()
    barrier(ws)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ws, ms)
    code = eng.device_error()
    if code != (0, 0):
        raise RuntimeError(f"device error {code}")
    value = ws * BATCH * steps / (ms_max / 1000.0)
    # outside the timed region: every rank's generated tokens to every rank (NCCL all-gather)
    from one import distributed as Dd
    tokens = Dd.gather_tokens(eng.history(min(steps + warmup, eng.hist_cap), BATCH).t().contiguous(), BATCH * ws)
    assert tokens.shape[0] == BATCH * ws

    # e2e through the public step API: pinned host ids in, next ids out, every step
    ids_host = torch.randint(0, cfg.vocab_size, (BATCH,), dtype=torch.int32, generator=g).pin_memory()
    out_host = torch.empty(BATCH, dtype=torch.int32).pin_memory()
    ids_dev = torch.empty(BATCH, dtype=torch.int32, device=f"cuda:{local}")
    for _ in range(max(warmup, 2)):
        ids_dev.copy_(ids_host, non_blocking=True)
        _, nx = eng.step(ids_dev)
        out_host.copy_(nx, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    barrier(ws)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e_start.record(stream)
    for _ in range(steps):
        ids_dev.copy_(ids_host, non_blocking=True)
        _, nx = eng.step(ids_dev)
        out_host.copy_(nx, non_blocking=True)
        stream.synchronize()
        ids_host.copy_(out_host)
    e_end.record(stream)
    e_end.synchronize()
    e_ms = max_over_ranks(ws, e_start.elapsed_time(e_end))
    e2e = ws * BATCH * steps / (e_ms / 1000.0)

    hbm, tf, tf_sus, src = peaks()
    sb = step_bytes(cfg, BATCH)
    t_step = ms_max / 1000.0 / steps
    achieved = sb["total"] / t_step / 1e9
    launches = eng.step_launches(BATCH)
    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
            "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights N(0,0.02) seed 4, uniform prompt ids)",
            "config": {"workload": "140M-class One (vocab 32000, hidden 768, 12 layers, 12 heads, 8 experts top-2, "
                                   "FFN 3072), bf16 greedy decode after a 128-token prompt",
                       "batch_per_gpu": BATCH, "global_batch": BATCH * ws, "prompt": PROMPT,
                       "parallelism": f"sequence-sharded dp{ws}, no collective on the step path",
                       "l2": "inputs larger than L2 (285 MB of weights streamed per step)"},
            "roofline": {"bound": "hbm", "kernel": f"decode step ({launches} launches, CUDA graph)",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": src, "traffic": None, "algorithmic_bytes_per_step": sb["total"],
                         "tflops_achieved": sb["flops"] / t_step / 1e12,
                         "tensor_frac_sustained": sb["flops"] / t_step / 1e12 / tf_sus},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": BATCH * 4, "d2h_bytes_per_step": BATCH * 4},
            "gpu_launches": launches * steps,
            "clocks": clocks,
        }
        if ws == 1 and not args.no_cpu_baseline:
            r = cpu_reference(cfg, 3, 1, BATCH, PROMPT)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
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
    print(json.dumps({"profile_case": "ok", "launches_per_step": eng.step_launches(BATCH)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", action="store_true", help="run the small ncu case and exit")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args)
        return
    if args.impl == "reference":
        # rank 0 alone times the host-CPU reference; other ranks exit without work
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), 0)
        return
    ws, rank, local = dist_init()
    try:
        run_native(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
