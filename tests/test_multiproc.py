"""Sequence-sharded decode across ranks (gloo, world size 2, CPU): every rank decodes its
shard with the oracle, tokens are gathered, and the result must equal one process decoding
the whole batch; the max-over-ranks timing helper returns the slowest rank's value."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from one.configuration_one import tiny_config
    from oracle import one_oracle as O
    cfg = tiny_config(num_hidden_layers=1, vocab_size=512)
    oc = O.OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, transformer_dim=cfg.transformer_dim,
                        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                        head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, num_experts=cfg.num_experts,
                        top_k_experts=cfg.top_k_experts, r=cfg.r)
    return cfg, oc


def _decode(ids, steps):
    from one.initialization import init_state_dict
    from oracle import one_oracle as O
    cfg, oc = _cfg()
    sd = init_state_dict(cfg, 11, torch.bfloat16)
    gen, _, _ = O.greedy(O.RunningDecoder(sd, oc, torch.bfloat16), ids, steps)
    return gen


def _worker(rank, world, port, prompt, steps, out):
    import sys
    for p in (os.path.join(REPO, "medit-one_b200"), REPO):
        if p not in sys.path:
            sys.path.insert(0, p)
    from one import distributed as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = D.shard(prompt.shape[0], world, rank)
        local = _decode(prompt[start:start + count], steps)
        allgen = D.gather_tokens(local, prompt.shape[0])
        slowest = D.max_over_ranks(float(rank + 1))
        if rank == 0:
            out.put((allgen, slowest))
    finally:
        dist.destroy_process_group()


def test_shard_covers_batch():
    from one import distributed as D
    for B in (1, 5, 256, 257):
        for W in (1, 2, 3, 8):
            spans = [D.shard(B, W, r) for r in range(W)]
            assert sum(c for _, c in spans) == B
            assert all(spans[r][0] + spans[r][1] == spans[r + 1][0] for r in range(W - 1))


def test_sharded_decode_equals_single_process():
    prompt = torch.randint(0, 512, (5, 6), generator=torch.Generator().manual_seed(2))
    steps = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompt, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    allgen, slowest = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert slowest == 2.0
    assert torch.equal(allgen, _decode(prompt, steps))
