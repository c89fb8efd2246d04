"""Failure detection among CPU ranks (gloo): a rank that leaves between steps.

Rank 1 runs one loop of the token-sharded expert-parallel block with rank 0,
then exits without taking part in the next loop's exchange (the host-side
stand-in for a rank that died between steps: none of its work is in flight).
Rank 0's next exchange must end with an error from the process group's short
timeout instead of waiting forever, and rank 0 must have computed the first
loop correctly before that.
"""
import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.ep import ep_loop

CFG = dict(hidden_size=32, num_heads=4, num_experts=4, top_k=2, edges_per_expert=2, num_loops=2,
           expert_ffn_size=48, loop_embed_size=8)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, result_q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from oracle import spider_oracle as O
    from ep_cpu_ops import CpuOps

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    cfg = ModelConfig(**CFG).validate()
    sd = synth.synthetic_state_dict(cfg, seed=23)
    p = O.params_from_state_dict(sd, cfg.num_experts)
    n = 4
    h, _ = synth.block_inputs(n * world, cfg.hidden_size, seed=24)
    h = h.view(-1, cfg.hidden_size)[rank * n:(rank + 1) * n]
    ops = CpuOps(p, cfg, rank, world)
    out = ep_loop(ops, h, h, 0, world, n)
    want = O.block_forward(p, h, h, 0, cfg)["h_out"]
    ok0 = float((out - want).abs().max() / want.abs().max()) < 1e-5
    if rank == 1:
        report(result_q, (rank, ok0, "left"))
        os._exit(0)  # leaves between loops: no collective of it is in flight
    try:
        ep_loop(ops, out, h, 1, world, n)
        report(result_q, (rank, ok0, "no error"))
    except Exception as e:  # the process group's timeout ends the exchange with an error
        report(result_q, (rank, ok0, f"error: {type(e).__name__}"))
    os._exit(0)


def report(q, item):
    """Put and flush before the process leaves with os._exit."""
    q.put(item)
    q.close()
    q.join_thread()


def test_surviving_rank_gets_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    for pr in procs:
        if pr.exitcode is None:
            pr.kill()
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
    res = dict((r, (ok, what)) for r, ok, what in (q.get(timeout=10) for _ in range(2)))
    assert res[1] == (True, "left")
    ok0, what = res[0]
    assert ok0, "rank 0's first loop differs from the oracle"
    assert what.startswith("error"), f"rank 0's exchange after the peer left: {what}"
