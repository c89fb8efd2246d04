"""Expert-parallel exchange logic on CPU ranks (gloo, world 2 and 3).

Each rank holds its own tokens; experts are owned by e % world.  The loop of
spider_web_moe_b200.ep (pack, all-to-all, owner-side experts, all-to-all back,
combine) with CPU compute steps must give every rank exactly what the
single-process oracle gives for that rank's tokens with all experts local.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.ep import ep_loop, local_expert_ids

CFG = dict(hidden_size=32, num_heads=4, num_experts=6, top_k=2, edges_per_expert=2, num_loops=2,
           expert_ffn_size=48, loop_embed_size=8)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, n_per_rank, result_q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from oracle import spider_oracle as O
    from ep_cpu_ops import CpuOps

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ModelConfig(**CFG).validate()
        sd = synth.synthetic_state_dict(cfg, seed=21, zipf=1.1)
        p = O.params_from_state_dict(sd, cfg.num_experts)
        h, _ = synth.block_inputs(n_per_rank * world, cfg.hidden_size, seed=22)
        h = h.view(-1, cfg.hidden_size)[rank * n_per_rank:(rank + 1) * n_per_rank]
        ops = CpuOps(p, cfg, rank, world)
        cap = n_per_rank
        out, want = h, h
        for l in range(cfg.num_loops):
            out = ep_loop(ops, out, h, l, world, cap)
            want = O.block_forward(p, want, h, l, cfg)["h_out"]
        err = float((out - want).abs().max() / want.abs().max())
        result_q.put((rank, err, local_expert_ids(cfg.num_experts, rank, world)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ep_loop_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, 5, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
        assert pr.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    owned = sorted(e for _, _, ids in res for e in ids)
    assert owned == list(range(CFG["num_experts"]))        # every expert owned exactly once
    for rank, err, _ in res:
        assert err < 1e-5, f"rank {rank}: relative error {err}"
