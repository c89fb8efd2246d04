"""Two-or-more-GPU check of the token-sharded expert-parallel block (run by torchrun).

Each rank holds its own slice of the tokens; experts are owned by e % world.
Loop by loop (same input to both), the rank's EP output must match a full
single-GPU block on the same tokens: routing identical, h_out within the bf16
tolerance.  The peer-memory transport must give bit-identical outputs to the
NCCL one, eagerly and replayed from a CUDA graph.

The reference's own expert-parallel contract is checked too: the drop-in
SpiderMoELayer and sparse_expert_delta with the process group initialised
(every rank holds ALL tokens, computes its experts e % world, SUM all-reduce
of the delta; spider_moe/sparse_experts.py:38-43,66-67) must give every rank
the single-GPU result.  Exits non-zero on a mismatch.
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from spider_web_moe_b200 import synth  # noqa: E402
from spider_web_moe_b200.config import ModelConfig, benchmark_configs  # noqa: E402
from spider_web_moe_b200.engine import BlockEngine  # noqa: E402
from spider_web_moe_b200.ep import ExpertParallelBlock  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    name = os.environ.get("EP_CONFIG", "cfg2")
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"]).validate()
    n = 48
    sd = synth.synthetic_state_dict(cfg, seed=31, device=dev, zipf=1.1 if spec["zipf"] else None, round_bf16=True)
    ep = ExpertParallelBlock(cfg, sd, dev, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"])
    # the same step over the peer-memory transport (stores into the owners'
    # regions over NVLink instead of NCCL all-to-all): bit-identical rows
    peer = ExpertParallelBlock(cfg, sd, dev, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"],
                               transport="peer")
    full = BlockEngine(cfg, sd, dev, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"])
    h, _ = synth.block_inputs(n * world, cfg.hidden_size, seed=32, device=dev, dtype=torch.bfloat16)
    h = h.view(-1, cfg.hidden_size)[rank * n:(rank + 1) * n].contiguous()
    x0 = h.clone()
    worst = 0.0
    ok = True
    same = True
    for l in range(cfg.num_loops):
        out_ep = ep.loop(h, x0, l)
        out_peer = peer.loop(h, x0, l)
        out_full = full.forward(h, x0, l, l + 1)
        torch.cuda.synchronize()
        same &= torch.equal(out_ep, out_peer)
        num = (out_ep.float() - out_full.float()).abs().amax(-1)
        den = out_full.float().abs().amax(-1).clamp_min(1e-30)
        err = float((num / den).max())
        worst = max(worst, err)
        ok &= err < 2e-2
        h = out_full
    full.check_status()
    peer.dense.check_status()
    # all loops in one CUDA graph over the peer transport, replayed twice
    peer.capture(n)
    h0, _ = synth.block_inputs(n * world, cfg.hidden_size, seed=33, device=dev, dtype=torch.bfloat16)
    h0 = h0.view(-1, cfg.hidden_size)[rank * n:(rank + 1) * n].contiguous()
    want = ep.forward(h0, h0)
    for _ in range(2):
        got = peer.replay(h0, h0)
        torch.cuda.synchronize()
        same &= torch.equal(got, want)
    peer.dense.check_status()
    peer.close()
    # two micro-batches per rank on two streams (their own NCCL communicator or
    # peer regions): the one-batch step's rows, and a graph replays them exactly
    for tr in ("nccl", "peer"):
        two = ExpertParallelBlock(cfg, sd, dev, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"],
                                  transport=tr, micro_batches=2)
        got = two.forward(h0, h0)
        n0 = (n + 1) // 2
        want_mb = torch.cat([ep.forward(h0[:n0], h0[:n0]), ep.forward(h0[n0:], h0[n0:])])
        torch.cuda.synchronize()
        num = (got.float() - want_mb.float()).abs().amax(-1)
        den = want_mb.float().abs().amax(-1).clamp_min(1e-30)
        e2 = float((num / den).max())
        two.capture(n)
        again = two.replay(h0, h0)
        torch.cuda.synchronize()
        two.check_status()
        ok &= e2 < 2e-2 and torch.equal(again, got)
        print(f"rank {rank}/{world} {name}: two micro-batches ({tr}) relative error {e2:.3e}", flush=True)
        two.close()
    ok &= same
    ok &= reference_semantics(cfg, sd, dev, rank, world)
    print(f"rank {rank}/{world} {name}: worst relative error {worst:.3e}, peer transport "
          f"{'identical' if same else 'DIFFERS'} {'ok' if ok else 'MISMATCH'}", flush=True)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 0 else 1)


def reference_semantics(cfg, sd, dev, rank, world) -> bool:
    """Drop-in layer and sparse_expert_delta under the process group vs one GPU."""
    from spider_web_moe_b200.layer import SpiderMoELayer
    from spider_web_moe_b200.sparse_experts import sparse_expert_delta

    n = 40
    layer = SpiderMoELayer(cfg)
    layer.load_state_dict({k: v.cpu() for k, v in sd.items()}, strict=False)
    layer = layer.to(dev).eval()
    full = BlockEngine(cfg, sd, dev, act_dtype=torch.bfloat16, max_tokens=n)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=34, device=dev, dtype=torch.bfloat16)  # same on all ranks
    h = h.view(1, n, -1)
    worst = 0.0
    for l in range(cfg.num_loops):
        got = layer(h, h, l)
        want = full.forward(h, h, l, l + 1)
        torch.cuda.synchronize()
        num = (got.float() - want.float()).abs().amax(-1)
        worst = max(worst, float((num / want.float().abs().amax(-1).clamp_min(1e-30)).max()))
        h = want
    E, U, H = cfg.num_experts, cfg.expert_ffn_size, cfg.hidden_size
    w_up = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).float()
    b_up = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).float()
    w_dn = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).float()
    b_dn = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).float()
    g = torch.Generator().manual_seed(35)
    msgs = torch.randn(2, 8, H, generator=g).to(dev)
    tw, ti = torch.randn(2, 8, E, generator=g).softmax(-1).topk(cfg.top_k, -1)
    tw, ti = tw.to(dev), ti.to(dev)
    d_ep = sparse_expert_delta(msgs, ti, tw, w_up, b_up, w_dn, b_dn, E, cfg.top_k, expert_parallel=True)
    d_one = sparse_expert_delta(msgs, ti, tw, w_up, b_up, w_dn, b_dn, E, cfg.top_k, expert_parallel=False)
    torch.cuda.synchronize()
    d_err = float((d_ep - d_one).abs().max() / d_one.abs().max())
    print(f"rank {rank}/{world} reference semantics: layer worst relative error {worst:.3e}, "
          f"sparse_expert_delta relative error {d_err:.3e}", flush=True)
    return worst < 2e-2 and d_err < 1e-5


if __name__ == "__main__":
    main()
