"""Token-sharded expert-parallel block on the GPU.

On one GPU the EP path (route, pack, owner-side experts, combine) runs with a
world of one and must match the full block loop by loop.  With two or more
GPUs, tests/ep_worker.py runs under torchrun (NCCL) and checks every rank
against a full single-GPU block on its own tokens.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig, benchmark_configs
from spider_web_moe_b200.engine import BlockEngine
from spider_web_moe_b200.ep import ExpertParallelBlock

from helpers import rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("name,n,activation", [("cfg2", 40, "gelu"), ("cfg5", 40, "gelu"), ("cfg3", 1024, "swiglu"),
                                               ("cfg4", 700, "swiglu"), ("cfg4", 2100, "swiglu"),
                                               ("cfg5", 2048, "swiglu")])
def test_ep_path_single_gpu_matches_block(name, n, activation, cuda_device):
    """The token-sharded EP loop at a world of one (route, pack, owner-side
    experts on the packed rows, combine, epilogue) against the block; the
    prefill-size cases take the tensor-core schedules on materialised rows, and
    from 128 expected rows per expert (cfg4 at 2100 tokens, cfg5 at 2048) the
    owner holds its fp8 / int4 experts as resident bf16 copies."""
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"], expert_activation=activation).validate()
    sd = synth.synthetic_state_dict(cfg, seed=41, device=cuda_device, zipf=1.1 if spec["zipf"] else None,
                                    round_bf16=True)
    ep = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"])
    full = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"])
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=42, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1)
    for l in range(cfg.num_loops):
        a = ep.loop(h, h, l)
        b = full.forward(h, h, l, l + 1)
        torch.cuda.synchronize()
        assert rel_err(a, b) < 2e-2, f"loop {l}"
        h = b


@pytest.mark.parametrize("name,n", [("cfg2", 40), ("cfg5", 40), ("cfg2", 600), ("cfg4", 700)])
def test_peer_transport_single_gpu_matches_nccl_path(name, n, cuda_device):
    """World of one over the peer-memory transport (the rank's own region as its
    only peer): the dispatch, flag waits and return run, and the outputs are
    bit-identical to the NCCL-transport path, eagerly and from a CUDA graph
    replayed twice (the flags keep counting across loops and replays).  From
    512 rows the owner's return and the source's epilogue run warp per row."""
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"], expert_activation=spec["activation"]).validate()
    sd = synth.synthetic_state_dict(cfg, seed=45, device=cuda_device, zipf=1.1 if spec["zipf"] else None,
                                    round_bf16=True)
    ref = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"])
    peer = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n,
                               weight_format=spec["wfmt"], transport="peer")
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=46, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1)
    try:
        want = ref.forward(h, h)
        got = peer.forward(h, h)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        peer.capture(n)
        for _ in range(2):
            out = peer.replay(h, h)
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        peer.dense.check_status()
    finally:
        peer.close()


@pytest.mark.parametrize("transport", ["nccl", "peer"])
@pytest.mark.parametrize("name,n", [("cfg2", 41), ("cfg4", 700)])
def test_micro_batches_match_one_batch(transport, name, n, cuda_device):
    """micro_batches=2: the rank's tokens as two halves on two streams, each
    with engines, an exchange group and (peer transport) regions of its own.
    The block is token-independent, so the result is the one-batch step run on
    each half (the same routing batch sizes, so no top-k near-tie can flip;
    the owner's GEMM schedules follow the exchange capacity, hence the GEMM
    tolerance), and a CUDA graph of the two-stream step replays it bit for bit."""
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"], expert_activation=spec["activation"]).validate()
    sd = synth.synthetic_state_dict(cfg, seed=47, device=cuda_device, zipf=1.1 if spec["zipf"] else None,
                                    round_bf16=True)
    one = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n,
                              weight_format=spec["wfmt"], transport=transport)
    two = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n,
                              weight_format=spec["wfmt"], transport=transport, micro_batches=2)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=48, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1)
    try:
        n0 = (n + 1) // 2
        want = torch.cat([one.forward(h[:n0], h[:n0]), one.forward(h[n0:], h[n0:])])
        got = two.forward(h, h)
        torch.cuda.synchronize()
        two.check_status()
        assert rel_err(got, want) < 2e-2
        two.capture(n)
        for _ in range(2):
            out = two.replay(h, h)
            torch.cuda.synchronize()
            assert torch.equal(out, got)
        two.check_status()
    finally:
        one.close()
        two.close()


def test_ep_owner_hot_expert_loops_row_tiles(cuda_device):
    """200 tokens with two experts taking every token: the owner plans 64-row tiles
    per expert (32 expected pairs per expert on average), so each hot expert's
    CTA loops over four row tiles."""
    cfg = ModelConfig(hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2,
                      num_loops=1, expert_ffn_size=512).validate()
    n = 200
    sd = synth.synthetic_state_dict(cfg, seed=43, device=cuda_device, round_bf16=True)
    sd["loop_bias"][0, 5] = 40.0
    sd["loop_bias"][0, 9] = 30.0
    ep = ExpertParallelBlock(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format="bf16")
    full = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=44, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1)
    a = ep.loop(h, h, 0)
    b = full.forward(h, h, 0, 1)
    torch.cuda.synchronize()
    ep.local.check_status()
    assert rel_err(a, b) < 2e-2


def test_reference_semantics_path_matches_block(cuda_device, monkeypatch):
    """The drop-in layer's expert-parallel forward (route, this rank's experts,
    SUM all-reduce, LayerNorm epilogue: all library calls) at a world of one
    with expert parallelism forced on computes what the block computes."""
    from spider_web_moe_b200 import expert_parallel as EPH
    from spider_web_moe_b200.layer import SpiderMoELayer

    spec = benchmark_configs()["cfg2"]
    cfg = ModelConfig(**spec["model"]).validate()
    n = 24
    sd = synth.synthetic_state_dict(cfg, seed=47, device="cpu", round_bf16=True)
    layer = SpiderMoELayer(cfg)
    layer.load_state_dict(sd, strict=False)
    layer = layer.to(cuda_device).eval()
    full = BlockEngine(cfg, {k: v.to(cuda_device) for k, v in sd.items()}, cuda_device, act_dtype=torch.bfloat16,
                       max_tokens=n)
    calls = []
    monkeypatch.setattr(EPH, "ep_enabled", lambda: True)
    monkeypatch.setattr(EPH, "get_rank_world", lambda: (0, 1))
    monkeypatch.setattr(EPH, "all_reduce_sum_", lambda t: calls.append(t.shape) or t)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=48, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(1, n, -1)
    for l in range(2):
        got = layer(h, h, l)
        want = full.forward(h, h, l, l + 1)
        torch.cuda.synchronize()
        assert rel_err(got, want) < 2e-2, f"loop {l}"
        h = want
    assert len(calls) == 2 and calls[0] == (n, cfg.hidden_size)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_nccl_and_peer():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
