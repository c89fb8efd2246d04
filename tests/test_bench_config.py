"""bench.py's JSON line on CPU: both arms describe a workload with the same
``config`` dict, the parallelism text follows --gpus / --parallel /
--micro-batches, and the roofline's algorithmic bytes cover every weight format
a workload names (cfg1's native weights run as bf16)."""
import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from spider_web_moe_b200.config import benchmark_configs  # noqa: E402


def parse(argv, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    return bench.parse()


@pytest.mark.parametrize("name", sorted(benchmark_configs()))
def test_both_arms_print_the_same_config(name, monkeypatch):
    args = parse(["--config", name], monkeypatch)
    cfg, spec = bench.workload(args)
    mine = bench.workload_config(args, cfg, spec, 1)
    ref_args = parse(["--config", name, "--impl", "reference"], monkeypatch)
    cfg_r, spec_r = bench.workload(ref_args)
    assert bench.workload_config(ref_args, cfg_r, spec_r, 1) == mine
    assert mine["workload"] == name and mine["tokens_per_step_per_gpu"] == spec["tokens"]
    assert mine["expert_activation"] == spec["activation"] and mine["parallelism"] == "single GPU"


def test_parallelism_text(monkeypatch):
    args = parse(["--gpus", "8"], monkeypatch)
    cfg, spec = bench.workload(args)
    assert bench.workload_config(args, cfg, spec, 8)["parallelism"].startswith("dp8")
    args = parse(["--gpus", "8", "--parallel", "ep"], monkeypatch)
    text = bench.workload_config(args, cfg, spec, 8)["parallelism"]
    assert text.startswith("ep8") and "micro-batches" not in text
    args = parse(["--gpus", "8", "--parallel", "ep", "--micro-batches", "2", "--transport", "nccl"], monkeypatch)
    text = bench.workload_config(args, cfg, spec, 8)["parallelism"]
    assert "NCCL all-to-all" in text and "two micro-batches" in text


@pytest.mark.parametrize("name", sorted(benchmark_configs()))
def test_algorithmic_bytes_every_format(name, monkeypatch):
    args = parse(["--config", name], monkeypatch)
    cfg, spec = bench.workload(args)
    n, K, M, E = 8, cfg.top_k, cfg.edges_per_expert, cfg.num_experts
    g = torch.Generator().manual_seed(0)
    top = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(n)])
    edges = torch.stack([torch.randperm(E, generator=g)[:K * M] for _ in range(n)])
    taps = {"top_idx": top.to(torch.int32), "ffn_offsets": torch.tensor([0, n * K]),
            "edge_idx": edges.to(torch.int32)}
    b = bench.algorithmic_bytes(cfg, spec, taps, n)
    assert set(b) == {"gemm_expert_up", "gemm_expert_down", "gemm_edge_values"}
    assert all(v > 0 for v in b.values())
