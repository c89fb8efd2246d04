"""return_stats=True statistics (sb_loop_stats) against the reference and the oracle.

The reference histograms the top-M destinations of all E sources
(model.py:329-333), so the device recomputes the full edge logits; these tests
check the module's stats dict against what the reference layer returned
(tests/golden/e8_stats.pt) and the engine entry point against the oracle's
restatement (oracle.loop_stats) over expert counts that take every selection
path (E <= 32, 64, 128, 256), both activation dtypes and both GEMM engines.
Counts are compared exactly except for (token, source) rows whose top-M is an
fp32-rounding tie; float statistics at 1e-5.
"""
import math

import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.engine import BlockEngine
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import golden_cfg, load_golden, rel_err, topk_tie_mask

pytestmark = pytest.mark.gpu


def close(a, b, tol=1e-5):
    a, b = float(a), float(b)
    if math.isnan(b):
        return math.isnan(a)
    return abs(a - b) <= tol * max(abs(b), 1e-6)


def test_module_stats_match_reference_fixture(cuda_device):
    fx = load_golden("e8_stats")
    cfg = golden_cfg(fx)
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=fx["seed"])
    layer.exit_head.load_state_dict(fx["exit_head"])
    layer = layer.to(cuda_device).eval()
    x0 = fx["x0"].to(cuda_device)
    for rec in fx["records"]:
        with torch.no_grad():
            out, st = layer(rec["h_in"].to(cuda_device), x0, rec["loop_idx"], return_stats=True)
        want = rec["stats"]
        assert set(want) <= set(st)
        assert rel_err(out, rec["h_out"]) < 1e-5
        assert torch.equal(st["expert_load"].cpu(), want["expert_load"])
        assert torch.equal(st["edge_load"].cpu(), want["edge_load"])
        assert st["router_probs"].shape == want["router_probs"].shape
        assert rel_err(st["router_probs"], want["router_probs"]) < 1e-5
        assert close(st["aux_loss"], want["aux_loss"]) and close(st["edge_loss"], want["edge_loss"])
        assert st["confidence"].shape == want["confidence"].shape
        assert rel_err(st["confidence"].reshape(1, -1), want["confidence"].reshape(1, -1)) < 1e-5


CASES = [
    # E, K, M, H, tokens, dtype, engine
    (16, 2, 2, 128, 64, torch.bfloat16, "auto"),
    (64, 4, 3, 128, 300, torch.bfloat16, "auto"),
    (64, 4, 3, 128, 300, torch.bfloat16, "simt"),
    (128, 8, 4, 256, 40, torch.float32, "auto"),
    (256, 2, 4, 64, 20, torch.float32, "auto"),
    (16, 2, 2, 64, 1, torch.float32, "auto"),
]


@pytest.mark.parametrize("E,K,M,H,n,dt,engine", CASES)
def test_loop_stats_match_oracle(E, K, M, H, n, dt, engine, cuda_device):
    cfg = ModelConfig(hidden_size=H, num_heads=4, num_experts=E, top_k=K, edges_per_expert=M, num_loops=2,
                      expert_ffn_size=64).validate()
    bf16 = dt == torch.bfloat16
    sd = synth.synthetic_state_dict(cfg, seed=E + n, zipf=1.1, round_bf16=bf16)
    eng = BlockEngine(cfg, {k: v.to(cuda_device) for k, v in sd.items()}, cuda_device, act_dtype=dt,
                      max_tokens=max(n, 1), engine=engine)
    g = torch.Generator().manual_seed(n)
    h = torch.randn(n, H, generator=g).to(dt).float()
    h_out = torch.randn(n, H, generator=g).to(dt).float()
    exit_w = torch.randn(1, H, generator=g) * 0.1
    exit_b = torch.tensor([0.3])
    l = 1
    st = eng.loop_stats(h.to(cuda_device, dt), h_out.to(cuda_device, dt), l, exit_w=exit_w.to(cuda_device),
                        exit_b=exit_b.to(cuda_device))
    torch.cuda.synchronize()
    eng.check_status()
    p = O.params_from_state_dict(sd, E)
    top_w, top_idx, probs = O.router(h, p.router_w, p.loop_bias[l], K)
    edge_idx, edge_w, edge_logits = O.edge_graph(h, p.loop_emb[l], p.gen_w, p.gen_b, E, M)
    want = O.loop_stats(dict(top_idx=top_idx, probs=probs, edge_idx=edge_idx, edge_w=edge_w, h_out=h_out),
                        exit_w, exit_b, E)
    assert rel_err(st["router_probs"], want["router_probs"]) < 1e-5
    # counts: exact outside fp32-rounding ties of the selections
    r_ties = int(topk_tie_mask(probs, K).sum())
    e_ties = int(topk_tie_mask(edge_logits, M).sum())
    cnt = (st["expert_load"].cpu() * n * K).round()
    want_cnt = (want["expert_load"] * n * K).round()
    assert float((cnt - want_cnt).abs().sum()) <= 2 * K * r_ties
    ecnt = (st["edge_load"].cpu() * n * E * M).round()
    want_ecnt = (want["edge_load"] * n * E * M).round()
    assert float((ecnt - want_ecnt).abs().sum()) <= 2 * M * e_ties
    if e_ties == 0:
        assert rel_err(st["edge_importance"].view(1, -1), want["edge_importance"].view(1, -1)) < 1e-5
        assert close(st["edge_loss"], want["edge_loss"])
    if r_ties == 0:
        assert torch.equal(st["expert_load"].cpu(), want["expert_load"])
        assert close(st["aux_loss"], want["aux_loss"])
    assert rel_err(st["confidence"].view(1, -1), want["confidence"].view(1, -1)) < 1e-5


def test_loop_stats_uses_given_routing(cuda_device):
    """top_idx passed in (the forward's routing) is what expert_load counts."""
    cfg = ModelConfig(hidden_size=64, num_heads=4, num_experts=8, top_k=2, edges_per_expert=2, num_loops=1,
                      expert_ffn_size=64).validate()
    sd = synth.synthetic_state_dict(cfg, seed=3, device=cuda_device)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.float32, max_tokens=10)
    h = torch.randn(10, 64, device=cuda_device)
    ti = torch.tensor([[7, 6]] * 10, dtype=torch.int32, device=cuda_device)
    st = eng.loop_stats(h, None, 0, top_idx=ti)
    load = st["expert_load"].cpu()
    assert torch.equal(load, torch.tensor([0, 0, 0, 0, 0, 0, 0.5, 0.5]))
    assert st["confidence"] is None


def test_loop_stats_no_tokens(cuda_device):
    """Zero tokens: loads 0, losses NaN (probs.mean over no tokens), as torch."""
    cfg = ModelConfig(hidden_size=64, num_heads=4, num_experts=8, top_k=2, edges_per_expert=2, num_loops=1,
                      expert_ffn_size=64).validate()
    sd = synth.synthetic_state_dict(cfg, seed=3, device=cuda_device)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.float32, max_tokens=1)
    h = torch.zeros(0, 64, device=cuda_device)
    st = eng.loop_stats(h, h, 0, exit_w=torch.zeros(64, device=cuda_device), exit_b=torch.zeros(1, device=cuda_device))
    assert float(st["expert_load"].abs().sum()) == 0.0 and float(st["edge_load"].abs().sum()) == 0.0
    assert math.isnan(float(st["aux_loss"]))
    assert st["router_probs"].shape == (0, 8) and st["confidence"].shape == (0,)


def test_loop_stats_repeatable(cuda_device):
    """Float sums are per-CTA partials added in a fixed order: bitwise repeatable."""
    cfg = ModelConfig(hidden_size=128, num_heads=4, num_experts=64, top_k=4, edges_per_expert=3, num_loops=1,
                      expert_ffn_size=64).validate()
    sd = synth.synthetic_state_dict(cfg, seed=5, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=2000)
    h = torch.randn(2000, 128, device=cuda_device).bfloat16()
    a = eng.loop_stats(h, h, 0, exit_w=torch.ones(128, device=cuda_device), exit_b=torch.zeros(1, device=cuda_device))
    b = eng.loop_stats(h, h, 0, exit_w=torch.ones(128, device=cuda_device), exit_b=torch.zeros(1, device=cuda_device))
    for k in a:
        assert torch.equal(a[k], b[k]), k
