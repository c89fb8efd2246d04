"""Early-exit decode with the active set on the device (sb_active_set_step).

SpiderWebLM._run_recurrent_decode(h, x0, early_exit=True) (model.py:450-473)
loops the block over the batch rows still active and drops rows whose exit
confidence passes the threshold.  Checked against what the reference returned
(tests/golden/e8_early_exit.pt, rows leaving at four different loops) and
against the oracle's restatement (oracle.run_recurrent_decode): the active
rows per loop exactly, h within the dtype's tolerance.  In bf16 the exit
confidence follows the rounding of h, and over several loops rows near the
threshold decide differently from an fp32 oracle; there each loop is checked
teacher-forced instead: the block's output on the device's own active rows
against the oracle (2e-2), the device confidences against the exit head on
those outputs (1e-5), the next active set against those decisions (exactly),
and the returned h against each row's output at the loop it left.
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import synth
from spider_web_moe_b200.backends import get_backend
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.engine import BlockEngine
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import golden_cfg, load_golden, rel_err

pytestmark = pytest.mark.gpu

# The fixture chains five loops of std-0.3 weights without teacher forcing, so
# the fp32 bound of one loop (1e-5) compounds: 1e-5 per loop.
CHAIN_TOL = 5e-5


def golden_layer(fx, cuda_device):
    cfg = golden_cfg(fx)
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=fx["seed"], std=fx["std"])
    layer.exit_head.load_state_dict(fx["exit_head"])
    return cfg, layer.to(cuda_device).eval()


def test_early_exit_matches_reference_fixture(cuda_device):
    fx = load_golden("e8_early_exit")
    cfg, layer = golden_layer(fx, cuda_device)
    eng = layer.engine(cuda_device, torch.float32, fx["h"].shape[0])
    trace = []
    out, loops = eng.run_recurrent_decode(fx["h"].to(cuda_device), fx["x0"].to(cuda_device), fx["threshold"],
                                          layer.exit_head.weight, layer.exit_head.bias, trace=trace)
    torch.cuda.synchronize()
    eng.check_status()
    assert [len(t["rows"]) for t in trace] == fx["active_rows"] and loops == cfg.num_loops
    assert rel_err(out, fx["out"]) < CHAIN_TOL
    got = layer.run_recurrent_decode(fx["h"].to(cuda_device), fx["x0"].to(cuda_device), True, fx["threshold"])
    assert torch.equal(got, out)


class ModelStandIn(torch.nn.Module):
    """The attributes of a SpiderWebLM the backend touches (recurrent, cfg)."""

    def __init__(self, cfg, layer):
        super().__init__()
        self.cfg = cfg
        self.recurrent = layer


def test_backend_routes_recurrent_drivers(cuda_device):
    fx = load_golden("e8_early_exit")
    cfg, layer = golden_layer(fx, cuda_device)
    cfg.early_exit_threshold = fx["threshold"]
    model = get_backend("spider_b200")(cfg, device=cuda_device, model=ModelStandIn(cfg, layer.cpu()))
    h, x0 = fx["h"].to(cuda_device), fx["x0"].to(cuda_device)
    assert rel_err(model._run_recurrent_decode(h, x0, True), fx["out"]) < CHAIN_TOL
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], std=fx["std"])
    want, _ = O.run_loops(O.params_from_state_dict(sd, cfg.num_experts), fx["h"], fx["x0"], cfg)
    assert rel_err(model._run_recurrent_full(h, x0), want) < CHAIN_TOL
    assert rel_err(model._run_recurrent_decode(h, x0, False), want) < CHAIN_TOL


def decode_case(B, T, dt, bias, cuda_device):
    cfg = ModelConfig(hidden_size=128, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2, num_loops=4,
                      expert_ffn_size=128).validate()
    bf16 = dt == torch.bfloat16
    sd = synth.synthetic_state_dict(cfg, seed=B, std=0.2, round_bf16=bf16)
    g = torch.Generator().manual_seed(B + T)
    exit_w = (torch.randn(1, 128, generator=g) * 0.05).to(dt).float()
    exit_b = torch.tensor([bias])
    h = torch.randn(B, T, 128, generator=g).to(dt).float()
    eng = BlockEngine(cfg, {k: v.to(cuda_device) for k, v in sd.items()}, cuda_device, act_dtype=dt,
                      max_tokens=B * T)
    trace = []
    out, _ = eng.run_recurrent_decode(h.to(cuda_device, dt), h.to(cuda_device, dt), cfg.early_exit_threshold,
                                      exit_w.to(cuda_device), exit_b.to(cuda_device), trace=trace)
    torch.cuda.synchronize()
    eng.check_status()
    return cfg, sd, h, exit_w, exit_b, out.cpu(), trace


@pytest.mark.parametrize("B,T,bias", [(40, 3, 1.7), (700, 1, 1.72)])
def test_early_exit_matches_oracle_fp32(B, T, bias, cuda_device):
    cfg, sd, h, exit_w, exit_b, out, trace = decode_case(B, T, torch.float32, bias, cuda_device)
    confs = []
    want, want_trace = O.run_recurrent_decode(O.params_from_state_dict(sd, cfg.num_experts), h, h, cfg, exit_w,
                                              exit_b, cfg.early_exit_threshold, confidences=confs)
    margin = min(float((c - cfg.early_exit_threshold).abs().min()) for c in confs if c.numel())
    assert margin > 1e-5, "seeded case too close to the threshold"
    assert [t["rows"].tolist() for t in trace] == [t.tolist() for t in want_trace]
    assert len({len(t) for t in want_trace}) >= 3
    assert rel_err(out, want) < 1e-5 * cfg.num_loops


@pytest.mark.parametrize("B,bias", [(300, 1.75), (64, 1.7)])
def test_early_exit_bf16_teacher_forced(B, bias, cuda_device):
    cfg, sd, h, exit_w, exit_b, out, trace = decode_case(B, 1, torch.bfloat16, bias, cuda_device)
    p = O.params_from_state_dict(sd, cfg.num_experts)
    thr = cfg.early_exit_threshold
    assert trace[0]["rows"].tolist() == list(range(B))
    last = {}
    for l, t in enumerate(trace):
        r = O.block_forward(p, t["h_in"].float(), h[t["rows"]], l, cfg)
        assert rel_err(t["h_new"], r["h_out"]) < 2e-2, f"loop {l}"
        z = t["h_new"].float()[:, 0, :] @ exit_w.view(-1) + exit_b
        assert rel_err(t["conf"].view(1, -1), torch.sigmoid(z).view(1, -1)) < 1e-5
        stay = t["rows"][~(t["conf"] > thr)]
        if l + 1 < len(trace):
            assert torch.equal(trace[l + 1]["rows"], stay)
            assert torch.equal(trace[l + 1]["h_in"], t["h_new"][~(t["conf"] > thr)])
        for i, row in enumerate(t["rows"].tolist()):
            last[row] = t["h_new"][i]
    assert len({len(t["rows"]) for t in trace}) >= 3
    assert torch.equal(out, torch.stack([last[i] for i in range(B)]))


def test_early_exit_extremes(cuda_device):
    """Threshold above every confidence: all loops for every row (= run_loops);
    below every confidence: one loop, every row leaves after it."""
    cfg = ModelConfig(hidden_size=64, num_heads=4, num_experts=8, top_k=2, edges_per_expert=2, num_loops=3,
                      expert_ffn_size=64).validate()
    sd = synth.synthetic_state_dict(cfg, seed=2, device=cuda_device)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.float32, max_tokens=20)
    h = torch.randn(20, 1, 64, device=cuda_device)
    w, b = torch.randn(64, device=cuda_device), torch.zeros(1, device=cuda_device)
    trace = []
    out, loops = eng.run_recurrent_decode(h, h, 2.0, w, b, trace=trace)
    assert loops == 3 and [len(t["rows"]) for t in trace] == [20, 20, 20]
    assert torch.equal(out, eng.forward(h, h))
    trace = []
    out, loops = eng.run_recurrent_decode(h, h, -1.0, w, b, trace=trace)
    assert loops == 1 and [len(t["rows"]) for t in trace] == [20]
    assert torch.equal(out, eng.forward(h, h, 0, 1))
    empty = torch.zeros(0, 1, 64, device=cuda_device)
    out, loops = eng.run_recurrent_decode(empty, empty, 0.5, w, b)
    assert out.shape == (0, 1, 64) and loops == 0
