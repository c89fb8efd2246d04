"""Lumen global workspace on the B200 kernels (sb_lumen_forward).

Checked against what the reference computed (tests/golden/lumen.pt): its
LumenWorkspace on its own (output, slots, slot weights, broadcast, J-lens
logits and read-out ids) and a SpiderMoELayer with use_lumen over two loops
with return_stats (h and the lumen_* statistics).  Plus the oracle on bf16 /
larger shapes through both GEMM engines, and the all-loop drivers.
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.layer import SpiderMoELayer
from spider_web_moe_b200.lumen import LumenWorkspace

from helpers import golden_cfg, load_golden, rel_err

pytestmark = pytest.mark.gpu


def test_module_matches_reference_fixture(cuda_device):
    m = load_golden("lumen")["module"]
    ws = LumenWorkspace(hidden_size=64, num_slots=4, slot_dim=16, vocab_size=50)
    ws.load_state_dict(m["state_dict"])
    ws = ws.to(cuda_device).eval()
    h = m["h"].to(cuda_device)
    with torch.no_grad():
        out, st = ws(h, return_state=True, j_lens=True)
        plain = ws(h)
    assert out.shape == h.shape and st.slots.shape == (2, 5, 4, 16) and st.slot_weights.shape == (2, 5, 4)
    assert rel_err(out, m["out"]) < 1e-5
    assert torch.equal(plain, out)
    for k in ("slots", "slot_weights", "broadcast", "j_logits"):
        assert rel_err(getattr(st, k), m[k]) < 1e-5, k
    assert ws.read_j_space(st, top_k=3) == m["j_space"]
    assert ws.stats()["name"] == "Lumen" and ws.stats()["j_lens"]


def test_layer_with_lumen_matches_reference_fixture(cuda_device):
    fx = load_golden("lumen")
    cfg = golden_cfg(fx)
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=fx["seed"], std=fx["std"])
    layer = layer.to(cuda_device).eval()
    x0 = fx["x0"].to(cuda_device)
    for rec in fx["records"]:
        with torch.no_grad():
            out, st = layer(rec["h_in"].to(cuda_device), x0, rec["loop_idx"], return_stats=True)
            plain = layer(rec["h_in"].to(cuda_device), x0, rec["loop_idx"])
        want = rec["stats"]
        assert set(want) <= set(st)
        assert rel_err(out, rec["h_out"]) < 1e-5
        assert torch.equal(plain, out)
        assert rel_err(st["lumen_slot_weights"], want["lumen_slot_weights"]) < 1e-5
        assert rel_err(st["lumen_broadcast_norm"].reshape(1, -1), want["lumen_broadcast_norm"].reshape(1, -1)) < 1e-5
        assert rel_err(st["confidence"].reshape(1, -1), want["confidence"].reshape(1, -1)) < 1e-5
        assert torch.equal(st["expert_load"].cpu(), want["expert_load"])
    # all loops in one driver call (Lumen after each loop's LayerNorm)
    h0 = fx["records"][0]["h_in"].to(cuda_device)
    assert rel_err(layer.run_recurrent_full(h0, x0), fx["records"][-1]["h_out"]) < 2e-5


@pytest.mark.parametrize("H,S,dt,engine,n", [(1024, 8, torch.bfloat16, "auto", 300), (256, 16, torch.float32, "simt", 70),
                                             (512, 8, torch.bfloat16, "simt", 33)])
def test_lumen_matches_oracle(H, S, dt, engine, n, cuda_device):
    torch.manual_seed(H + S)
    ws = LumenWorkspace(hidden_size=H, num_slots=S)
    with torch.no_grad():
        for p in ws.parameters():
            p.copy_(torch.randn_like(p) * 0.05)
        ws.norm.weight.fill_(1.0)
        ws.norm.bias.zero_()
        if dt == torch.bfloat16:
            for p in ws.parameters():
                p.copy_(p.bfloat16().float())
    ws.engine_name = engine
    ws = ws.to(cuda_device).eval()
    h = torch.randn(n, H).to(dt).float()
    with torch.no_grad():
        out, st = ws(h.to(cuda_device, dt), return_state=True)
    want, wst = O.lumen_forward(h, {k: v.cpu() for k, v in ws.state_dict().items()})
    tol = 2e-2 if dt == torch.bfloat16 else 1e-5
    assert rel_err(out, want) < tol
    # the state comes back in the activation dtype (bf16 rounding: 2^-8 relative)
    assert rel_err(st.slot_weights.float(), wst["slot_weights"]) < (8e-3 if dt == torch.bfloat16 else 1e-5)
    assert rel_err(st.broadcast.float(), wst["broadcast"]) < tol
