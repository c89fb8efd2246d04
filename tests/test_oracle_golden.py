"""Pin the CPU oracle against fixtures captured from the reference (CPU only).

tests/golden/*.pt hold what the reference's own SpiderMoELayer computed
(captured by tests/golden/make_golden.py); the oracle must reproduce them
before it may check the CUDA path.
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import quant as Q
from spider_web_moe_b200 import synth
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import TIE_REL, compare_indices, golden_cfg, golden_state, load_golden, rel_err

CASES = ["cfg1_model", "e4_fp32", "e16_fp32", "e16_zipf_bf16", "e64_fp8", "e128_int4"]


def oracle_params(fx, cfg):
    sd = golden_state(fx, cfg)
    p = O.params_from_state_dict(sd, cfg.num_experts)
    if fx.get("fp8"):
        q_up, s_up = O.quantize_fp8_per_channel(p.w_up)
        q_dn, s_dn = O.quantize_fp8_per_channel(p.w_down)
        p.w_up = O.dequantize_fp8_per_channel(q_up, s_up)
        p.w_down = O.dequantize_fp8_per_channel(q_dn, s_dn)
    if fx.get("int4_group"):
        gs = fx["int4_group"]
        pu, su = O.quantize_int4(p.w_up, gs)
        pd, sd_ = O.quantize_int4(p.w_down, gs)
        p.w_up = O.dequantize_int4(pu, su.bfloat16().float(), gs)
        p.w_down = O.dequantize_int4(pd, sd_.bfloat16().float(), gs)
    return p


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_reference(name):
    fx = load_golden(name)
    cfg = golden_cfg(fx)
    p = oracle_params(fx, cfg)
    for rec in fx["records"]:
        l = rec["loop_idx"]
        r = O.block_forward(p, rec["h_in"], rec["x0"], l, cfg)
        n = r["top_idx"].shape[0]
        ties = O.topk_margin(r["probs"], cfg.top_k) < TIE_REL
        bad, _ = compare_indices(r["top_idx"], rec["top_indices"].reshape(n, -1), ties)
        assert bad == 0, f"{name} loop {l}: router indices differ"
        assert rel_err(r["top_w"], rec["top_weights"].reshape(n, -1)) < 1e-6
        e_ties = (rec["edge_margin"].reshape(n, cfg.num_experts) < TIE_REL)
        bad, _ = compare_indices(r["edge_idx"], rec["edge_indices"].reshape(n, cfg.num_experts, -1), e_ties)
        assert bad == 0, f"{name} loop {l}: edge indices differ"
        assert rel_err(r["messages"], rec["messages"]) < 1e-5
        assert rel_err(r["delta"], rec["delta"]) < 1e-5
        assert rel_err(r["h_out"], rec["h_out"]) < 1e-5
        off, tok, w = O.plan_offsets(O.dispatch_plan(r["top_idx"], r["top_w"], cfg.num_experts),
                                     cfg.num_experts)
        assert torch.equal(off, rec["plan_offsets"])
        assert torch.equal(tok, rec["plan_tokens"])
        assert rel_err(w.view(1, -1), rec["plan_weights"].view(1, -1)) < 1e-6


@pytest.mark.parametrize("name", [c for c in CASES if c != "cfg1_model"])
def test_synthetic_params_match_reference_draw(name):
    """The seeded parameter generator draws exactly what the fixture's reference module held."""
    import hashlib

    fx = load_golden(name)
    cfg = golden_cfg(fx)
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=fx["seed"], zipf=fx["zipf"])
    if fx["bf16"]:
        synth.round_params_to_bf16_(layer)
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], zipf=fx["zipf"], round_bf16=fx["bf16"])
    for k, v in layer.state_dict().items():
        assert torch.equal(v.float(), sd[k]), k
    if fx.get("fp8"):
        return  # the fixture digest is of the dequantised weights; checked in test_quant_formats
    h = hashlib.sha256()
    for k, v in layer.named_parameters():
        h.update(k.encode())
        h.update(v.detach().float().contiguous().numpy().tobytes())
    assert h.hexdigest() == fx["param_digest"]


def tensor_digest(t):
    import hashlib

    t = t.detach().contiguous()
    if t.is_floating_point():
        t = t.float()
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def test_quant_formats_match_reference_vectors():
    v = load_golden("quant_vectors")
    for gs in (64, 128):
        for mod in (O, None):
            if mod is O:
                packed, scales = O.quantize_int4(v["w"], gs)
                deq = O.dequantize_int4(packed, scales, gs)
            else:
                q = Q.quantize_int4(v["w"], gs)
                packed, scales, deq = q.packed, q.scales, q.dequantize(torch.float32)
            assert torch.equal(packed, v[f"int4_g{gs}_packed"])
            assert torch.equal(scales, v[f"int4_g{gs}_scales"])
            assert torch.equal(deq, v[f"int4_g{gs}_deq"])
    s = v["fp8_scale"]
    qo, so = O.quantize_fp8_per_channel(v["fp8_w"])
    qp = Q.quantize_fp8_per_channel(v["fp8_w"])
    assert torch.equal(so, s) and torch.equal(qp.scale, s)
    assert torch.equal(qo.view(torch.uint8), v["fp8_q_u8"])
    assert torch.equal(qp.q.view(torch.uint8), v["fp8_q_u8"])


def test_quantized_expert_fixtures():
    """int4 / fp8 expert packing of the fixtures' bf16 weights matches the reference bytes."""
    fx = load_golden("e128_int4")
    cfg = golden_cfg(fx)
    sd = golden_state(fx, cfg)
    up = torch.stack([sd[f"experts.{i}.0.weight"] for i in range(cfg.num_experts)])
    down = torch.stack([sd[f"experts.{i}.2.weight"] for i in range(cfg.num_experts)])
    qu, qd = Q.quantize_int4(up, 128), Q.quantize_int4(down, 128)
    assert tensor_digest(qu.packed) == fx["int4_digest"]["up_packed"]
    assert tensor_digest(qd.packed) == fx["int4_digest"]["down_packed"]
    assert tensor_digest(qu.scales.bfloat16().float()) == fx["int4_digest"]["up_scales"]
    assert tensor_digest(qd.scales.bfloat16().float()) == fx["int4_digest"]["down_scales"]
    fx = load_golden("e64_fp8")
    cfg = golden_cfg(fx)
    sd = golden_state(fx, cfg)
    for i in range(cfg.num_experts):
        for j in (0, 2):
            q = Q.quantize_fp8_per_channel(sd[f"experts.{i}.{j}.weight"])
            assert tensor_digest(q.q.view(torch.uint8)) == fx["fp8_digest"][f"experts.{i}.{j}.q"]
            assert tensor_digest(q.scale) == fx["fp8_digest"][f"experts.{i}.{j}.s"]


def test_oracle_stats_match_reference():
    """return_stats=True (model.py:324-349): the oracle's loop statistics equal
    what the reference layer returned, loop by loop."""
    fx = load_golden("e8_stats")
    cfg = golden_cfg(fx)
    p = oracle_params(fx, cfg)
    ew, eb = fx["exit_head"]["weight"], fx["exit_head"]["bias"]
    h = fx["records"][0]["h_in"]
    for rec in fx["records"]:
        r = O.block_forward(p, h, fx["x0"], rec["loop_idx"], cfg)
        assert rel_err(r["h_out"], rec["h_out"]) < 1e-5
        st = O.loop_stats(r, ew, eb, cfg.num_experts)
        want = rec["stats"]
        assert torch.equal(st["expert_load"], want["expert_load"])
        assert torch.equal(st["edge_load"], want["edge_load"])
        assert rel_err(st["router_probs"], want["router_probs"].reshape(-1, cfg.num_experts)) < 1e-6
        for k in ("aux_loss", "edge_loss"):
            assert abs(float(st[k]) - float(want[k])) <= 1e-6 * abs(float(want[k])), k
        assert rel_err(st["confidence"].view(1, -1), want["confidence"].reshape(1, -1)) < 1e-6
        h = rec["h_out"]


def test_oracle_early_exit_decode_matches_reference():
    """_run_recurrent_decode(h, x0, early_exit=True) (model.py:450-473): the
    oracle's active rows per loop and returned h equal the reference's."""
    fx = load_golden("e8_early_exit")
    cfg = golden_cfg(fx)
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], std=fx["std"])
    p = O.params_from_state_dict(sd, cfg.num_experts)
    ew, eb = fx["exit_head"]["weight"], fx["exit_head"]["bias"]
    out, trace = O.run_recurrent_decode(p, fx["h"], fx["x0"], cfg, ew, eb, fx["threshold"])
    assert [t.numel() for t in trace] == fx["active_rows"]
    assert len(set(fx["active_rows"])) >= 4  # rows leave at several different loops
    assert rel_err(out, fx["out"]) < 1e-5


def test_oracle_lumen_matches_reference():
    """LumenWorkspace.forward (lumen.py:81-123) on its own and inside the layer
    with return_stats (model.py:318-348): the oracle reproduces the reference."""
    fx = load_golden("lumen")
    m = fx["module"]
    out, st = O.lumen_forward(m["h"], m["state_dict"], j_lens=True)
    assert rel_err(out, m["out"]) < 1e-5
    for k in ("slots", "slot_weights", "broadcast", "j_logits"):
        assert rel_err(st[k], m[k]) < 1e-5, k
    cfg = golden_cfg(fx)
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], std=fx["std"])
    p = O.params_from_state_dict(sd, cfg.num_experts)
    for rec in fx["records"]:
        r = O.block_forward(p, rec["h_in"], fx["x0"], rec["loop_idx"], cfg)
        assert rel_err(r["h_out"], rec["h_out"]) < 1e-5
        want = rec["stats"]
        got = O.loop_stats(r, sd["exit_head.weight"], sd["exit_head.bias"], cfg.num_experts)
        assert rel_err(got["lumen_slot_weights"], want["lumen_slot_weights"].reshape(-1, 4)) < 1e-5
        assert rel_err(got["lumen_broadcast_norm"].view(1, -1), want["lumen_broadcast_norm"].reshape(1, -1)) < 1e-5
        assert torch.equal(got["expert_load"], want["expert_load"])


def test_fp8_helpers_match_reference_vectors():
    """quant.py's general fp8 helpers reproduce the reference's bytes and values."""
    v = load_golden("fp8_helpers")
    x = v["x"]
    q, s = Q.quantize_fp8(x)
    assert torch.equal(q.view(torch.uint8), v["q"]) and torch.equal(s, v["s"])
    assert torch.equal(Q.compute_fp8_scale(x), v["scale"])
    q2, s2 = Q.quantize_fp8(x, 0.05)
    assert torch.equal(q2.view(torch.uint8), v["q2"]) and torch.equal(s2, v["s2"])
    q3, s3 = Q.quantize_fp8(x, torch.tensor([0.02]))
    assert torch.equal(q3.view(torch.uint8), v["q3"]) and torch.equal(s3, v["s3"])
    assert torch.equal(Q.dequantize_fp8(q, s), v["deq"])
    assert torch.equal(Q.dequantize_fp8(q, s, torch.bfloat16), v["deq_bf16"])
    assert torch.equal(Q.dequantize_fp8(q), v["deq_plain"])
    q4 = Q.quantize_fp8_with_scale_tensor(x, v["rows"])
    assert torch.equal(q4.view(torch.uint8), v["q4"])
    assert torch.equal(Q.dequantize_fp8_with_scale_tensor(q4, v["rows"]), v["deq4"])
    assert Q.fp8_available() and Q.is_fp8_dtype(Q.fp8_dtype()) and not Q.is_fp8_dtype(torch.float16)
