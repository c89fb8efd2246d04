"""GPU parity of the whole block against the oracle and the reference fixtures.

Every case runs the CUDA path through the C ABI (libspider_b200.so via the
BlockEngine) and compares with the CPU oracle on the same seeded inputs:
routing / edge indices and the dispatch permutation bit-exact (rows within
fp32 rounding of a tie excluded and counted), activations within the stated
relative tolerance (fp32 1e-5, bf16 / fp8 2e-2, int4 3e-2).
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200.config import ModelConfig, benchmark_configs
from spider_web_moe_b200.engine import BlockEngine, CapturedBlock
from spider_web_moe_b200 import synth

from helpers import TIE_REL, TOL, compare_indices, golden_cfg, golden_state, load_golden, rel_err
from test_oracle_golden import oracle_params

pytestmark = pytest.mark.gpu

FIXTURES = [("cfg1_model", "fp32", "simt"), ("e4_fp32", "fp32", "simt"), ("e16_fp32", "fp32", "simt"),
            ("e16_zipf_bf16", "bf16", "tcgen05"), ("e16_zipf_bf16", "bf16", "simt"),
            ("e64_fp8", "fp8", "tcgen05"), ("e64_fp8", "fp8", "simt"),
            ("e128_int4", "int4", "tcgen05"), ("e128_int4", "int4", "simt")]


def engine_for_fixture(fx, cfg, kind, engine, device):
    sd = golden_state(fx, cfg)
    dt = torch.float32 if kind == "fp32" else torch.bfloat16
    wf = {"fp32": "native", "bf16": "bf16", "fp8": "fp8", "int4": "int4"}[kind]
    if kind == "int4":
        cfg.moe_int4_group_size = fx["int4_group"]
    return BlockEngine(cfg, sd, device, act_dtype=dt, max_tokens=fx["tokens"], weight_format=wf, engine=engine), dt


def check_loop(eng, cfg, rec_in, x0, l, want, tol, dt, label):
    """Run loop l on the GPU from rec_in and compare with the dict `want`."""
    n = rec_in.numel() // cfg.hidden_size
    dev = eng.device
    h = rec_in.reshape(n, -1).to(dev, dt)
    x = x0.reshape(n, -1).to(dev, dt)
    taps = eng.make_taps(n)
    out = eng.forward(h, x, l, l + 1, taps=taps)
    torch.cuda.synchronize()
    eng.check_status()
    probs = want["probs"]
    ties = O.topk_margin(probs, cfg.top_k) < TIE_REL
    bad, nt = compare_indices(taps["top_idx"], want["top_idx"], ties)
    assert bad == 0, f"{label} loop {l}: {bad} router rows differ ({nt} ties)"
    assert rel_err(taps["top_w"], want["top_w"]) < max(tol, 1e-5) * (0.1 if dt == torch.float32 else 1)
    # Edge indices: only rows of selected sources exist on the device ([n, K, M]).
    sel = want["top_idx"].long()
    e_logits = want["edge_logits"]
    src_logits = torch.gather(e_logits, 1, sel.unsqueeze(-1).expand(-1, -1, cfg.num_experts))
    e_ties = O.topk_margin(src_logits, cfg.edges_per_expert) < TIE_REL
    e_ties = e_ties | ties.unsqueeze(-1)
    want_e = torch.gather(want["edge_idx"], 1, sel.unsqueeze(-1).expand(-1, -1, cfg.edges_per_expert))
    bad, _ = compare_indices(taps["edge_idx"], want_e, e_ties)
    assert bad == 0, f"{label} loop {l}: {bad} edge rows differ"
    mtol = 1e-5 if dt == torch.float32 else 1e-4
    assert rel_err(taps["messages"], want["messages"]) < mtol, f"{label} messages"
    assert rel_err(taps["delta"], want["delta"]) < tol, f"{label} delta"
    assert rel_err(out, want["h_out"].reshape(n, -1)) < tol, f"{label} h_out"
    # dispatch permutation, bit-exact vs the reference plan
    if not bool(ties.any()):
        off, tok, w = O.plan_offsets(O.dispatch_plan(want["top_idx"], want["top_w"], cfg.num_experts),
                                     cfg.num_experts)
        got_off = taps["ffn_offsets"].cpu().long()
        assert torch.equal(got_off, off), f"{label} offsets"
        assert torch.equal(taps["ffn_rows"].cpu().long()[: int(off[-1])], tok), f"{label} permutation"
    return out


@pytest.mark.parametrize("name,kind,engine", FIXTURES)
def test_block_matches_reference_fixture(name, kind, engine, cuda_device):
    fx = load_golden(name)
    cfg = golden_cfg(fx)
    eng, dt = engine_for_fixture(fx, cfg, kind, engine, cuda_device)
    p = oracle_params(fx, cfg)
    tol = TOL[kind]
    for rec in fx["records"]:
        l = rec["loop_idx"]
        h_in = rec["h_in"]
        if dt == torch.bfloat16:
            h_in = h_in.to(torch.bfloat16).float()  # teacher forcing with the bf16 block input
        want = O.block_forward(p, h_in, rec["x0"], l, cfg)
        check_loop(eng, cfg, h_in, rec["x0"], l, want, tol, dt, f"{name}/{engine}")
        # and the reference's own output for this loop
        n = h_in.numel() // cfg.hidden_size
        out = eng.forward(h_in.reshape(n, -1).to(cuda_device, dt), rec["x0"].reshape(n, -1).to(cuda_device, dt),
                          l, l + 1)
        if dt == torch.float32:
            assert rel_err(out, rec["h_out"].reshape(n, -1)) < tol


def full_config(name, tokens=None, activation="gelu"):
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"], expert_activation=activation).validate()
    return cfg, spec, tokens or spec["tokens"]


@pytest.mark.parametrize("name,tokens,engine,activation", [
    ("cfg2", None, "tcgen05", "gelu"), ("cfg2", None, "simt", "gelu"), ("cfg3", 512, "tcgen05", "gelu"),
    ("cfg4", 128, "tcgen05", "gelu"), ("cfg5", 64, "tcgen05", "gelu"), ("cfg5", 64, "simt", "gelu"),
    ("cfg2", None, "tcgen05", "swiglu"), ("cfg2", None, "simt", "swiglu"), ("cfg3", 512, "tcgen05", "swiglu"),
    ("cfg4", 128, "tcgen05", "swiglu"), ("cfg4", 128, "simt", "swiglu"), ("cfg5", 64, "tcgen05", "swiglu"),
    ("cfg5", 64, "simt", "swiglu")])
def test_full_size_config_one_loop(name, tokens, engine, activation, cuda_device):
    """Full-width configs (bounded token counts for the CPU oracle), loop 1, teacher forced;
    the reference's GELU FFN and the SwiGLU mode (gate weights expert_gates.*) in bf16, fp8
    and int4 on both engines."""
    cfg, spec, n = full_config(name, tokens, activation)
    zipf = 1.1 if spec["zipf"] else None
    sd = synth.synthetic_state_dict(cfg, seed=0, device=cuda_device, zipf=zipf, round_bf16=True)
    wf = spec["wfmt"]
    if wf == "int4":
        cfg.moe_int4_group_size = 128
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=wf,
                      engine=engine)
    sd_cpu = {k: v.cpu() for k, v in sd.items()}
    p = O.params_from_state_dict(sd_cpu, cfg.num_experts)
    for short in ["up", "down"] + (["gate"] if activation == "swiglu" else []):
        q, s, _ = eng.expert_tensors(short)
        if wf == "fp8":
            setattr(p, "w_" + short, (q.view(torch.float8_e4m3fn).float() * s.unsqueeze(-1)).cpu())
        if wf == "int4":
            setattr(p, "w_" + short, O.dequantize_int4(q.cpu(), s.float().cpu(), 128))
    h, x0 = synth.block_inputs(n, cfg.hidden_size, seed=1)
    h = h.to(torch.bfloat16).float()
    want = O.block_forward(p, h, h, 1, cfg)
    check_loop(eng, cfg, h, h, 1, want, TOL[{"bf16": "bf16", "fp8": "fp8", "int4": "int4"}[wf]],
               torch.bfloat16, f"{name}/{engine}")


def test_engines_agree_and_are_deterministic(cuda_device):
    """tcgen05 and CUDA-core engines agree loop by loop (same input to both); each
    engine is bitwise deterministic across calls (no float atomics anywhere)."""
    cfg, spec, n = full_config("cfg2")
    sd = synth.synthetic_state_dict(cfg, seed=3, device=cuda_device, round_bf16=True)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=4, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1)
    engs = {e: BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, engine=e)
            for e in ("tcgen05", "simt")}
    for name, eng in engs.items():
        a = eng.forward(h, h).clone()
        b = eng.forward(h, h).clone()
        torch.cuda.synchronize()
        eng.check_status()
        assert torch.equal(a, b), f"{name} not deterministic"
    cur = h
    for l in range(cfg.num_loops):
        outs, taps = {}, {}
        for name, eng in engs.items():
            taps[name] = eng.make_taps(n)
            outs[name] = eng.forward(cur, h, l, l + 1, taps=taps[name]).clone()
        same = (taps["tcgen05"]["top_idx"] == taps["simt"]["top_idx"]).all(-1) & \
               (taps["tcgen05"]["edge_idx"] == taps["simt"]["edge_idx"]).reshape(n, -1).all(-1)
        # rows whose routing differs can only be near-ties of the fp32 logits
        assert int((~same).sum()) <= max(1, n // 32), f"loop {l}: {int((~same).sum())} rows route differently"
        keep = same.cpu()
        assert rel_err(outs["tcgen05"][same], outs["simt"][same]) < 2e-2
        cur = outs["tcgen05"]


def test_cuda_graph_replay_matches_eager(cuda_device):
    cfg, spec, n = full_config("cfg2")
    sd = synth.synthetic_state_dict(cfg, seed=5, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=6, device=cuda_device, dtype=torch.bfloat16)
    eager = eng.forward(h, h).clone()
    g = CapturedBlock(eng, n)
    out = g(h.view(n, -1), h.view(n, -1)).clone()
    torch.cuda.synchronize()
    assert torch.equal(out.view_as(eager), eager)


@pytest.mark.parametrize("n", [1, 7, 37, 130, 1536])
def test_ragged_token_counts(n, cuda_device):
    cfg = ModelConfig(hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2,
                      num_loops=2, expert_ffn_size=512).validate()
    sd = synth.synthetic_state_dict(cfg, seed=7, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n)
    p = O.params_from_state_dict({k: v.cpu() for k, v in sd.items()}, cfg.num_experts)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=8)
    h = h.to(torch.bfloat16).float()
    want = O.block_forward(p, h, h, 0, cfg)
    check_loop(eng, cfg, h, h, 0, want, TOL["bf16"], torch.bfloat16, f"n={n}")


def test_zero_tokens_is_a_noop(cuda_device):
    cfg = ModelConfig(hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2,
                      num_loops=2, expert_ffn_size=512).validate()
    sd = synth.synthetic_state_dict(cfg, seed=7, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=4)
    h = torch.zeros(0, cfg.hidden_size, device=cuda_device, dtype=torch.bfloat16)
    out = eng.forward(h, h)
    assert out.shape == h.shape


@pytest.mark.parametrize("n", [200, 300])
def test_all_tokens_on_one_expert(n, cuda_device):
    """A dominant loop bias sends every token to the same experts (one huge group).
    With 200 tokens the expected rows per expert stay small, so the hot expert's
    rows are covered by one CTA looping over several row tiles; with 300 the
    row tiles are spread over CTAs."""
    cfg = ModelConfig(hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2,
                      num_loops=1, expert_ffn_size=512).validate()
    sd = synth.synthetic_state_dict(cfg, seed=9, device=cuda_device, round_bf16=True)
    sd["loop_bias"][0, 3] = 40.0
    sd["loop_bias"][0, 11] = 30.0
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n)
    p = O.params_from_state_dict({k: v.cpu() for k, v in sd.items()}, cfg.num_experts)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=10)
    h = h.to(torch.bfloat16).float()
    want = O.block_forward(p, h, h, 0, cfg)
    check_loop(eng, cfg, h, h, 0, want, TOL["bf16"], torch.bfloat16, "one-expert")


@pytest.mark.parametrize("wf,activation", [("fp8", "swiglu"), ("int4", "swiglu"), ("fp8", "gelu"), ("int4", "gelu")])
def test_quantised_prefill_through_bf16_copies(wf, activation, cuda_device):
    """Prefill-size batches (here 256 expected rows per expert) of fp8 / int4
    experts convert the expert weights to bf16 once per call and run the bf16
    CTA-pair GEMMs (fp8 keeping its per-row scale in the epilogue): the same
    weights the in-GEMM dequantisation makes, checked against the oracle."""
    cfg = ModelConfig(hidden_size=512, num_heads=4, num_experts=8, top_k=2, edges_per_expert=2, num_loops=1,
                      expert_ffn_size=512, expert_activation=activation, moe_int4_group_size=128).validate()
    n = 1024
    sd = synth.synthetic_state_dict(cfg, seed=13, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=wf)
    p = O.params_from_state_dict({k: v.cpu() for k, v in sd.items()}, cfg.num_experts)
    for short in ["up", "down"] + (["gate"] if activation == "swiglu" else []):
        q, s, _ = eng.expert_tensors(short)
        if wf == "fp8":
            setattr(p, "w_" + short, (q.view(torch.float8_e4m3fn).float() * s.unsqueeze(-1)).cpu())
        else:
            setattr(p, "w_" + short, O.dequantize_int4(q.cpu(), s.float().cpu(), 128))
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=14)
    h = h.to(torch.bfloat16).float()
    want = O.block_forward(p, h, h, 0, cfg)
    check_loop(eng, cfg, h, h, 0, want, TOL[wf], torch.bfloat16, f"{wf}/{activation}/bf16-copies")
