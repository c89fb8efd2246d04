"""GPU parity of the benchmark workloads at the token counts the benchmark runs.

bench.py times cfg3 at 8192 tokens, cfg4 at 4096 and cfg5 at 256; those
counts select the schedules the timed runs use (multi-CTA groupings, the
CTA-pair and persistent tcgen05 GEMMs, the warp-per-token combines), so they
are checked here at exactly those sizes.  Every loop runs on the GPU over all
tokens through the C ABI (BlockEngine -> sb_block_forward); the CPU oracle then
recomputes a seeded sample of 512 rows from the same loop input (teacher
forced: the block is token-independent, so a row's result depends only on that
row):

* router and edge indices of the sampled rows bit-exact (rows within fp32
  rounding of a tie excluded and counted);
* the dispatch plan of ALL rows -- per-expert offsets, token order and summed
  weights -- bit-exact against the reference's plan (build_dispatch_plan order,
  spider_infer/forge/ep/dispatch.py:56-115) built from the device's routing;
* messages within 1e-4, delta and h_out within the activation tolerance
  (bf16 / fp8 2e-2, int4 3e-2; relative to each row's max-norm).

Workloads run with the expert FFN each names (SwiGLU), and cfg3 / cfg5 also
with the reference's erf-GELU FFN (spider_moe/sparse_experts.py:59-62).
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig, benchmark_configs
from spider_web_moe_b200.engine import BlockEngine

from helpers import TIE_REL, TOL, compare_indices, rel_err

pytestmark = pytest.mark.gpu

SAMPLE = 512


def workload_engine(name, activation, device):
    """The benchmark's block (same seeds as bench.py) and the oracle parameters
    with the expert weights exactly as the device stores them."""
    spec = benchmark_configs()[name]
    cfg = ModelConfig(**spec["model"], expert_activation=activation).validate()
    wf = spec["wfmt"]
    if wf == "int4":
        cfg.moe_int4_group_size = 128
    sd = synth.synthetic_state_dict(cfg, seed=0, device=device, zipf=1.1 if spec["zipf"] else None,
                                    round_bf16=True)
    eng = BlockEngine(cfg, sd, device, act_dtype=torch.bfloat16, max_tokens=spec["tokens"], weight_format=wf)
    p = O.params_from_state_dict({k: v.cpu() for k, v in sd.items()}, cfg.num_experts)
    del sd
    names = ["up", "down"] + (["gate"] if activation == "swiglu" else [])
    for short in names:
        q, s, _ = eng.expert_tensors(short)
        if wf == "fp8":
            w = O.dequantize_fp8_per_channel(q.view(torch.float8_e4m3fn).cpu(), s.cpu())
        elif wf == "int4":
            w = O.dequantize_int4(q.cpu(), s.float().cpu(), 128)
        else:
            continue
        setattr(p, "w_" + short, w)
    return cfg, spec, eng, p


def check_workload_loop(eng, cfg, p, cur, x0, loop, rows, tol, label):
    """Loop `loop` on all tokens of `cur` on the GPU; the sampled `rows` against the oracle."""
    n = cur.shape[0]
    taps = eng.make_taps(n)
    out = eng.forward(cur, x0, loop, loop + 1, taps=taps)
    torch.cuda.synchronize()
    eng.check_status()
    h_s = cur[rows].float().cpu()
    x_s = x0[rows].float().cpu()
    want = O.block_forward(p, h_s, x_s, loop, cfg)
    ties = O.topk_margin(want["probs"], cfg.top_k) < TIE_REL
    rows_c = rows.cpu()
    bad, nt = compare_indices(taps["top_idx"][rows], want["top_idx"], ties)
    assert bad == 0, f"{label} loop {loop}: {bad} of {rows.numel()} sampled router rows differ ({nt} ties)"
    sel = want["top_idx"].long()
    src_logits = torch.gather(want["edge_logits"], 1, sel.unsqueeze(-1).expand(-1, -1, cfg.num_experts))
    e_ties = (O.topk_margin(src_logits, cfg.edges_per_expert) < TIE_REL) | ties.unsqueeze(-1)
    want_e = torch.gather(want["edge_idx"], 1, sel.unsqueeze(-1).expand(-1, -1, cfg.edges_per_expert))
    bad, _ = compare_indices(taps["edge_idx"][rows], want_e, e_ties)
    assert bad == 0, f"{label} loop {loop}: {bad} sampled edge rows differ"
    keep = ~(ties | e_ties.any(-1))  # activations of tie rows legitimately differ
    assert rel_err(taps["messages"][rows].cpu()[keep], want["messages"][keep]) < 1e-4, f"{label} messages"
    assert rel_err(taps["delta"][rows].cpu()[keep], want["delta"][keep]) < tol, f"{label} delta"
    assert rel_err(out[rows].cpu()[keep], want["h_out"][keep]) < tol, f"{label} h_out"
    # the whole dispatch plan, bit-exact against the reference's plan of the device routing
    off, tok, w = O.plan_offsets(O.dispatch_plan(taps["top_idx"].cpu().long(), taps["top_w"].cpu(),
                                                 cfg.num_experts), cfg.num_experts)
    assert torch.equal(taps["ffn_offsets"].cpu().long(), off), f"{label} loop {loop}: expert offsets"
    used = int(off[-1])
    assert torch.equal(taps["ffn_rows"].cpu().long()[:used], tok), f"{label} loop {loop}: permutation"
    assert torch.equal(taps["ffn_weights"].cpu()[:used], w), f"{label} loop {loop}: summed weights"
    # the sampled rows' experts appear in the plan exactly where the oracle's routing puts them
    for r, e_row in zip(rows_c[keep][:32].tolist(), want["top_idx"][keep][:32].tolist()):
        for e in set(e_row):
            seg = tok[off[e]:off[e + 1]]
            assert bool((seg == r).any()), f"{label}: row {r} missing from expert {e}"
    return out, int(nt)


@pytest.mark.parametrize("name,activation", [
    ("cfg3", "swiglu"), ("cfg3", "gelu"), ("cfg4", "swiglu"), ("cfg5", "swiglu"), ("cfg5", "gelu"),
    ("cfg2", "swiglu")])
def test_benchmark_workload_all_loops_at_full_size(name, activation, cuda_device):
    cfg, spec, eng, p = workload_engine(name, activation, cuda_device)
    n = spec["tokens"]
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=1, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1).contiguous()
    g = torch.Generator().manual_seed(1234)
    rows = torch.randperm(n, generator=g)[:min(SAMPLE, n)].sort().values.to(cuda_device)
    tol = TOL[{"bf16": "bf16", "fp8": "fp8", "int4": "int4"}[spec["wfmt"]]]
    cur, ties = h, 0
    for loop in range(cfg.num_loops):
        cur, nt = check_workload_loop(eng, cfg, p, cur, h, loop, rows, tol, f"{name}/{activation}")
        ties += nt
    checked = rows.numel() * cfg.num_loops
    assert ties <= checked // 50, f"{ties} of {checked} rows are ties: the tie rule would hide real mismatches"


def test_full_size_graph_replay_matches_eager(cuda_device):
    """The captured graph bench.py times computes what the eager loops compute (cfg3, 8192 tokens)."""
    from spider_web_moe_b200.engine import CapturedBlock

    cfg, spec, eng, _ = workload_engine("cfg3", "swiglu", cuda_device)
    n = spec["tokens"]
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=1, device=cuda_device, dtype=torch.bfloat16)
    h = h.view(n, -1).contiguous()
    eager = eng.forward(h, h).clone()
    g = CapturedBlock(eng, n, x0_is_h=True)
    out = g(h).clone()
    torch.cuda.synchronize()
    eng.check_status()
    assert torch.equal(out, eager)
