"""Generate the golden fixtures from the reference implementation itself.

Run in a container where the reference tree is available:

    PYTHONPATH=<reference root>:. python tests/golden/make_golden.py <reference root>

It imports the reference package (``spider_moe``, ``spider_infer``), builds the
reference ``SpiderMoELayer`` / ``SpiderWebLM`` with this package's seeded
synthetic parameters (``spider_web_moe_b200.synth``), runs the reference forward
and records what the reference computed:

* ``top_indices``, ``top_weights``, ``messages`` and the returned ``delta`` are
  the arguments / result of the reference's own ``sparse_expert_delta`` call
  (spider_moe/model.py:310), captured by wrapping that function;
* ``edge_logits`` is the output of the reference's ``edge_generator`` module
  (model.py:263), captured by a forward hook; the fixture also stores
  ``edge_indices`` / ``edge_weights`` obtained from those logits with the
  reference's own expressions (model.py:265-266);
* ``h_out`` is the block output; ``plan_*`` is the reference's
  ``build_dispatch_plan`` (forge/ep/dispatch.py:56) on the captured routing;
* int4 / fp8 fixtures are outputs of the reference's ``quantize_int4`` and
  ``quantize_fp8_with_scale_tensor`` (spider_moe/quant.py:89,146).

The fixtures are read by tests/test_oracle_golden.py (CPU) and by the GPU
parity tests; nothing reads the reference at test time.
"""
from __future__ import annotations

import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def param_digest(module) -> str:
    h = hashlib.sha256()
    for name, p in module.named_parameters():
        h.update(name.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def tensor_digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (float32 view for floating tensors)."""
    t = t.detach().contiguous()
    if t.is_floating_point():
        t = t.float()
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


class Capture:
    """Wraps the reference's sparse_expert_delta / edge_generator to record one forward."""

    def __init__(self, model_mod, layer):
        self.model_mod = model_mod
        self.layer = layer
        self.records = []
        self._orig = model_mod.sparse_expert_delta
        self._cur = {}

    def __enter__(self):
        def wrapped(messages, top_indices, top_weights, *a, **kw):
            out = self._orig(messages, top_indices, top_weights, *a, **kw)
            self._cur.update(messages=messages.detach().clone(),
                             top_indices=top_indices.detach().clone(),
                             top_weights=top_weights.detach().clone(),
                             delta=out.detach().clone())
            return out

        def hook(mod, inp, out):
            self._cur["edge_logits"] = out.detach().clone()

        def pre(mod, args):
            self._cur = {"h_in": args[0].detach().clone(), "x0": args[1].detach().clone(),
                         "loop_idx": int(args[2])}

        def post(mod, args, out):
            o = out[0] if isinstance(out, tuple) else out
            self._cur["h_out"] = o.detach().clone()
            self.records.append(self._cur)

        self.model_mod.sparse_expert_delta = wrapped
        self._hooks = [self.layer.edge_generator.register_forward_hook(hook),
                       self.layer.register_forward_pre_hook(pre),
                       self.layer.register_forward_hook(post)]
        return self

    def __exit__(self, *exc):
        self.model_mod.sparse_expert_delta = self._orig
        for hk in self._hooks:
            hk.remove()


def finish_record(rec, layer, build_dispatch_plan, store_logits):
    """Add edge indices/weights (model.py:264-266) and the reference dispatch plan."""
    e, m = layer.num_experts, layer.edges_per_expert
    logits = rec["edge_logits"]
    b, t = logits.shape[:2]
    lg = logits.view(b, t, e, e)
    vals, idx = lg.topk(m, dim=-1)
    rec["edge_indices"] = idx
    rec["edge_weights"] = vals.float().softmax(dim=-1)
    srt = lg.float().sort(dim=-1, descending=True).values
    rec["edge_margin"] = (srt[..., : m] - srt[..., 1 : m + 1]).min(dim=-1).values if m < e else \
        torch.full(lg.shape[:-1], float("inf"))
    if not store_logits:
        del rec["edge_logits"]
    plan = build_dispatch_plan(rec["top_indices"], rec["top_weights"], num_experts=e, local_only=False)
    offsets = [0]
    toks, ws = [], []
    counts = {a.expert_id: a for a in plan.assignments}
    for eid in range(e):
        a = counts.get(eid)
        if a is None:
            offsets.append(offsets[-1])
            continue
        toks.append(a.token_index)
        ws.append(a.weights)
        offsets.append(offsets[-1] + a.token_index.numel())
    rec["plan_offsets"] = torch.tensor(offsets, dtype=torch.int64)
    rec["plan_tokens"] = torch.cat(toks) if toks else torch.zeros(0, dtype=torch.int64)
    rec["plan_weights"] = torch.cat(ws) if ws else torch.zeros(0)
    return rec


def layer_case(name, ref, synth, cfg_kw, tokens, *, bf16=False, zipf=None, int4_group=None,
               fp8=False, seed=0, input_seed=1, store_weights=False):
    from spider_moe.config import ModelConfig
    import spider_moe.model as model_mod
    from spider_infer.forge.ep.dispatch import build_dispatch_plan

    cfg = ModelConfig(**dict(dict(vocab_size=512, num_heads=4), **cfg_kw)).validate()
    cfg.expert_parallel = False
    layer = model_mod.SpiderMoELayer(cfg).eval()
    synth.init_block_params_(layer, seed=seed, zipf=zipf)
    if bf16:
        synth.round_params_to_bf16_(layer)
    fp8_data = None
    if fp8:
        from spider_moe.quant import quantize_fp8_with_scale_tensor, dequantize_fp8_with_scale_tensor
        fp8_data = {}
        with torch.no_grad():
            for i, ex in enumerate(layer.experts):
                for j in (0, 2):
                    w = ex[j].weight
                    s = (w.detach().float().abs().amax(dim=1, keepdim=True) / 448.0).clamp_min(1e-12)
                    q = quantize_fp8_with_scale_tensor(w, s)
                    ex[j].weight.copy_(dequantize_fp8_with_scale_tensor(q, s, torch.float32))
                    fp8_data[f"experts.{i}.{j}.q"] = q.view(torch.uint8).clone()
                    fp8_data[f"experts.{i}.{j}.s"] = s.view(-1).clone()
    digest_before_quant = param_digest(layer)
    int4_data = None
    if int4_group:
        layer.quantize_experts(group_size=int4_group)
        for q in (layer._int4_w_up, layer._int4_w_down):
            q.scales = q.scales.bfloat16().float()
        int4_data = dict(up_packed=layer._int4_w_up.packed.clone(), up_scales=layer._int4_w_up.scales.clone(),
                         down_packed=layer._int4_w_down.packed.clone(),
                         down_scales=layer._int4_w_down.scales.clone())
    h, x0 = synth.block_inputs(tokens, cfg.hidden_size, seed=input_seed)
    if bf16:
        h = h.to(torch.bfloat16).float()
        x0 = h.clone()
    records = []
    with torch.no_grad(), Capture(model_mod, layer) as cap:
        hh = h
        for l in range(cfg.num_loops):
            hh = layer(hh, x0, l)
        records = cap.records
    records = [finish_record(r, layer, build_dispatch_plan, store_logits=False) for r in records]
    out = dict(name=name, cfg=cfg_kw, tokens=tokens, bf16=bf16, zipf=zipf, int4_group=int4_group,
               fp8=fp8, seed=seed, input_seed=input_seed, param_digest=digest_before_quant,
               records=records)
    if int4_data is not None:
        # Full packed tensors are large: keep their digests and expert 0 verbatim.
        out["int4"] = {k: v[:1].clone() for k, v in int4_data.items()}
        out["int4_digest"] = {k: tensor_digest(v) for k, v in int4_data.items()}
    if fp8_data is not None:
        keep = [k for k in fp8_data if k.startswith("experts.0.")]
        out["fp8"] = {k: fp8_data[k] for k in keep}
        out["fp8_digest"] = {k: tensor_digest(v) for k, v in fp8_data.items()}
    if store_weights:
        out["state_dict"] = {k: v.detach().clone() for k, v in layer.state_dict().items()}
    torch.save(out, os.path.join(HERE, f"{name}.pt"))
    print(name, "loops", len(records), "digest", digest_before_quant[:12])


def cfg1_full_model(synth):
    """README smoke SpiderWebLM, fp32, full forward on 2x32 ids."""
    from spider_moe.config import ModelConfig
    import spider_moe.model as model_mod
    from spider_infer.forge.ep.dispatch import build_dispatch_plan

    cfg = ModelConfig(vocab_size=512, hidden_size=64, num_heads=4, num_experts=4, top_k=2,
                      edges_per_expert=2, num_loops=2, expert_ffn_size=128).validate()
    cfg.expert_parallel = False
    torch.manual_seed(0)
    model = model_mod.SpiderWebLM(cfg).eval()
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name == "recurrent.loop_bias":
                p.zero_()
            else:
                p.copy_(torch.empty(p.shape).normal_(0.0, 0.02, generator=g))
        for mod in model.modules():
            if isinstance(mod, torch.nn.LayerNorm):
                mod.weight.fill_(1.0)
                mod.bias.fill_(0.0)
    ids = torch.randint(0, 512, (2, 32), generator=torch.Generator().manual_seed(0))
    with torch.no_grad(), Capture(model_mod, model.recurrent) as cap:
        logits = model(ids)["logits"]
        records = cap.records
    records = [finish_record(r, model.recurrent, build_dispatch_plan, store_logits=True)
               for r in records]
    out = dict(name="cfg1_model", cfg=dict(vocab_size=512, hidden_size=64, num_heads=4,
                                           num_experts=4, top_k=2, edges_per_expert=2,
                                           num_loops=2, expert_ffn_size=128),
               tokens=64, ids=ids, logits=logits,
               state_dict={k: v.detach().clone() for k, v in model.recurrent.state_dict().items()},
               records=records)
    torch.save(out, os.path.join(HERE, "cfg1_model.pt"))
    print("cfg1_model loops", len(records))


def stats_case(synth):
    """SpiderMoELayer.forward(..., return_stats=True) (model.py:324-349) of the
    reference on seeded parameters: each loop's input, output and stats dict."""
    from spider_moe.config import ModelConfig
    import spider_moe.model as model_mod

    kw = dict(num_heads=4, loop_embed_size=32, hidden_size=64, num_experts=8, top_k=2, edges_per_expert=3,
              num_loops=3, expert_ffn_size=96)
    cfg = ModelConfig(**dict(dict(vocab_size=512), **kw)).validate()
    cfg.expert_parallel = False
    layer = model_mod.SpiderMoELayer(cfg).eval()
    synth.init_block_params_(layer, seed=7)
    with torch.no_grad():
        layer.exit_head.weight.normal_(0.0, 0.3, generator=torch.Generator().manual_seed(8))
        layer.exit_head.bias.fill_(0.25)
    h, x0 = synth.block_inputs(24, cfg.hidden_size, seed=9)
    records = []
    with torch.no_grad():
        hh = h
        for l in range(cfg.num_loops):
            out, st = layer(hh, x0, l, return_stats=True)
            records.append(dict(loop_idx=l, h_in=hh.clone(), h_out=out.clone(),
                                stats={k: v.detach().clone() for k, v in st.items()}))
            hh = out
    res = dict(name="e8_stats", cfg=kw, tokens=24, seed=7, zipf=None, bf16=False,
               exit_head={k: v.detach().clone() for k, v in layer.exit_head.state_dict().items()},
               x0=x0, records=records)
    torch.save(res, os.path.join(HERE, "e8_stats.pt"))
    print("e8_stats loops", len(records))


def early_exit_case(synth):
    """SpiderWebLM._run_recurrent_decode(h, x0, early_exit=True) (model.py:450-473)
    of the reference on seeded recurrent-block parameters: the returned h and
    the active batch rows each loop ran on."""
    from spider_moe.config import ModelConfig
    import spider_moe.model as model_mod

    kw = dict(num_heads=4, loop_embed_size=32, hidden_size=64, num_experts=8, top_k=2, edges_per_expert=2,
              num_loops=5, expert_ffn_size=96)
    cfg = ModelConfig(**dict(dict(vocab_size=512), **kw)).validate()
    cfg.expert_parallel = False
    model = model_mod.SpiderWebLM(cfg).eval()
    layer = model.recurrent
    # weights of std 0.3 make each loop move h, so rows leave at different loops
    synth.init_block_params_(layer, seed=11, std=0.3)
    with torch.no_grad():
        layer.exit_head.weight.normal_(0.0, 0.05, generator=torch.Generator().manual_seed(12))
        layer.exit_head.bias.fill_(1.7)
    h, _ = synth.block_inputs(32, cfg.hidden_size, seed=13)
    h = h.view(32, 1, cfg.hidden_size)
    x0 = h.clone()
    active_rows = []
    hook = layer.register_forward_pre_hook(lambda mod, args: active_rows.append(args[0].shape[0]))
    with torch.no_grad():
        out = model._run_recurrent_decode(h.clone(), x0, True)
    hook.remove()
    res = dict(name="e8_early_exit", cfg=kw, seed=11, std=0.3, zipf=None, bf16=False,
               threshold=float(cfg.early_exit_threshold),
               exit_head={k: v.detach().clone() for k, v in layer.exit_head.state_dict().items()},
               h=h, x0=x0, out=out.clone(), active_rows=active_rows)
    torch.save(res, os.path.join(HERE, "e8_early_exit.pt"))
    print("e8_early_exit active rows per loop", active_rows)


def lumen_case(synth):
    """The reference's LumenWorkspace on its own (return_state, J-lens) and a
    SpiderMoELayer with use_lumen over two loops with return_stats
    (lumen.py:81-123, model.py:318-348)."""
    from spider_moe.config import ModelConfig
    from spider_moe.lumen import LumenWorkspace
    import spider_moe.model as model_mod

    torch.manual_seed(3)
    ws = LumenWorkspace(hidden_size=64, num_slots=4, slot_dim=16, vocab_size=50).eval()
    with torch.no_grad():
        ws.slot_bias.normal_(0.0, 0.5)
    h = torch.randn(2, 5, 64, generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        out, st = ws(h, return_state=True, j_lens=True)
    module = dict(state_dict={k: v.clone() for k, v in ws.state_dict().items()}, h=h, out=out,
                  slots=st.slots, slot_weights=st.slot_weights, broadcast=st.broadcast, j_logits=st.j_logits,
                  j_space=ws.read_j_space(st, top_k=3))
    kw = dict(num_heads=4, loop_embed_size=32, hidden_size=64, num_experts=4, top_k=2, edges_per_expert=2,
              num_loops=2, expert_ffn_size=96, use_lumen=True, lumen_slots=4)
    cfg = ModelConfig(**dict(dict(vocab_size=512), **kw)).validate()
    cfg.expert_parallel = False
    layer = model_mod.SpiderMoELayer(cfg).eval()
    synth.init_block_params_(layer, seed=5, std=0.1)
    hb, x0 = synth.block_inputs(24, 64, seed=6)
    records = []
    with torch.no_grad():
        hh = hb
        for l in range(cfg.num_loops):
            o, stats = layer(hh, x0, l, return_stats=True)
            records.append(dict(loop_idx=l, h_in=hh.clone(), h_out=o.clone(),
                                stats={k: v.detach().clone() for k, v in stats.items()}))
            hh = o
    res = dict(name="lumen", module=module, cfg=kw, seed=5, std=0.1, zipf=None, bf16=False, x0=x0,
               records=records)
    torch.save(res, os.path.join(HERE, "lumen.pt"))
    print("lumen loops", len(records), "stats keys", sorted(records[0]["stats"]))


def spiderw_case(synth, ref_root):
    """.spiderw bundles (docs/NATIVE_WEIGHT_FORMAT.md): a block exported by the
    reference's own exporter (scripts/export_native_weights.py) from seeded
    parameters, what the reference's loader (spider_infer/orbit/weight_loader.py)
    reads back from it, and a bundle of mixed section kinds written by the
    reference's writer."""
    import importlib.util
    import numpy as np
    from spider_moe.config import ModelConfig
    from spider_infer.orbit.weight_loader import SpiderWMeta, load_spiderw, write_spiderw

    spec = importlib.util.spec_from_file_location(
        "export_native_weights", os.path.join(ref_root, "scripts", "export_native_weights.py"))
    exporter = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(exporter)
    kw = dict(vocab_size=64, num_heads=4, loop_embed_size=32, hidden_size=32, num_experts=4, top_k=2,
              edges_per_expert=2, num_loops=2, expert_ffn_size=64)
    cfg = ModelConfig(**kw).validate()
    sd = synth.synthetic_state_dict(cfg, seed=21, std=0.1)
    state = {"recurrent." + k: v for k, v in sd.items()}
    state["token_embedding.weight"] = torch.randn(64, 32, generator=torch.Generator().manual_seed(22))
    block_path = os.path.join(HERE, "e4_block.spiderw")
    exporter.export_from_state_dict(state, cfg, block_path)
    ref = load_spiderw(block_path)
    mixed = {"router": np.arange(12, dtype=np.float32).reshape(3, 4), "loop_bias": np.ones((2, 3), np.float16),
             "csr_row_ptr": np.array([0, 2, 4], np.int32), "prelude.0.W_qkv": np.full((2, 5), 0.5, np.float32),
             "extra_f64": np.linspace(0, 1, 7)}
    meta = SpiderWMeta(version=1, flags=2, vocab_size=10, hidden_size=4, num_heads=2, num_experts=3, top_k=2,
                       edges_per_expert=1, num_loops=2, expert_ffn_size=8, num_prelude_layers=1,
                       num_coda_layers=0)
    mixed_path = os.path.join(HERE, "mixed_sections.spiderw")
    write_spiderw(mixed_path, meta, mixed)
    ref_mixed = load_spiderw(mixed_path)
    res = dict(cfg=kw, seed=21, std=0.1, block_meta=vars(ref.meta), block_sections={k: torch.from_numpy(v.copy())
                                                                                     for k, v in ref.tensors.items()},
               mixed_meta=vars(meta), mixed_in={k: torch.from_numpy(np.asarray(v).copy()) for k, v in mixed.items()},
               mixed_sections={k: torch.from_numpy(v.copy()) for k, v in ref_mixed.tensors.items()},
               mixed_csr=sorted(ref_mixed.csr) if ref_mixed.csr else None)
    torch.save(res, os.path.join(HERE, "spiderw.pt"))
    print("spiderw sections", sorted(ref.tensors), "mixed", sorted(ref_mixed.tensors))


def dobu_case(synth):
    """The reference's Dobu store (expert_store.py:40-205): a sequence of
    sparse_delta calls with its LRU statistics after each, and a layer with
    offload_experts over two loops (model.py:185-199, 294-297)."""
    from torch import nn
    from spider_moe.config import ModelConfig
    from spider_moe.expert_store import ExpertChunkStore
    import spider_moe.model as model_mod

    torch.manual_seed(7)
    experts = nn.ModuleList([nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16)) for _ in range(6)])
    store = ExpertChunkStore(experts, storage_device="cpu", compute_device="cpu", max_gpu_experts=2)
    g = torch.Generator().manual_seed(8)
    routes = [[[0, 1], [1, 2], [0, 2], [1, 0], [2, 1]],       # experts 0,1,2: misses, 2 evicts 0
              [[3, 4], [4, 3], [3, 3], [4, 5], [3, 4]],       # 3,4,5
              [[5, 4], [5, 5], [4, 5], [4, 4], [5, 4]],       # hits on 4,5
              [[0, 5], [1, 5], [0, 1], [5, 0], [1, 1]]]       # 0,1 misses, 5 hit
    calls = []
    for r in routes:
        msgs = torch.randn(1, 5, 16, generator=g)
        idx = torch.tensor([r])
        w = torch.rand(1, 5, 2, generator=g)
        w[0, 2, 1] = -0.5                                        # a non-positive slot weight
        d = store.sparse_delta(msgs, idx, w, top_k=2)
        st = store.stats()
        calls.append(dict(msgs=msgs, idx=idx, w=w, delta=d, hits=st["hits"], misses=st["misses"],
                          loads=st["loads"], hot=st["gpu_hot_experts"], storage_bytes=st["storage_bytes"],
                          gpu_bytes=st["gpu_working_set_bytes"]))
    kw = dict(num_heads=4, loop_embed_size=32, hidden_size=64, num_experts=8, top_k=2, edges_per_expert=2,
              num_loops=2, expert_ffn_size=96, offload_experts=True, offload_max_gpu_experts=3)
    cfg = ModelConfig(**dict(dict(vocab_size=512), **kw)).validate()
    cfg.expert_parallel = False
    layer = model_mod.SpiderMoELayer(cfg).eval()
    synth.init_block_params_(layer, seed=9, std=0.1)
    # the store copied the experts at construction: rebuild it from the seeded weights
    layer._expert_store = ExpertChunkStore(layer.experts, storage_device="cpu", compute_device="cpu",
                                           max_gpu_experts=3)
    h, x0 = synth.block_inputs(16, 64, seed=10)
    outs = []
    with torch.no_grad():
        hh = h
        for l in range(cfg.num_loops):
            hh = layer(hh, x0, l)
            outs.append(hh.clone())
    st = layer._expert_store.stats()
    res = dict(name="dobu", experts={k: v.clone() for k, v in experts.state_dict().items()}, calls=calls,
               cfg=kw, seed=9, std=0.1, zipf=None, bf16=False, h=h, x0=x0, outs=outs,
               layer_stats={k: st[k] for k in ("hits", "misses", "loads", "gpu_hot_experts")})
    torch.save(res, os.path.join(HERE, "dobu.pt"))
    print("dobu calls", [(c["hits"], c["misses"], c["loads"], c["hot"]) for c in calls], res["layer_stats"])


def fp8_helper_vectors():
    """The reference's general fp8 helpers (spider_moe/quant.py:16-69, 146-169)
    on seeded tensors: per-tensor quantize with a computed, a float and a tensor
    scale, dequantize in the default and an explicit dtype, and the
    broadcastable-scale pair."""
    from spider_moe import quant as RQ

    g = torch.Generator().manual_seed(6)
    x = torch.randn(5, 24, generator=g) * 3.0
    q, s = RQ.quantize_fp8(x)
    q2, s2 = RQ.quantize_fp8(x, 0.05)
    q3, s3 = RQ.quantize_fp8(x, torch.tensor([0.02]))
    rows = torch.rand(5, generator=g) * 0.1 + 1e-3
    q4 = RQ.quantize_fp8_with_scale_tensor(x, rows)
    res = dict(x=x, rows=rows, q=q.view(torch.uint8), s=s, q2=q2.view(torch.uint8), s2=s2, q3=q3.view(torch.uint8),
               s3=s3, deq=RQ.dequantize_fp8(q, s), deq_bf16=RQ.dequantize_fp8(q, s, torch.bfloat16),
               deq_plain=RQ.dequantize_fp8(q), q4=q4.view(torch.uint8),
               deq4=RQ.dequantize_fp8_with_scale_tensor(q4, rows), scale=RQ.compute_fp8_scale(x))
    torch.save(res, os.path.join(HERE, "fp8_helpers.pt"))
    print("fp8 helper vectors")


def quant_vectors():
    from spider_moe.quant import quantize_int4, quantize_fp8_with_scale_tensor, dequantize_int4
    g = torch.Generator().manual_seed(5)
    w = torch.randn(6, 256, generator=g) * 0.05
    res = {"w": w}
    for gs in (64, 128):
        q = quantize_int4(w, group_size=gs)
        res[f"int4_g{gs}_packed"] = q.packed
        res[f"int4_g{gs}_scales"] = q.scales
        res[f"int4_g{gs}_deq"] = dequantize_int4(q.packed, q.scales, q.shape, q.group_size,
                                                 dtype=torch.float32)
    wf = torch.randn(16, 64, generator=g) * 0.03
    s = (wf.abs().amax(dim=1, keepdim=True) / 448.0).clamp_min(1e-12)
    res["fp8_w"] = wf
    res["fp8_scale"] = s.view(-1)
    res["fp8_q_u8"] = quantize_fp8_with_scale_tensor(wf, s).view(torch.uint8)
    torch.save(res, os.path.join(HERE, "quant_vectors.pt"))
    print("quant vectors")


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPIDER_REFERENCE", "")
    if ref_root:
        sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    from spider_web_moe_b200 import synth

    torch.set_num_threads(8)
    cfg1_full_model(synth)
    base = dict(num_heads=4, loop_embed_size=32)
    layer_case("e4_fp32", None, synth, dict(base, hidden_size=64, num_experts=4, top_k=2,
               edges_per_expert=2, num_loops=2, expert_ffn_size=128), 64, store_weights=True)
    layer_case("e16_fp32", None, synth, dict(base, hidden_size=64, num_experts=16, top_k=2,
               edges_per_expert=2, num_loops=3, expert_ffn_size=128), 48)
    layer_case("e16_zipf_bf16", None, synth, dict(base, hidden_size=128, num_experts=16, top_k=2,
               edges_per_expert=2, num_loops=2, expert_ffn_size=256), 40, bf16=True, zipf=1.1)
    layer_case("e64_fp8", None, synth, dict(base, hidden_size=128, num_experts=64, top_k=4,
               edges_per_expert=3, num_loops=2, expert_ffn_size=128), 24, bf16=True, fp8=True)
    layer_case("e128_int4", None, synth, dict(base, hidden_size=128, num_experts=128, top_k=8,
               edges_per_expert=4, num_loops=2, expert_ffn_size=256), 12, bf16=True, zipf=1.1,
               int4_group=128)
    quant_vectors()
    stats_case(synth)
    early_exit_case(synth)
    lumen_case(synth)
    spiderw_case(synth, ref_root)
    dobu_case(synth)
    fp8_helper_vectors()


if __name__ == "__main__":
    main()
