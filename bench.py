"""Benchmark: recurrent Spider-MoE block tokens/s on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3] [--impl b200|reference]

A step is one forward of the block -- all ``num_loops`` loops -- over one batch
of synthetic tokens of the named config.  The default is cfg3, the largest
single-GPU configuration: bf16 prefill, 8192 tokens (8 x 1024), H 1024, 16
experts with a Zipf(1.1) router bias, top-2, 2 edges, 6 loops, SwiGLU FFN
2048.  Weights N(0,0.02) (seeded), inputs N(0,1), no network data.

Arms:
* ``--impl b200`` (default): the CUDA path.  ``value`` = tokens/s of CUDA-graph
  replays with inputs resident in HBM (device-timed with CUDA events, max over
  ranks); ``e2e`` = the same through the public API with the step's input
  copied from pinned host memory and the output copied back inside the timed
  region; ``roofline`` = the grouped-GEMM launches' algorithmic bytes over
  their event-timed duration (a separate pass with per-stage events); and
  ``cpu_baseline`` = the reference algorithm on the host cores (rank 0).
* ``--impl reference``: the reference block's CPU algorithm (the oracle
  restatement, dense as the reference computes it) on all host threads, rank 0.

With N > 1 (torchrun) every rank holds its own batch of the config's token
count (weak scaling).  The block is token-independent, so by default
(``--parallel dp``) every rank runs it on its own tokens with the weights
replicated and no collective on the data path.  ``--parallel ep`` runs the
token-sharded expert-parallel block instead (spider_web_moe_b200.ep: experts
e % N, message rows to the expert owners and back every loop, over peer memory
or NCCL all-to-all).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, one ncu capture) of
# the edge-value, expert-up and expert-down GEMM launches of one step, keyed by
# "config:activation"; a workload without a capture reports traffic null.
#   cfg2:gelu    -- the 18 launches of one cfg2 replay with GELU experts (profiles/gemm_tcgen05_cfg2.txt)
#   cfg2:swiglu  -- the 18 launches of one cfg2 replay (profiles/cfg2_launch_list.txt)
#   cfg3:swiglu  -- the 18 launches of one cfg3 replay (profiles/cfg3_launch_list.txt)
#   cfg4:swiglu  -- the 18 launches of one cfg4 step (profiles/cfg4_launch_list.txt)
#   cfg5:swiglu  -- the 12 launches of one cfg5 replay (profiles/gemm_qdec_cfg5.txt)
NCU_TRAFFIC_PER_STEP = {"cfg2:gelu": 1013465344, "cfg2:swiglu": 1417670144, "cfg3:swiglu": 3237011456,
                        "cfg4:swiglu": 12730709760, "cfg5:swiglu": 5183200000}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="cfg3")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--engine", default="auto", choices=["auto", "tcgen05", "simt"])
    ap.add_argument("--activation", default=None, choices=["gelu", "swiglu"],
                    help="expert FFN; default: the one the workload names (SwiGLU for cfg2-cfg5)")
    ap.add_argument("--parallel", default="dp", choices=["dp", "ep"],
                    help="N > 1: dp = every rank runs the whole block on its own tokens (weights replicated, no "
                         "collective on the data path); ep = token-sharded expert parallelism (experts e % N, "
                         "message rows exchanged with the expert owners every loop)")
    ap.add_argument("--micro-batches", type=int, default=1, choices=[1, 2],
                    help="N > 1 expert parallelism: tokens per rank as one batch (1), or as two halves on two "
                         "streams, one half's exchange overlapping the other's GEMMs (2)")
    ap.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                    help="N > 1 expert-parallel exchange: stores into the peers' memory over NVLink (peer) or NCCL "
                         "all-to-all")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-only", action="store_true",
                    help="capture the graph, replay warmup+steps times, print nothing else (for ncu)")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime

        backend = "nccl" if args.impl == "b200" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world <= 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML while running."""

    def __init__(self, index: int, period_s: float = 0.01):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.index]) if vis else self.index
            self.h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.nv = nv
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return self
        bits = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
                0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                    r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    for b, name in bits.items():
                        if r & b:
                            self.reasons.add(name)
                except Exception:
                    pass
                time.sleep(self.period)

        self._thr = threading.Thread(target=run, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr:
            self._thr.join(timeout=1)

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------- workload
def workload(args):
    from spider_web_moe_b200.config import ModelConfig, benchmark_configs

    spec = benchmark_configs()[args.config]
    model = dict(spec["model"])
    model["expert_activation"] = args.activation or spec["activation"]
    cfg = ModelConfig(**model).validate()
    return cfg, spec


def workload_config(args, cfg, spec, world: int) -> dict:
    """The ``config`` object of the JSON line.  Both arms print this same dict
    for the same arguments: it names the workload, not the implementation (the
    reference arm's bounded sample is described in its ``cpu_baseline``)."""
    if world <= 1:
        par = "single GPU"
    elif args.parallel == "dp":
        par = f"dp{world}: tokens sharded by rank, block weights replicated, no collective on the data path"
    else:
        mb = args.micro_batches
        par = (f"ep{world}: tokens sharded by rank, experts e % {world}, "
               + ("dispatch/combine stored into peer memory over NVLink" if args.transport == "peer"
                  else "NCCL all-to-all")
               + (", two micro-batches on two streams (exchange overlaps the other half's GEMMs)" if mb == 2
                  else ""))
    return {"workload": args.config, "tokens_per_step_per_gpu": spec["tokens"], "num_loops": cfg.num_loops,
            "hidden": cfg.hidden_size, "experts": cfg.num_experts, "top_k": cfg.top_k,
            "edges_per_expert": cfg.edges_per_expert, "ffn": cfg.expert_ffn_size,
            "expert_activation": cfg.expert_activation, "expert_weights": spec["wfmt"],
            "router_bias": "zipf(1.1)" if spec["zipf"] else "none", "parallelism": par,
            "l2": "not flushed: every step re-reads the block's weights, a working set larger than the 126 MB L2"}


def algorithmic_bytes(cfg, spec, taps, n):
    """Bytes the grouped-GEMM launches of one loop must move (weights of touched
    groups in their stored format + rows in/out), from the loop's routing."""
    H, U, E = cfg.hidden_size, cfg.expert_ffn_size, cfg.num_experts
    # "native" weights take the activation dtype, which the benchmark runs in bf16
    wfmt = "bf16" if spec["wfmt"] == "native" else spec["wfmt"]
    wb = {"bf16": 2.0, "fp8": 1.0, "int4": 0.5}[wfmt]
    top = taps["top_idx"].long().cpu()
    experts = int(torch.unique(top).numel())
    pairs = int(taps["ffn_offsets"][-1].item())
    eidx = taps["edge_idx"].long().cpu().reshape(n, -1)
    dsts = int(torch.unique(eidx).numel())
    dst_pairs = sum(int(torch.unique(eidx[i]).numel()) for i in range(n))
    gates = 2 if cfg.expert_activation == "swiglu" else 1

    def wbytes(rows, cols):  # one expert matrix in its stored format, scales included
        sc = {"bf16": 0.0, "fp8": rows * 4.0, "int4": rows * (cols / cfg.moe_int4_group_size) * 2.0}[wfmt]
        return rows * cols * wb + sc

    up = experts * gates * (wbytes(U, H) + U * 4) + pairs * H * 2 + pairs * U * 2
    down = experts * (wbytes(H, U) + H * 4) + pairs * U * 2 + pairs * H * 4
    edge = dsts * H * H * 2 + dst_pairs * H * 2 + dst_pairs * H * 4
    return {"gemm_expert_up": up, "gemm_expert_down": down, "gemm_edge_values": edge}


def algorithmic_flops(cfg, taps, n):
    """Multiply-add FLOPs (2 per MAC) of the grouped-GEMM launches of one loop,
    from the loop's routing: edge values per (token, destination) pair, expert
    up (and gate) and down per (token, expert) pair."""
    H, U = cfg.hidden_size, cfg.expert_ffn_size
    pairs = int(taps["ffn_offsets"][-1].item())
    eidx = taps["edge_idx"].long().cpu().reshape(n, -1)
    dst_pairs = sum(int(torch.unique(eidx[i]).numel()) for i in range(n))
    gates = 2 if cfg.expert_activation == "swiglu" else 1
    return {"gemm_edge_values": 2.0 * dst_pairs * H * H, "gemm_expert_up": 2.0 * pairs * H * U * gates,
            "gemm_expert_down": 2.0 * pairs * U * H}


def gemm_roofline(gemm_bytes, gemm_flops, gemm_ms, launches, peaks, peak_kind, traffic):
    """Roofline of the grouped-GEMM family: HBM-bound (GB/s against the measured
    copy peak) when its arithmetic intensity is below the ridge point of the
    measured peaks, tensor-bound (TFLOP/s against the measured bf16 GEMM peak)
    above it."""
    sec = gemm_ms / 1e3
    gbs = gemm_bytes / sec / 1e9
    tflops = gemm_flops / sec / 1e12
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    tensor = gemm_flops / max(gemm_bytes, 1.0) > ridge
    r = {"bound": "tensor" if tensor else "hbm",
         "achieved": tflops if tensor else gbs,
         "peak": peaks["bf16_tflops"] if tensor else peaks["hbm_gbs"],
         "unit": "TFLOP/s" if tensor else "GB/s",
         "peak_kind": f"{peak_kind} ({'cuBLAS bf16 GEMM, burst' if tensor else 'STREAM copy'})",
         "traffic": (traffic / launches if traffic else None),
         "kernel": "tc_gemm_kernel (grouped GEMM, tcgen05) edge-value + expert up/down launches",
         "algorithmic_bytes_per_launch": gemm_bytes / launches, "algorithmic_flops_per_launch": gemm_flops / launches,
         "arithmetic_intensity": gemm_flops / max(gemm_bytes, 1.0), "ridge": ridge,
         "achieved_gbs": gbs, "achieved_tflops": tflops, "launch_ms": gemm_ms / launches}
    r["frac"] = r["achieved"] / r["peak"]
    return r


def build_engine(cfg, spec, args, device, n):
    from spider_web_moe_b200 import synth
    from spider_web_moe_b200.engine import BlockEngine

    zipf = 1.1 if spec["zipf"] else None
    sd = synth.synthetic_state_dict(cfg, seed=0, device=device, zipf=zipf, round_bf16=True)
    if spec["wfmt"] == "int4":
        cfg.moe_int4_group_size = cfg.moe_int4_group_size or 128
    eng = BlockEngine(cfg, sd, device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"],
                      engine=args.engine)
    del sd
    return eng


def stage_timing(eng, h, steps):
    """Per-stage device time (ms per step) from events recorded around each launch."""
    import ctypes as C

    lib = eng.lib
    ns = lib.sb_num_stages()
    lib.sb_stage_timing(1)
    for _ in range(steps):
        # Keep the GPU busy while the host enqueues the step, so every event
        # pair brackets device execution, not host launch latency.
        torch.cuda._sleep(4_000_000)
        eng.forward(h, h)
    torch.cuda.synchronize()
    ms = (C.c_double * ns)()
    cnt = (C.c_int * ns)()
    lib.sb_stage_timing_read(ms, cnt, ns)
    lib.sb_stage_timing(0)
    return {lib.sb_stage_name(i).decode(): {"ms_per_step": ms[i] / steps, "launches_per_step": cnt[i] / steps}
            for i in range(ns)}


PORT_NOTE = ("the reference block's algorithm restated in fp32 PyTorch (oracle/spider_oracle.py: the dense "
             "edge transform of all E destinations as spider_moe/model.py:271-288 computes it); the restatement "
             "packs the expert and edge weights once, where the reference module re-stacks them on every loop "
             "(model.py:271,305-308), so it runs faster than the module itself")


def port_params(cfg, spec):
    """Oracle parameters of the workload (bf16-valued fp32 weights, seeded as the GPU arm)."""
    from oracle import spider_oracle as O
    from spider_web_moe_b200 import synth

    zipf = 1.1 if spec["zipf"] else None
    sd = synth.synthetic_state_dict(cfg, seed=0, device="cpu", zipf=zipf, round_bf16=True)
    return O.params_from_state_dict(sd, cfg.num_experts)


def port_seconds_per_token(p, cfg) -> float:
    """Calibration: one token through all loops (after one untimed call)."""
    from oracle import spider_oracle as O
    from spider_web_moe_b200 import synth

    h, _ = synth.block_inputs(1, cfg.hidden_size, seed=1)
    O.run_loops(p, h.view(1, -1), h.view(1, -1), cfg, dense=True)
    t0 = time.perf_counter()
    O.run_loops(p, h.view(1, -1), h.view(1, -1), cfg, dense=True)
    return time.perf_counter() - t0


def cpu_baseline(cfg, spec, seconds, threads=None):
    """The reference block's algorithm on the host cores (the oracle port, fp32,
    bf16-valued weights) on a bounded sample of the workload's tokens."""
    from oracle import spider_oracle as O
    from spider_web_moe_b200 import synth

    if threads:
        torch.set_num_threads(threads)
    p = port_params(cfg, spec)
    per_tok = port_seconds_per_token(p, cfg)
    chunk = int(max(1, min(spec["tokens"], seconds / 4 / max(per_tok, 1e-6))))
    h, _ = synth.block_inputs(chunk, cfg.hidden_size, seed=1)
    h = h.view(chunk, -1)
    done = 0
    t0 = time.perf_counter()
    while True:
        O.run_loops(p, h, h, cfg, dense=True)
        done += chunk
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{done} of the workload's tokens ({chunk}-token chunks; the block is token-independent) x "
                      f"{cfg.num_loops} loops of {spec_name(spec)} {cfg.expert_activation} in {dt:.1f} s; "
                      + PORT_NOTE}


def step_median(marks) -> float:
    """Median device time of one step from the events recorded between replays."""
    return statistics.median(marks[i].elapsed_time(marks[i + 1]) for i in range(len(marks) - 1))


def spec_name(spec):
    return f"H{spec['model']['hidden_size']} E{spec['model']['num_experts']} K{spec['model']['top_k']}"


# ---------------------------------------------------------------------------- arms
def run_reference(args):
    rank, world, local = dist_setup(args)
    cfg, spec = workload(args)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import spider_oracle as O
    from spider_web_moe_b200 import synth

    p = port_params(cfg, spec)
    per_tok = port_seconds_per_token(p, cfg)
    budget = 150.0  # seconds for the whole --steps/--warmup run
    chunk = int(max(1, min(spec["tokens"], budget / max(1, args.steps + args.warmup) / max(per_tok, 1e-6))))
    h, _ = synth.block_inputs(chunk, cfg.hidden_size, seed=1)
    h = h.view(chunk, -1)
    for _ in range(args.warmup):
        O.run_loops(p, h, h, cfg, dense=True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.run_loops(p, h, h, cfg, dense=True)
    dt = time.perf_counter() - t0
    value = chunk * args.steps / dt
    line = {
        "impl": "reference", "metric": "spider_moe_block_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, cfg, spec, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"each step: {chunk} of the workload's {spec['tokens']} tokens (the block is "
                                   f"token-independent) x {cfg.num_loops} loops; " + PORT_NOTE},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_b200_ep(args, rank, world, local, device):
    """N > 1: token-sharded expert parallelism, one batch per rank, experts e % N."""
    from spider_web_moe_b200 import synth
    from spider_web_moe_b200.ep import ExpertParallelBlock

    cfg, spec = workload(args)
    n = spec["tokens"]
    zipf = 1.1 if spec["zipf"] else None
    if spec["wfmt"] == "int4":
        cfg.moe_int4_group_size = cfg.moe_int4_group_size or 128
    sd = synth.synthetic_state_dict(cfg, seed=0, device=device, zipf=zipf, round_bf16=True)
    mb = args.micro_batches
    ep = ExpertParallelBlock(cfg, sd, device, act_dtype=torch.bfloat16, max_tokens=n, weight_format=spec["wfmt"],
                             engine=args.engine, transport=args.transport, micro_batches=mb)
    del sd
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=1 + rank, device=device, dtype=torch.bfloat16)
    h = h.view(n, -1).contiguous()
    stream = torch.cuda.current_stream(device)
    ep.capture(n)  # all loops, kernels and NCCL exchanges, in one CUDA graph
    ep.g_h.copy_(h)
    ep.g_x0.copy_(h)
    for _ in range(max(3, args.warmup)):
        ep.graph.replay()
    torch.cuda.synchronize(device)
    ep.check_status()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            marks[i].record(stream)
            ep.graph.replay()
        marks[-1].record(stream)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms_step = max_over_ranks(start.elapsed_time(end), world, device) / args.steps
    med_step = max_over_ranks(step_median(marks), world, device)
    # e2e through the public API: pinned host input in, output back, every step
    h_host = h.cpu().pin_memory()
    out_host = torch.empty(n, cfg.hidden_size, dtype=torch.bfloat16).pin_memory()
    barrier(world)
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(args.steps):
        ep.g_h.copy_(h_host, non_blocking=True)
        ep.g_x0.copy_(h_host, non_blocking=True)
        ep.graph.replay()
        out_host.copy_(ep.g_out, non_blocking=True)
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms = max_over_ranks(start.elapsed_time(end), world, device) / args.steps
    peaks, peak_kind = load_peaks()
    per_rank_bytes = (ep.dense.weight_bytes() + (ep.local.weight_bytes() if ep.local else 0)) * cfg.num_loops
    achieved = per_rank_bytes / (ms_step / 1e3) / 1e9
    line = {
        "metric": "spider_moe_block_tokens_per_s", "value": n * world / (ms_step / 1e3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden states)",
        "config": workload_config(args, cfg, spec, world), "engine": args.engine,
        "ms_per_step_median": med_step,
        "clocks": clk.summary(),
        "e2e": {"value": n * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 2 * n * cfg.hidden_size * 2,
                "d2h_bytes_per_step": n * cfg.hidden_size * 2, "ms_per_step": e2e_ms},
        "gpu_launches": ep.kernels_per_replay * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} (STREAM copy)",
                     "traffic": None, "kernel": "whole expert-parallel step per rank (dense + local expert weights)"},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, spec, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize(device)
    ep.close()  # the graph (NCCL work) and the peer regions go before the process group
    barrier(world)
    dist.destroy_process_group()


def run_b200(args):
    rank, world, local = dist_setup(args)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --impl b200 needs a CUDA device")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1 and args.parallel == "ep" and not args.profile_only:
        return run_b200_ep(args, rank, world, local, device)
    from spider_web_moe_b200 import synth
    from spider_web_moe_b200.engine import CapturedBlock, HostPipeline

    cfg, spec = workload(args)
    n = spec["tokens"]
    eng = build_engine(cfg, spec, args, device, n)
    h, _ = synth.block_inputs(n, cfg.hidden_size, seed=1 + rank, device=device, dtype=torch.bfloat16)
    h = h.view(n, -1).contiguous()

    # graph of all loops; inputs resident in HBM
    g = CapturedBlock(eng, n)
    g.h.copy_(h)
    g.x0.copy_(h)
    stream = torch.cuda.current_stream(device)
    for _ in range(max(3, args.warmup)):
        g.graph.replay()
    torch.cuda.synchronize(device)
    eng.check_status()
    if args.profile_only:
        for _ in range(args.steps):
            g.graph.replay()
        torch.cuda.synchronize(device)
        eng.check_status()
        if world > 1:
            dist.destroy_process_group()
        return

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            marks[i].record(stream)
            g.graph.replay()
        marks[-1].record(stream)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms = start.elapsed_time(end)
    ms = max_over_ranks(ms, world, device)
    ms_step = ms / args.steps
    med_step = max_over_ranks(step_median(marks), world, device)
    value = n * world / (ms_step / 1e3)
    gpu_launches = g.kernels_per_replay * args.steps  # libspider_b200 kernels counted at capture

    # e2e through the public API (HostPipeline): every step copies its input in
    # from pinned host memory and its output back; step s + 1's input and step
    # s - 1's output move while step s runs.  x0 = h, the block input.
    pipe = HostPipeline(eng, n, x0_is_h=True)
    h_hosts = [h.cpu().pin_memory() for _ in range(2)]
    out_hosts = [torch.empty(n, cfg.hidden_size, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    pipe.run([h_hosts[s & 1] for s in range(3)], [out_hosts[s & 1] for s in range(3)])
    torch.cuda.synchronize(device)
    barrier(world)
    start.record(stream)
    pipe.run([h_hosts[s & 1] for s in range(args.steps)], [out_hosts[s & 1] for s in range(args.steps)])
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms = max_over_ranks(start.elapsed_time(end), world, device) / args.steps
    assert torch.equal(out_hosts[(args.steps - 1) & 1], g.out.cpu()), "e2e output differs from the device run"
    h2d = n * cfg.hidden_size * 2
    d2h = n * cfg.hidden_size * 2

    # per-stage timing pass (eager, events around every launch) for the roofline
    taps = eng.make_taps(n)
    eng.forward(h, h, cfg.num_loops - 1, cfg.num_loops, taps=taps)
    torch.cuda.synchronize(device)
    stages = stage_timing(eng, h, steps=20)
    bytes_loop = algorithmic_bytes(cfg, spec, taps, n)
    flops_loop = algorithmic_flops(cfg, taps, n)
    gemm_names = ["gemm_edge_values", "gemm_expert_up", "gemm_expert_down"]
    gemm_ms = sum(stages[k]["ms_per_step"] for k in gemm_names)
    gemm_bytes = sum(bytes_loop[k] for k in gemm_names) * cfg.num_loops
    gemm_flops = sum(flops_loop[k] for k in gemm_names) * cfg.num_loops
    launches = sum(stages[k]["launches_per_step"] for k in gemm_names)
    peaks, peak_kind = load_peaks()
    roofline = gemm_roofline(gemm_bytes, gemm_flops, gemm_ms, launches, peaks, peak_kind,
                             NCU_TRAFFIC_PER_STEP.get(f"{args.config}:{cfg.expert_activation}"))

    line = {
        "metric": "spider_moe_block_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden states)",
        "config": workload_config(args, cfg, spec, world), "engine": args.engine,
        "weight_bytes": eng.weight_bytes(), "ms_per_step_median": med_step,
        "clocks": clk.summary(),
        "e2e": {"value": n * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": gpu_launches,
        "roofline": roofline,
        "stages_ms_per_step": {k: round(v["ms_per_step"], 5) for k, v in stages.items()},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, spec, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g
    if world > 1:
        barrier(world)
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
