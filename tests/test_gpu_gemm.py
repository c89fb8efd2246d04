"""sb_grouped_gemm against a plain PyTorch fp32 statement of the same op.

out[r] = epilogue(W_g x[r] * s_g + b_g) for every row r of group g (rows
offsets[g] .. offsets[g+1]); LINEAR scales by row_scale[r] and writes fp32
(K-split partials summed by the caller), GELU / SwiGLU write bf16.  The cases
cover every tcgen05 schedule the library picks from the row counts (fixed
groups with 16-row boxes or 4-row gathers, the slot grid for mid-size tiles,
the persistent kernel for 128 / 256-column tiles), each weight format, and the
CUDA-core engine.  The weights are the device operands dequantised on the host
(fp8 -> bf16 with the per-row scale applied in fp32; int4 -> q * bf16 group
scale rounded to bf16), so the tolerance measures the GEMM alone: fp32
accumulation order and the bf16 rounding of the output.
"""
import ctypes as C

import pytest
import torch

from spider_web_moe_b200 import _lib as L
from spider_web_moe_b200.engine import interleave_gate_up, split_gate_up
from spider_web_moe_b200.quant import quantize_fp8_per_channel, quantize_int4

pytestmark = pytest.mark.gpu

EPI = {"linear": L.SB_EPI_LINEAR, "gelu": L.SB_EPI_GELU, "swiglu": L.SB_EPI_SWIGLU,
       "swiglu_il": L.SB_EPI_SWIGLU_IL}
WFMT = {"bf16": L.SB_W_BF16, "fp8": L.SB_W_FP8, "int4": L.SB_W_INT4}
ENGINE = {"tcgen05": L.SB_ENGINE_TCGEN05, "simt": L.SB_ENGINE_SIMT}


def device_weight(w, wfmt, group_size, dev):
    """(device operand, device scale, fp32 weights the device multiplies by)."""
    G, m, k = w.shape
    if wfmt == "bf16":
        wb = w.to(torch.bfloat16)
        return wb.to(dev), None, wb.float(), None
    if wfmt == "fp8":
        q = quantize_fp8_per_channel(w)
        return q.q.to(dev), q.scale.float().to(dev), q.q.float(), q.scale.float()
    t = quantize_int4(w, group_size)
    s_bf = t.scales.to(torch.bfloat16)
    packed = t.packed
    lo = (packed & 0x0F).to(torch.int8)
    hi = (packed >> 4).to(torch.int8)
    lo = torch.where(lo > 7, lo - 16, lo)
    hi = torch.where(hi > 7, hi - 16, hi)
    q = torch.stack([lo, hi], dim=-1).reshape(G, m, k).float()
    deq = (q * s_bf.float().repeat_interleave(group_size, dim=-1)).to(torch.bfloat16).float()
    return packed.to(dev), s_bf.to(dev), deq, None


def run_case(rows, m, k, wfmt, epi, engine, dev, bound=0, splits=1, gather=False, group_size=128, seed=0,
             null_offsets=False):
    g = torch.Generator().manual_seed(seed)
    G = len(rows)
    total = sum(rows)
    off = torch.tensor([0] + list(torch.tensor(rows).cumsum(0)), dtype=torch.int32)
    w = torch.randn(G, m, k, generator=g) * 0.05
    wg = torch.randn(G, m, k, generator=g) * 0.05
    bias = torch.randn(G, m, generator=g) * 0.1
    bias_g = torch.randn(G, m, generator=g) * 0.1
    x = torch.randn(total, k, generator=g).to(torch.bfloat16)
    row_scale = torch.rand(total, generator=g) + 0.5
    il = epi == "swiglu_il"
    if il:
        # one operand: gate and up rows interleaved in blocks of 64 (per-row scales
        # and biases likewise); the reference reads the two halves back
        a, a_s, deq_il, s_il = device_weight(interleave_gate_up(wg, w), wfmt, group_size, dev)
        deq, deq_g = split_gate_up(deq_il, "up"), split_gate_up(deq_il, "gate")
        s_row, s_row_g = (None, None) if s_il is None else (split_gate_up(s_il, "up"), split_gate_up(s_il, "gate"))
        ag = ag_s = None
    else:
        a, a_s, deq, s_row = device_weight(w, wfmt, group_size, dev)
        ag, ag_s, deq_g, s_row_g = (device_weight(wg, wfmt, group_size, dev) if epi == "swiglu"
                                    else (None, None, None, None))

    # torch fp32 statement
    want = torch.zeros(total, m)
    for gi in range(G):
        lo, hi = int(off[gi]), int(off[gi + 1])
        if hi == lo:
            continue
        y = x[lo:hi].float() @ deq[gi].T
        if s_row is not None:
            y = y * s_row[gi]
        y = y + bias[gi]
        if epi == "linear":
            y = y * row_scale[lo:hi, None]
        elif epi == "gelu":
            y = torch.nn.functional.gelu(y)
        else:
            z = x[lo:hi].float() @ deq_g[gi].T
            if s_row_g is not None:
                z = z * s_row_g[gi]
            y = torch.nn.functional.silu(z + bias_g[gi]) * y
        want[lo:hi] = y

    # the GEMM's token rows: contiguous, or gathered from a permuted source
    perm = torch.randperm(total, generator=g)
    src = torch.empty_like(x)
    src[perm] = x
    d_x = (src if gather else x).to(dev)
    d_idx = perm.to(torch.int32).to(dev)
    d_off = off.to(dev)
    out_dtype = torch.float32 if epi == "linear" else torch.bfloat16
    out = torch.full((splits, total, m), float("nan"), dtype=out_dtype, device=dev)
    status = torch.zeros(64, dtype=torch.int32, device=dev)
    keep = [a, a_s, ag, ag_s, d_x, d_idx, d_off, out, status]
    d_bias, d_bias_g, d_rs = bias.to(dev), bias_g.to(dev), row_scale.to(dev)
    if il:
        d_bias = interleave_gate_up(bias_g, bias).to(dev)
    keep += [d_bias, d_bias_g, d_rs]

    args = L.GemmArgs()
    args.engine = ENGINE[engine]
    args.wfmt = WFMT[wfmt]
    args.act_dtype = L.SB_BF16
    args.epilogue = EPI[epi]
    args.num_groups = G
    rows_a = 2 * m if il else m  # weight rows per group
    args.m_rows = rows_a
    args.k = k
    args.group_size = group_size
    args.a_group_rows = rows_a
    args.lda = k
    args.a_rows_total = G * rows_a
    args.a = a.data_ptr()
    args.a_scale = a_s.data_ptr() if a_s is not None else None
    if epi == "swiglu":
        args.a_gate = ag.data_ptr()
        args.a_gate_scale = ag_s.data_ptr() if ag_s is not None else None
        args.bias_gate = d_bias_g.data_ptr()
    args.bias = d_bias.data_ptr()
    args.bias_group_stride = rows_a
    args.x = d_x.data_ptr()
    args.ldx = k
    if gather:
        args.x_row_index = d_idx.data_ptr()
        args.x_rows = total
    args.max_rows = total
    args.rows_hint = total
    args.group_rows_bound = bound
    args.offsets = None if null_offsets else d_off.data_ptr()  # NULL: one dense group (G == 1)
    args.row_scale = d_rs.data_ptr() if epi == "linear" else None
    args.out = out.data_ptr()
    args.ldo = m
    args.splits = splits
    args.split_stride = total * m
    args.status = status.data_ptr()
    lib = L.load()
    L.check(lib.sb_grouped_gemm(C.byref(args), C.c_void_p(torch.cuda.current_stream().cuda_stream)), "sb_grouped_gemm")
    torch.cuda.synchronize()
    assert int(status.abs().sum()) == 0, status[:8].tolist()
    got = out.float().sum(0).cpu() if epi == "linear" else out[0].float().cpu()
    assert not torch.isnan(got).any()
    del keep
    return got, want


def check(got, want, epi):
    epi = "swiglu" if epi == "swiglu_il" else epi
    err = (got - want).abs()
    # fp32 accumulation order (LINEAR), plus bf16 rounding of the output (GELU / SwiGLU)
    tol = (1e-4 if epi == "linear" else 8e-3) * want.abs() + 2e-4 * want.abs().max()
    bad = err > tol
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} outside tolerance, max err {float(err.max()):.3e}"


# (rows per group, bound, splits, gather): which schedule the library takes
SCHEDULES = {
    "fixed16_gather": ([5, 0, 16, 9, 1], 16, 1, True),
    "fixed64": ([40, 64, 3, 0, 57], 64, 1, False),
    "fixed_multi_tile": ([150, 7, 0, 70], 64, 1, False),   # groups beyond the bound loop over row tiles
    "fixed64_split2": ([40, 64, 3, 0, 57], 64, 2, False),  # fp8 / int4: the fixed kernel's conversion
    "slot64": ([70, 40, 90, 1], 0, 1, False),
    # fp8 / int4 decode batches with one hot group (2 items of 256 rows) and many
    # small ones: the quantised decode kernel, token rows gathered
    "qdec_skewed_gather": ([300, 2, 0, 17, 64, 1, 0, 5, 33, 9, 0, 3, 40, 8, 1, 6], 0, 1, True),
    "slot64_split2": ([70, 40, 90, 1], 0, 2, False),
    "persistent128": ([100, 130, 0, 90, 120], 0, 1, False),
    "persistent256": ([300, 0, 517, 129], 0, 1, False),
    "tile256_split2": ([300, 0, 517, 129], 0, 2, False),
}


@pytest.mark.parametrize("sched", sorted(SCHEDULES))
@pytest.mark.parametrize("wfmt", ["bf16", "fp8", "int4"])
def test_tcgen05_linear_and_gelu(sched, wfmt, cuda_device):
    rows, bound, splits, gather = SCHEDULES[sched]
    for epi in (["linear"] if splits > 1 else ["linear", "gelu"]):
        got, want = run_case(rows, 256, 512, wfmt, epi, "tcgen05", cuda_device, bound=bound, splits=splits,
                             gather=gather, seed=len(sched) + len(wfmt))
        check(got, want, epi)


@pytest.mark.parametrize("sched", ["fixed64", "slot64", "persistent128", "persistent256"])
@pytest.mark.parametrize("wfmt", ["bf16", "fp8", "int4"])
def test_tcgen05_swiglu(sched, wfmt, cuda_device):
    rows, bound, splits, gather = SCHEDULES[sched]
    got, want = run_case(rows, 256, 384, wfmt, "swiglu", "tcgen05", cuda_device, bound=bound, splits=splits,
                         gather=gather, seed=7)
    check(got, want, "swiglu")


@pytest.mark.parametrize("sched", ["fixed16_gather", "fixed64", "fixed_multi_tile", "slot64", "qdec_skewed_gather",
                                   "persistent128", "persistent256"])
@pytest.mark.parametrize("wfmt", ["bf16", "fp8", "int4"])
def test_tcgen05_swiglu_interleaved(sched, wfmt, cuda_device):
    """SB_EPI_SWIGLU_IL, the layout the block's SwiGLU experts use: gate and up
    rows of one operand, the two halves of each 128-row tile handed across
    between epilogue warps; every schedule (fixed groups, slot grid, the
    persistent and CTA-pair kernels)."""
    rows, bound, splits, gather = SCHEDULES[sched]
    got, want = run_case(rows, 256, 384, wfmt, "swiglu_il", "tcgen05", cuda_device, bound=bound, splits=splits,
                         gather=gather, seed=9)
    check(got, want, "swiglu_il")


@pytest.mark.parametrize("epi", ["linear", "gelu"])
@pytest.mark.parametrize("rows", [[300, 0, 517, 129], [40, 256, 0, 1000]])
def test_cta_pair_kernel(epi, rows, cuda_device):
    """bf16 weights with at least two 256-row pair tiles take the CTA-pair
    kernel (tcgen05.mma.cta_group::2); ragged groups end in short tiles whose
    MMA width shrinks to the rows they hold."""
    got, want = run_case(rows, 512, 384, "bf16", epi, "tcgen05", cuda_device, seed=len(rows) + sum(rows) % 7)
    check(got, want, epi)


@pytest.mark.parametrize("wfmt", ["fp8", "int4"])
@pytest.mark.parametrize("epi,m", [("linear", 192), ("swiglu_il", 256), ("swiglu_il", 192), ("gelu", 320)])
def test_quantised_decode_many_items(wfmt, epi, m, cuda_device):
    """The quantised decode kernel at a cfg5-like shape: 128 groups with
    Zipf-skewed rows (2048 in all, the largest above 256: two items), a weight
    matrix whose rows are not a multiple of 128 (LINEAR), and more items than
    SMs, so every CTA walks several items and both TMEM accumulators turn over.
    Weight matrices whose rows end inside a 256-row tile: LINEAR 192, GELU 320,
    SwiGLU 384 interleaved rows (the last tile holds one 128-row block)."""
    g = torch.Generator().manual_seed(21)
    weights = 1.0 / torch.arange(1, 129).float() ** 1.1
    picks = torch.multinomial(weights, 2048, replacement=True, generator=g)
    rows = [int(v) for v in torch.bincount(picks, minlength=128)]
    rows[0] = max(rows[0], 300)
    got, want = run_case(rows, m, 512, wfmt, epi, "tcgen05", cuda_device, gather=epi != "linear", seed=13)
    check(got, want, epi)


def test_persistent_many_tiles_and_groups(cuda_device):
    """More tiles than SMs (each CTA loops, both TMEM accumulators turn over many
    times) and 200 groups of ragged sizes, zeros included."""
    g = torch.Generator().manual_seed(5)
    rows = [int(v) for v in torch.randint(0, 400, (200,), generator=g)]
    rows[3] = rows[50] = 0
    got, want = run_case(rows, 384, 256, "bf16", "gelu", "tcgen05", cuda_device, seed=11)
    check(got, want, "gelu")


@pytest.mark.parametrize("epi", ["linear", "gelu", "swiglu", "swiglu_il"])
@pytest.mark.parametrize("wfmt", ["bf16", "fp8", "int4"])
def test_simt_engine(epi, wfmt, cuda_device):
    m = 192 if epi == "swiglu_il" else 160  # the interleaved layout comes in 64-feature blocks
    got, want = run_case([33, 0, 70, 5], m, 256, wfmt, epi, "simt", cuda_device, seed=3)
    check(got, want, epi)


@pytest.mark.parametrize("engine", ["tcgen05", "simt"])
@pytest.mark.parametrize("n", [40, 300, 2000])
def test_single_dense_group_without_offsets(engine, n, cuda_device):
    """offsets = NULL with num_groups = 1 (the router-logit GEMM): one group of all rows."""
    got, want = run_case([n], 64, 512, "bf16", "linear", engine, cuda_device, seed=n, null_offsets=True)
    check(got, want, "linear")
