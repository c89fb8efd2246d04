"""Host-side packing layouts (no GPU): the interleaved gate/up layout of the
SwiGLU experts (SB_EPI_SWIGLU_IL) round-trips and puts, for every block of 64
features, the 64 gate rows before the 64 up rows."""
import torch

from spider_web_moe_b200.engine import interleave_gate_up, split_gate_up


def test_interleave_round_trip_and_block_order():
    g = torch.randn(3, 192, 7)
    u = torch.randn(3, 192, 7)
    p = interleave_gate_up(g, u)
    assert p.shape == (3, 384, 7) and p.is_contiguous()
    for b in range(3):
        assert torch.equal(p[:, 128 * b:128 * b + 64], g[:, 64 * b:64 * b + 64])
        assert torch.equal(p[:, 128 * b + 64:128 * b + 128], u[:, 64 * b:64 * b + 64])
    assert torch.equal(split_gate_up(p, "gate"), g) and torch.equal(split_gate_up(p, "up"), u)


def test_interleave_per_row_vectors_and_packed_bytes():
    # biases / fp8 scales are [E, U]; int4 weights are uint8 [E, U, H/2]
    bg, bu = torch.randn(2, 128), torch.randn(2, 128)
    assert torch.equal(split_gate_up(interleave_gate_up(bg, bu), "up"), bu)
    qg = torch.randint(0, 256, (2, 128, 16), dtype=torch.uint8)
    qu = torch.randint(0, 256, (2, 128, 16), dtype=torch.uint8)
    assert torch.equal(split_gate_up(interleave_gate_up(qg, qu), "gate"), qg)
