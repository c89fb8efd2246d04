"""Oracle sub-steps against the reference's scalar C++ library and its known-answer tests.

The library is built from the reference's own sources by oracle/Makefile
(``__graft_entry__.build()`` does it where the reference tree exists); the
known answers are the ones the reference's test suites assert
(kernels/tests/test_phase1_1.cpp, test_phase1_2.cpp, test_kernels.cpp,
tests/test_forge_04.py, tests/test_sparse_experts_parity.py).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ref_scalar as R
from oracle import spider_oracle as O

needs_ref = pytest.mark.skipif(not R.available(), reason="oracle/_ref not built (reference tree absent)")


@needs_ref
def test_router_matches_reference_scalar():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(200, 16, generator=g) * 2
    bias = torch.randn(3, 16, generator=g)
    rc, w, idx = R.router(logits.numpy(), bias.numpy(), 2, 4)
    assert rc == 0
    probs = (logits + bias[2]).softmax(-1)
    tw, ti = probs.topk(4, dim=-1)
    tw = tw / tw.sum(-1, keepdim=True).clamp_min(1e-9)
    assert np.array_equal(idx, ti.numpy())
    assert np.allclose(w, tw.numpy(), rtol=1e-6, atol=1e-7)
    # the oracle's router on h with an identity router weight gives the same routing
    tw2, ti2, _ = O.router(logits, torch.eye(16), bias[2], 4)
    assert torch.equal(ti2, ti)


@needs_ref
def test_edge_topm_matches_reference_scalar():
    g = torch.Generator().manual_seed(1)
    lg = torch.randn(50, 8, 8, generator=g)
    rc, idx, w = R.edge_topk(lg.numpy(), 3)
    assert rc == 0
    vals, ti = lg.topk(3, dim=-1)
    assert np.array_equal(idx, ti.numpy())
    assert np.allclose(w, vals.softmax(-1).numpy(), rtol=1e-6, atol=1e-7)


@needs_ref
def test_dynamic_messages_match_reference_scalar():
    g = torch.Generator().manual_seed(2)
    n, h, e, k, m = 40, 32, 8, 2, 3
    hid = torch.randn(n, h, generator=g)
    w_edge = torch.randn(e, h, h, generator=g) * 0.1
    probs = torch.randn(n, e, generator=g).softmax(-1)
    _, top_idx = probs.topk(k, -1)
    lg = torch.randn(n, e, e, generator=g)
    vals, eidx = lg.topk(m, -1)
    ew = vals.softmax(-1)
    rc, proj = R.edge_project(hid.numpy(), w_edge.numpy())
    assert rc == 0
    rc, msgs = R.message_passing_dynamic(proj, eidx.numpy(), ew.numpy(), top_idx.numpy())
    assert rc == 0
    coef = O.destination_coefficients(top_idx, eidx, ew, e)
    ours = O.messages_from_coefficients(hid, w_edge, coef)
    assert np.allclose(ours.numpy(), msgs, rtol=1e-5, atol=1e-5)
    dense = O.messages_dense(hid, w_edge, top_idx, eidx, ew)
    assert np.allclose(dense.numpy(), msgs, rtol=1e-5, atol=1e-5)


@needs_ref
def test_layernorm_epilogue_matches_reference_scalar():
    g = torch.Generator().manual_seed(3)
    n, h = 30, 64
    hh, d, x0 = (torch.randn(n, h, generator=g) for _ in range(3))
    gamma, beta = torch.randn(h, generator=g), torch.randn(h, generator=g)
    rc, out = R.loop_epilogue(hh.numpy(), d.numpy(), x0.numpy(), 0.5, 0.1, gamma.numpy(), beta.numpy(), 1e-5)
    assert rc == 0
    ours = O.block_epilogue(hh, d, x0, gamma, beta, 0.5, 0.1, 1e-5)
    assert np.allclose(ours.numpy(), out, rtol=1e-5, atol=2e-5)


# --- known-answer tests of the reference's own suites, applied to the oracle ---------

def test_kat_edge_topk():
    """kernels/tests/test_phase1_2.cpp:7-19: row [0,1,2] -> indices [2,1], weights sum to 1."""
    lg = torch.tensor([[[0., 1., 2.], [3., 0., 1.], [0., 0., 1.]]])
    vals, idx = lg.topk(2, -1)
    assert idx[0, 0].tolist() == [2, 1]
    w = vals.softmax(-1)
    assert abs(float(w[0, 0].sum()) - 1) < 1e-5
    if R.available():
        rc, ridx, rw = R.edge_topk(lg.numpy(), 2)
        assert rc == 0 and ridx[0, 0].tolist() == [2, 1]


def test_kat_dynamic_graph():
    """test_phase1_2.cpp:21-32: projected [[1,0],[0,4]], source 0 -> dst 1 with w 0.5: messages [0,2]."""
    proj = torch.tensor([[[1., 0.], [0., 4.]]])
    eidx = torch.tensor([[[1], [0]]])
    ew = torch.tensor([[[0.5], [1.0]]])
    top = torch.tensor([[0]])
    coef = O.destination_coefficients(top, eidx, ew, 2)
    msgs = (coef.unsqueeze(-1) * proj).sum(1)
    assert torch.allclose(msgs, torch.tensor([[0., 2.]]))


def test_kat_identity_projection():
    """test_phase1_1.cpp:8-20: identity W_edge reproduces h for every destination."""
    h = torch.arange(1, 9, dtype=torch.float32).view(2, 4) * 0.1
    w = torch.eye(4).expand(3, 4, 4)
    t = torch.einsum("nh,eoh->neo", h, w)
    assert torch.allclose(t, h.unsqueeze(1).expand(2, 3, 4))


def test_kat_router_weights_sum_to_one():
    """test_kernels.cpp:7-19: renormalised top-k weights sum to 1."""
    lg = torch.tensor([[1., 2, 3, 4], [4, 3, 2, 1]])
    tw, ti, _ = O.router(lg, torch.eye(4), torch.zeros(4), 2)
    assert torch.allclose(tw.sum(-1), torch.ones(2))
    assert ti.tolist() == [[3, 2], [0, 1]]


def test_kat_dispatch_plan_packing():
    """tests/test_forge_04.py:18-27: experts {0,1,2}; expert 1 holds both tokens."""
    top_i = torch.tensor([[0, 1], [1, 2]])
    top_w = torch.tensor([[0.7, 0.3], [0.6, 0.4]])
    plan = O.dispatch_plan(top_i, top_w, 4)
    assert {e for e, _, _ in plan} == {0, 1, 2}
    p1 = [p for e, p, _ in plan if e == 1][0]
    assert p1.tolist() == [0, 1]
    off, tok, w = O.plan_offsets(plan, 4)
    assert off.tolist() == [0, 1, 3, 4, 4]
    assert tok.tolist() == [0, 0, 1, 1]
    assert torch.allclose(w, torch.tensor([0.7, 0.3, 0.6, 0.4]))


def _dense_expert_delta(messages, top_indices, top_weights, w_up, b_up, w_down, b_down):
    """Dense mix of all experts weighted by the router (the reference test's formula,
    tests/test_sparse_experts_parity.py:41-50)."""
    e = w_up.shape[0]
    up = F.gelu(torch.einsum("nh,eoh->neo", messages, w_up) + b_up.view(1, e, -1))
    out = torch.einsum("neu,eou->neo", up, w_down) + b_down.view(1, e, -1)
    wt = messages.new_zeros(messages.shape[0], e).scatter_add_(-1, top_indices, top_weights)
    return (out * wt.unsqueeze(-1)).sum(1)


def test_sparse_delta_matches_dense_mix():
    """test_sparse_experts_parity.py:53-74 (seed 42, rtol=atol=1e-5)."""
    torch.manual_seed(42)
    n, h, e, k, u = 15, 32, 4, 2, 64
    msgs = torch.randn(n, h)
    tw, ti = torch.randn(n, e).softmax(-1).topk(k, -1)
    tw = tw / tw.sum(-1, keepdim=True).clamp_min(1e-9)
    w_up, b_up, w_down, b_down = torch.randn(e, u, h), torch.randn(e, u), torch.randn(e, h, u), torch.randn(e, h)
    got = O.expert_delta(msgs, ti, tw, w_up, b_up, w_down, b_down, e)
    want = _dense_expert_delta(msgs, ti, tw, w_up, b_up, w_down, b_down)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_sparse_delta_duplicate_slots_accumulate():
    """test_sparse_experts_parity.py:77-98: the same expert in both slots adds its weights."""
    torch.manual_seed(7)
    n, h, e, u = 6, 16, 3, 32
    msgs = torch.randn(n, h)
    ti = torch.ones(n, 2, dtype=torch.long)
    tw = torch.tensor([0.4, 0.6]).expand(n, 2).contiguous()
    w_up, b_up, w_down, b_down = torch.randn(e, u, h), torch.randn(e, u), torch.randn(e, h, u), torch.randn(e, h)
    got = O.expert_delta(msgs, ti, tw, w_up, b_up, w_down, b_down, e)
    want = _dense_expert_delta(msgs, ti, tw, w_up, b_up, w_down, b_down)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
    plan = O.dispatch_plan(ti, tw, e)
    assert len(plan) == 1 and plan[0][0] == 1 and torch.allclose(plan[0][2], torch.ones(n))
