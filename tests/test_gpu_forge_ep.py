"""Forge EP mirror (spider_web_moe_b200.forge_ep) against the reference semantics.

Cases follow the reference's tests/test_forge_04.py: the two-token plan KAT
(experts {0,1,2}, expert 1 holding both tokens), dispatch -> FFN -> combine
against a dense per-token mix, and the ForgeEP front end.  Plans are compared
bit-exact with the oracle's restatement of build_dispatch_plan.
"""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import forge_ep as F

pytestmark = pytest.mark.gpu


def test_plan_kat_two_tokens(cuda_device):
    top_indices = torch.tensor([[[0, 1], [1, 2]]], device=cuda_device)
    top_weights = torch.tensor([[[0.7, 0.3], [0.6, 0.4]]], device=cuda_device)
    plan = F.build_dispatch_plan(top_indices, top_weights, num_experts=4, local_only=False)
    assert {a.expert_id for a in plan.assignments} == {0, 1, 2}
    a1 = plan.tokens_for(1)
    assert a1 is not None and a1.token_index.numel() == 2
    assert a1.token_index.tolist() == [0, 1]
    assert torch.equal(a1.weights.cpu(), torch.tensor([0.3, 0.6]))
    assert plan.tokens_for(3) is None
    assert F.get_last_ep_dispatch_backend().startswith("dispatch_plan")


@pytest.mark.parametrize("n,k,e", [(37, 2, 5), (300, 4, 16), (1000, 8, 64)])
def test_plan_matches_oracle_bit_exact(n, k, e, cuda_device):
    g = torch.Generator().manual_seed(n + k)
    idx = torch.randint(0, e, (n, k), generator=g)
    idx[::3, -1] = idx[::3, 0]                 # repeated experts inside a token
    w = torch.rand(n, k, generator=g) - 0.1    # some non-positive summed weights
    want = O.dispatch_plan(idx, w, e)
    plan = F.build_dispatch_plan(idx.to(cuda_device), w.to(cuda_device), num_experts=e, local_only=False)
    assert len(plan.assignments) == len(want)
    for a, (eid, pos, tw) in zip(plan.assignments, want):
        assert a.expert_id == eid
        assert torch.equal(a.token_index.cpu(), pos)
        assert torch.equal(a.weights.cpu(), tw)
    off, tok, tw = O.plan_offsets(want, e)
    assert torch.equal(plan.offsets.cpu().long(), off)
    assert torch.equal(plan.rows.cpu().long(), tok)


def test_dispatch_tokens_gathers_rows(cuda_device):
    msgs = torch.randn(2, 5, 24, device=cuda_device)
    top_i = torch.tensor([[[1, 0], [2, 1], [0, 0], [1, 2], [2, 0]]] * 2, device=cuda_device)
    top_w = torch.full(top_i.shape, 0.5, device=cuda_device)
    plan = F.build_dispatch_plan(top_i, top_w, num_experts=3, local_only=False)
    for a in plan.assignments:
        got = F.dispatch_tokens(msgs, a)
        assert torch.equal(got, msgs.reshape(-1, 24).index_select(0, a.token_index))
        got_bf = F.dispatch_tokens(msgs.bfloat16(), a)
        assert torch.equal(got_bf, msgs.bfloat16().reshape(-1, 24).index_select(0, a.token_index))


def dense_mix(messages, top_i, top_w, w_up, b_up, w_down, b_down):
    """The reference test's per-token loop (test_forge_04.py:47-60), on the CPU in fp32."""
    b, t, h = messages.shape
    k = top_i.shape[-1]
    ref = torch.zeros(b * t, h)
    flat_m, flat_i, flat_w = messages.reshape(-1, h), top_i.reshape(-1, k), top_w.reshape(-1, k)
    for n in range(flat_m.shape[0]):
        for slot in range(k):
            eid = int(flat_i[n, slot])
            out = O.expert_ffn(flat_m[n:n + 1], w_up[eid], b_up[eid], w_down[eid], b_down[eid])
            ref[n] += out[0] * flat_w[n, slot]
    return ref.view(b, t, h)


def test_dispatch_ffn_matches_dense_mix(cuda_device):
    torch.manual_seed(0)
    b, t, h, e, k = 2, 3, 16, 4, 2
    messages = torch.randn(b, t, h)
    top_w, top_i = torch.topk(torch.randn(b, t, e), k=k, dim=-1)
    top_w = torch.softmax(top_w, dim=-1)
    w_up, b_up = torch.randn(e, 32, h), torch.randn(e, 32)
    w_down, b_down = torch.randn(e, h, 32), torch.randn(e, h)
    dev = lambda x: x.to(cuda_device)
    delta = F.dispatch_expert_ffn(dev(messages), dev(top_i), dev(top_w), w_up=dev(w_up), b_up=dev(b_up),
                                  w_down=dev(w_down), b_down=dev(b_down), num_experts=e)
    assert delta.shape == messages.shape
    ref = dense_mix(messages, top_i, top_w, w_up, b_up, w_down, b_down)
    assert torch.allclose(delta.cpu(), ref, rtol=1e-4, atol=1e-4)
    assert "dispatch" in F.get_last_ep_dispatch_backend()


def test_forge_ep_front_end_and_expert_fn(cuda_device):
    torch.manual_seed(1)
    b, t, h, e, k = 1, 4, 8, 3, 2
    messages = torch.randn(b, t, h, device=cuda_device)
    top_i = torch.randint(0, e, (b, t, k), device=cuda_device)
    top_w = torch.softmax(torch.randn(b, t, k, device=cuda_device), dim=-1)
    w_up, b_up = torch.randn(e, 16, h, device=cuda_device), torch.zeros(e, 16, device=cuda_device)
    w_down, b_down = torch.randn(e, h, 16, device=cuda_device), torch.zeros(e, h, device=cuda_device)
    ep = F.ForgeEP()
    fused = ep.run_dispatched_ffn(messages, top_i, top_w, w_up=w_up, b_up=b_up, w_down=w_down, b_down=b_down,
                                  num_experts=e)
    assert fused.shape == (b, t, h)
    st = ep.stats()
    assert st["forge_version_target"] == "0.4" and "dispatch" in st["last_kernel"] and st["calls"] == 1

    def expert_fn(eid, toks):
        up = torch.nn.functional.gelu(torch.nn.functional.linear(toks, w_up[eid], b_up[eid]))
        return torch.nn.functional.linear(up, w_down[eid], b_down[eid])

    looped = ep.run_dispatched_ffn(messages, top_i, top_w, w_up=w_up, b_up=b_up, w_down=w_down, b_down=b_down,
                                   num_experts=e, expert_fn=expert_fn)
    assert torch.allclose(looped, fused, rtol=1e-4, atol=1e-4)
    meta = ep.dispatch_meta(top_i, e)
    assert meta["world"] == 1 and meta["local_experts"] == [0, 1, 2]
    assert isinstance(F.DeepEPStyleDispatcher(), F.ForgeEP)
