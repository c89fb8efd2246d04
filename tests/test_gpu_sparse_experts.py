"""The drop-in sparse_expert_delta (sparse_experts.py:11-68 signature) on the
device against the oracle, on the cases of the reference's
test_sparse_experts_parity.py:53-98 (sparse == per-token dense mix, the same
expert in both slots adds its weights) plus a bf16 case on the tcgen05 engine.
Relative error per row (max-norm): 1e-5 fp32, 2e-2 bf16."""
import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200.sparse_experts import sparse_expert_delta

from helpers import rel_err

pytestmark = pytest.mark.gpu


def weights(e, u, h, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g) * scale for s in ((e, u, h), (e, u), (e, h, u), (e, h))]


@pytest.mark.parametrize("expert_parallel", [True, False])
def test_matches_dense_mix_fp32(expert_parallel, cuda_device):
    b, t, h, e, k, u = 3, 5, 32, 4, 2, 64
    g = torch.Generator().manual_seed(42)
    msgs = torch.randn(b, t, h, generator=g)
    tw, ti = torch.randn(b, t, e, generator=g).softmax(-1).topk(k, -1)
    tw = tw / tw.sum(-1, keepdim=True).clamp_min(1e-9)
    w = weights(e, u, h, 43)
    dev = [x.to(cuda_device) for x in w]
    got = sparse_expert_delta(msgs.to(cuda_device), ti.to(cuda_device), tw.to(cuda_device), *dev, num_experts=e,
                              top_k=k, expert_parallel=expert_parallel)
    assert got.shape == msgs.shape and got.dtype == msgs.dtype
    want = O.expert_delta(msgs, ti, tw, *w, e)
    assert rel_err(got, want) < 1e-5


def test_duplicate_slots_accumulate(cuda_device):
    n, h, e, u = 6, 16, 3, 32
    g = torch.Generator().manual_seed(7)
    msgs = torch.randn(1, n, h, generator=g)
    ti = torch.ones(1, n, 2, dtype=torch.long)
    tw = torch.tensor([0.4, 0.6]).expand(1, n, 2).contiguous()
    w = weights(e, u, h, 8)
    got = sparse_expert_delta(msgs.to(cuda_device), ti.to(cuda_device), tw.to(cuda_device),
                              *[x.to(cuda_device) for x in w], num_experts=e, top_k=2)
    want = O.expert_delta(msgs, ti, tw, *w, e)
    assert rel_err(got, want) < 1e-5


def test_bf16_tcgen05(cuda_device):
    b, t, h, e, k, u = 2, 50, 256, 16, 2, 512
    g = torch.Generator().manual_seed(44)
    msgs = torch.randn(b, t, h, generator=g).bfloat16()
    tw, ti = torch.randn(b, t, e, generator=g).softmax(-1).topk(k, -1)
    tw = tw / tw.sum(-1, keepdim=True).clamp_min(1e-9)
    w = [x.bfloat16() for x in weights(e, u, h, 45, scale=0.05)]
    got = sparse_expert_delta(msgs.to(cuda_device), ti.to(cuda_device), tw.to(cuda_device),
                              *[x.to(cuda_device) for x in w], num_experts=e, top_k=k)
    assert got.dtype == torch.bfloat16
    want = O.expert_delta(msgs.float(), ti, tw, *[x.float() for x in w], e)
    assert rel_err(got, want) < 2e-2


def test_new_weights_are_never_served_from_a_stale_engine(cuda_device):
    """The engine cache must not reuse packed weights for different tensors:
    weights freed and reallocated (the caching allocator tends to hand back the
    same addresses, at version 0), weights changed in place, and the same
    weights called with another top_k each give the oracle's result."""
    n, h, e, u = 12, 32, 4, 64
    g = torch.Generator().manual_seed(9)
    msgs = torch.randn(1, n, h, generator=g)
    tw, ti = torch.randn(1, n, e, generator=g).softmax(-1).topk(2, -1)
    tw = tw / tw.sum(-1, keepdim=True)
    md, tid, twd = msgs.to(cuda_device), ti.to(cuda_device), tw.to(cuda_device)
    for seed in (10, 11, 12):  # a fresh set of device weights each time, the old set freed
        w = weights(e, u, h, seed)
        dev = [x.to(cuda_device) for x in w]
        got = sparse_expert_delta(md, tid, twd, *dev, num_experts=e, top_k=2)
        assert rel_err(got, O.expert_delta(msgs, ti, tw, *w, e)) < 1e-5, f"weights of seed {seed}"
        del dev, got
    w = weights(e, u, h, 13)
    dev = [x.to(cuda_device) for x in w]
    sparse_expert_delta(md, tid, twd, *dev, num_experts=e, top_k=2)
    dev[0].mul_(2.0)  # in place: same address, new version
    w[0] = w[0] * 2.0
    got = sparse_expert_delta(md, tid, twd, *dev, num_experts=e, top_k=2)
    assert rel_err(got, O.expert_delta(msgs, ti, tw, *w, e)) < 1e-5, "in-place update"
    t1w, t1i = tw[..., :1] / tw[..., :1], ti[..., :1].contiguous()
    got = sparse_expert_delta(md, t1i.to(cuda_device), t1w.contiguous().to(cuda_device), *dev, num_experts=e, top_k=1)
    assert rel_err(got, O.expert_delta(msgs, t1i, t1w, *w, e)) < 1e-5, "another top_k"
