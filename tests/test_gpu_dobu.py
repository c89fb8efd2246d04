"""Dobu expert offload (spider_web_moe_b200.dobu.ExpertChunkStore) against the
reference's store (tests/golden/dobu.pt): the delta of every call within fp32
tolerance, and the LRU accounting (hits, misses, loads, resident experts in
recency order, byte counts) equal after every call; a layer with
offload_experts over two loops against the reference layer."""
import pytest
import torch
from torch import nn

from spider_web_moe_b200 import synth
from spider_web_moe_b200.dobu import ExpertChunkStore
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import golden_cfg, load_golden, rel_err

pytestmark = pytest.mark.gpu


def test_store_matches_reference_calls(cuda_device):
    fx = load_golden("dobu")
    experts = nn.ModuleList([nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16)) for _ in range(6)])
    experts.load_state_dict(fx["experts"])
    store = ExpertChunkStore(experts, storage_device="cpu", compute_device=cuda_device, max_gpu_experts=2)
    for c in fx["calls"]:
        d = store.sparse_delta(c["msgs"].to(cuda_device), c["idx"].to(cuda_device), c["w"].to(cuda_device), top_k=2)
        assert d.shape == c["delta"].shape and d.dtype == c["delta"].dtype
        assert rel_err(d, c["delta"]) < 1e-5
        st = store.stats()
        assert (st["hits"], st["misses"], st["loads"]) == (c["hits"], c["misses"], c["loads"])
        assert st["gpu_hot_experts"] == c["hot"]
        assert st["storage_bytes"] == c["storage_bytes"] and st["gpu_working_set_bytes"] == c["gpu_bytes"]
    store.release_gpu()
    assert store.stats()["gpu_hot_experts"] == []


@pytest.mark.parametrize("cap", [0, 1, 6])
def test_store_any_capacity_same_delta(cap, cuda_device):
    """Streaming (0), one slot (a wave per expert) and everything resident give
    the same delta; with room for every expert the second call only hits."""
    fx = load_golden("dobu")
    experts = nn.ModuleList([nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16)) for _ in range(6)])
    experts.load_state_dict(fx["experts"])
    store = ExpertChunkStore(experts, compute_device=cuda_device, max_gpu_experts=cap)
    c = fx["calls"][0]
    args = (c["msgs"].to(cuda_device), c["idx"].to(cuda_device), c["w"].to(cuda_device))
    assert rel_err(store.sparse_delta(*args, top_k=2), c["delta"]) < 1e-5
    assert rel_err(store.sparse_delta(*args, top_k=2), c["delta"]) < 1e-5
    st = store.stats()
    if cap == 6:
        assert st["misses"] == 3 and st["hits"] == 3 and st["loads"] == 3
    if cap == 0:
        assert st["misses"] == 6 and st["loads"] == 6 and st["gpu_hot_experts"] == []


def test_layer_with_offload_matches_reference(cuda_device):
    fx = load_golden("dobu")
    cfg = golden_cfg(fx)
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=fx["seed"], std=fx["std"])
    layer = layer.to(cuda_device).eval()
    h, x0 = fx["h"].to(cuda_device), fx["x0"].to(cuda_device)
    with torch.no_grad():
        for l, want in enumerate(fx["outs"]):
            h = layer(h, x0, l)
            assert rel_err(h, want) < 1e-5 * (l + 1), l
    st = layer.expert_store(cuda_device).stats()
    assert {k: st[k] for k in fx["layer_stats"]} == fx["layer_stats"]
