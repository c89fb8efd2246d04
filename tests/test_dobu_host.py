"""Host side of the Dobu store (CPU): its residency decisions replay the
reference store's LRU accounting (tests/golden/dobu.pt) call for call, with the
device copies stubbed out.  The experts a call materialises are those with a
positive summed routing weight for some token, in ascending order
(expert_store.py:142-152), which sb_active_experts computes on the device."""
import torch
from torch import nn

from spider_web_moe_b200.dobu import ExpertChunkStore

from helpers import load_golden


def active_experts(idx, w, num_experts):
    idx, w = idx.reshape(-1, idx.shape[-1]), w.reshape(-1, w.shape[-1])
    act = set()
    for t in range(idx.shape[0]):
        for e in set(idx[t].tolist()):
            if float((w[t] * (idx[t] == e)).sum()) > 0:
                act.add(e)
    return sorted(a for a in act if 0 <= a < num_experts)


def test_lru_accounting_matches_reference(monkeypatch):
    fx = load_golden("dobu")
    experts = nn.ModuleList([nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16)) for _ in range(6)])
    experts.load_state_dict(fx["experts"])
    store = ExpertChunkStore(experts, compute_device="cpu", max_gpu_experts=2)
    loaded = []
    monkeypatch.setattr(store, "_load", lambda pool, e, slot: (loaded.append((e, slot)), setattr(store, "loads",
                                                                                              store.loads + 1)))
    pool = {"dtype": torch.float32}
    for c in fx["calls"]:
        used = active_experts(c["idx"], c["w"], 6)
        S = store._slots()
        for w0 in range(0, len(used), S):
            wave = {}
            for e in used[w0:w0 + S]:
                store._materialise(pool, e, wave)
            assert len(set(wave.values())) == len(wave)  # a wave's experts sit in distinct slots
        st = store.stats()
        assert (st["hits"], st["misses"], st["loads"]) == (c["hits"], c["misses"], c["loads"])
        assert st["gpu_hot_experts"] == c["hot"]
        assert st["storage_bytes"] == c["storage_bytes"] and st["gpu_working_set_bytes"] == c["gpu_bytes"]
    assert len(loaded) == fx["calls"][-1]["loads"]
