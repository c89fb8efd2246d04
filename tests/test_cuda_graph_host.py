"""Host logic of the CUDA-graph decode runner (CPU): key, buckets, fallbacks
(spider_infer/cuda_graph.py:16-130)."""
import torch

from spider_web_moe_b200.cuda_graph import CudaGraphDecodeRunner, DecodeGraphKey


def test_key_and_bucket():
    r = CudaGraphDecodeRunner(length_bucket_size=64)
    assert r._bucket(1) == 64 and r._bucket(64) == 64 and r._bucket(65) == 128
    assert DecodeGraphKey(4, 64, 2) == DecodeGraphKey(4, 64, 2)
    assert len({DecodeGraphKey(4, 64, 2), DecodeGraphKey(4, 64, 2), DecodeGraphKey(4, 64, 3)}) == 2


def test_cpu_inputs_fall_back():
    r = CudaGraphDecodeRunner()
    calls = []

    def fn(ids, rids):
        calls.append(ids.shape)
        return ids.float() * 2

    out = r.run(fn, torch.ones(3, 1, dtype=torch.long), [0, 1, 2], cache_length=10)
    assert torch.equal(out, torch.full((3, 1), 2.0)) and calls == [(3, 1)]
    assert r.stats()["fallbacks"] == 1 and r.stats()["graphs"] == 0
    r.clear()
    assert r.stats()["fallbacks"] == 0
