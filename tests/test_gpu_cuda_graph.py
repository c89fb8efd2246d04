"""The block inside captured decode steps (spider_web_moe_b200.cuda_graph).

A decode callable in the shape of the reference's (embedding, the recurrent
block over all loops, a head) is captured by CudaGraphDecodeRunner and replayed
with new token ids: replays must equal eager calls bit for bit, for the
one-call driver (run_recurrent_full) and for the reference's per-loop module
calls alike, and the runner's key / hit / miss / fallback accounting follows
spider_infer/cuda_graph.py:79-130.
"""
import pytest
import torch

from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.cuda_graph import CudaGraphDecodeRunner
from spider_web_moe_b200.layer import SpiderMoELayer

pytestmark = pytest.mark.gpu


def decode_parts(cuda_device, dtype):
    cfg = ModelConfig(vocab_size=512, hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2,
                      num_loops=4, expert_ffn_size=512).validate()
    layer = SpiderMoELayer(cfg)
    synth.init_block_params_(layer, seed=21, std=0.05)
    torch.manual_seed(0)
    emb = torch.nn.Embedding(512, 256)
    head = torch.nn.Linear(256, 512)
    return cfg, layer.to(cuda_device), emb.to(cuda_device, dtype), head.to(cuda_device, dtype)


@pytest.mark.parametrize("dtype,per_loop", [(torch.bfloat16, False), (torch.float32, True),
                                            (torch.bfloat16, True)])
def test_decode_step_replays_match_eager(dtype, per_loop, cuda_device):
    cfg, layer, emb, head = decode_parts(cuda_device, dtype)

    def fn(ids, rids):
        x0 = emb(ids)
        if per_loop:  # the reference's _run_recurrent_full: one module call per loop
            h = x0
            for l in range(cfg.num_loops):
                h = layer(h, x0, l)
        else:
            h = layer.run_recurrent_full(x0, x0)
        return head(h)

    runner = CudaGraphDecodeRunner(length_bucket_size=64)
    g = torch.Generator(device="cpu").manual_seed(1)
    rids = list(range(48))
    with torch.no_grad():
        ids0 = torch.randint(0, 512, (48, 1), generator=g).to(cuda_device)
        first = runner.run(fn, ids0, rids, cache_length=70, num_loops=cfg.num_loops)
        assert torch.equal(first, fn(ids0, rids))  # the capturing call returns real logits
        for _ in range(3):
            ids = torch.randint(0, 512, (48, 1), generator=g).to(cuda_device)
            got = runner.run(fn, ids, rids, cache_length=100, num_loops=cfg.num_loops)  # same bucket (128)
            assert torch.equal(got, fn(ids, rids))
        st = runner.stats()
        assert st["graphs"] == 1 and st["misses"] == 1 and st["hits"] == 3 and st["fallbacks"] == 0
        assert st["keys"] == [{"batch_size": 48, "length_bucket": 128, "num_loops": cfg.num_loops}]
        # another bucket captures a second graph; other request ids and multi-token steps fall back
        runner.run(fn, ids0, rids, cache_length=129, num_loops=cfg.num_loops)
        runner.run(fn, ids0, rids[::-1], cache_length=100, num_loops=cfg.num_loops)
        two = torch.randint(0, 512, (48, 2), generator=g).to(cuda_device)
        assert torch.equal(runner.run(fn, two, rids, cache_length=100), fn(two, rids))
        st = runner.stats()
        assert st["graphs"] == 2 and st["misses"] == 2 and st["fallbacks"] == 2
    layer.engine(cuda_device, dtype, 48).check_status()

