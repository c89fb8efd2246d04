"""HostPipeline: block steps from pinned host memory with the copies of the
neighbouring steps overlapping each step's graph; every step's output must
equal a plain device run of that step's input."""
import pytest
import torch

from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.engine import BlockEngine, HostPipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("x0_is_h", [True, False])
def test_pipeline_steps_equal_device_runs(x0_is_h, cuda_device):
    cfg = ModelConfig(hidden_size=256, num_heads=4, num_experts=16, top_k=2, edges_per_expert=2, num_loops=3,
                      expert_ffn_size=512).validate()
    sd = synth.synthetic_state_dict(cfg, seed=31, device=cuda_device, round_bf16=True)
    eng = BlockEngine(cfg, sd, cuda_device, act_dtype=torch.bfloat16, max_tokens=48)
    pipe = HostPipeline(eng, 48, x0_is_h=x0_is_h)
    g = torch.Generator().manual_seed(2)
    steps = 7
    hs = [torch.randn(48, 256, generator=g).bfloat16().pin_memory() for _ in range(steps)]
    xs = [torch.randn(48, 256, generator=g).bfloat16().pin_memory() for _ in range(steps)]
    outs = [torch.empty(48, 256, dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    pipe.run(hs, outs, None if x0_is_h else xs)
    torch.cuda.synchronize()
    eng.check_status()
    for s in range(steps):
        h = hs[s].to(cuda_device)
        want = eng.forward(h, h if x0_is_h else xs[s].to(cuda_device)).cpu()
        assert torch.equal(outs[s], want), s
