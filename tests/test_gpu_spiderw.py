"""A block loaded from a .spiderw bundle (written by the reference's exporter)
runs on the device and matches the oracle on the bundle's parameters (biases
zero: the format stores none)."""
import os

import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import spiderw as W
from spider_web_moe_b200 import synth
from spider_web_moe_b200.engine import BlockEngine
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
PATH = os.path.join(GOLDEN, "e4_block.spiderw")


def oracle_params(bf16=False):
    sd = {k: v.contiguous() for k, v in W.block_state_dict(W.load_spiderw(PATH)).items()}
    if bf16:  # the bf16 engine stores the weights rounded to bf16
        sd = {k: v.bfloat16().float() for k, v in sd.items()}
    return O.params_from_state_dict(sd, 4)


def test_layer_from_spiderw_matches_oracle(cuda_device):
    layer = SpiderMoELayer.from_spiderw(PATH, device=cuda_device)
    cfg = layer.cfg
    h, x0 = synth.block_inputs(40, cfg.hidden_size, seed=23)
    p = oracle_params()
    with torch.no_grad():
        for l in range(cfg.num_loops):
            got = layer(h.to(cuda_device), x0.to(cuda_device), l)
            want = O.block_forward(p, h, x0, l, cfg)["h_out"]
            assert rel_err(got, want) < 1e-5, l
            h = want


def test_engine_from_spiderw_bf16_all_loops(cuda_device):
    eng = BlockEngine.from_spiderw(PATH, cuda_device, act_dtype=torch.bfloat16, max_tokens=64)
    cfg = eng.cfg
    h, x0 = synth.block_inputs(64, cfg.hidden_size, seed=24)
    out = eng.forward(h.to(cuda_device, torch.bfloat16), x0.to(cuda_device, torch.bfloat16))
    torch.cuda.synchronize()
    eng.check_status()
    want, _ = O.run_loops(oracle_params(bf16=True), h.bfloat16().float(), x0.bfloat16().float(), cfg)
    assert rel_err(out, want) < 2e-2
