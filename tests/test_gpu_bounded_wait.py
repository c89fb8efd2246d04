"""Failure detection on the GPU without a GPU fault: a bounded wait runs out.

Every spin-wait in the library's kernels (mbarriers of the TMA / MMA pipeline,
peer ranks' exchange flags) gives up after about 2 s of %globaltimer time,
ORs its bit into a device status word and returns.  This test makes one run
out on purpose in the safe way: sb_ep_wait on a world-of-one exchange region
whose flag nothing ever raises (the peer that would raise it "died" before
sending).  It checks that the kernel returns by itself within a few seconds,
that SB_DEVERR_PEER_WAIT is set, that the engine's check_status() raises, and
that the context is still healthy afterwards (a block forward on the same
device matches the oracle).  Nothing here traps, faults or hangs.
"""
import time

import pytest
import torch

from oracle import spider_oracle as O
from spider_web_moe_b200 import _lib as L
from spider_web_moe_b200 import synth
from spider_web_moe_b200.config import ModelConfig
from spider_web_moe_b200.engine import BlockEngine

from helpers import TOL, rel_err

pytestmark = pytest.mark.gpu


def small_engine(device):
    cfg = ModelConfig(hidden_size=128, num_heads=4, num_experts=8, top_k=2, edges_per_expert=2, num_loops=1,
                      expert_ffn_size=256).validate()
    sd = synth.synthetic_state_dict(cfg, seed=51, device=device, round_bf16=True)
    return cfg, sd, BlockEngine(cfg, sd, device, act_dtype=torch.bfloat16, max_tokens=16)


def test_peer_flag_wait_expires_and_reports(cuda_device):
    lib = L.load()
    cfg, sd, eng = small_engine(cuda_device)
    world, cap, hidden = 1, 4, cfg.hidden_size
    pitch = lib.sb_ep_row_pitch(hidden, L.SB_BF16, cfg.top_k)
    nbytes = lib.sb_ep_peer_region_bytes(world, cap, pitch, hidden)
    assert nbytes > 0
    region = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)  # flags at zero: nobody will raise them
    assert eng.status() == 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib.sb_ep_wait(region.data_ptr(), world, cap, pitch, hidden, 0, eng.status_ptr(),
                        torch.cuda.current_stream().cuda_stream)
    L.check(rc, "sb_ep_wait")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 1.0 < waited < 30.0, f"the wait returned after {waited:.2f} s"
    assert eng.status() & L.SB_DEVERR_PEER_WAIT
    with pytest.raises(L.SpiderB200Error) as ei:
        eng.check_status()
    assert ei.value.code == L.SB_ERR_DEVICE_STATUS

    # the context is intact: the block still computes the right thing
    n = 16
    h, _ = synth.block_inputs(n, hidden, seed=52)
    h = h.to(torch.bfloat16).float().view(n, -1)
    out = eng.forward(h.to(cuda_device, torch.bfloat16), h.to(cuda_device, torch.bfloat16), 0, 1)
    p = O.params_from_state_dict({k: v.cpu() for k, v in sd.items()}, cfg.num_experts)
    want = O.block_forward(p, h, h, 0, cfg)
    assert rel_err(out, want["h_out"]) < TOL["bf16"]
