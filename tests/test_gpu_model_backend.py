"""The spider_b200 backend inside a whole SpiderWebLM, against the reference's logits.

The model is the full-model restatement (oracle/spider_lm_oracle.py, pinned to
the reference's own logits on CPU by tests/test_oracle_model.py) with the
fixture's parameters; ``get_backend("spider_b200")(cfg, model=...)`` swaps its
recurrent block for the B200 layer (spider_infer/backends/spider.py:3-6 is the
builder signature it keeps) and routes the model's recurrent drivers to the
device.  The forward then runs the prelude / coda attention in torch on the GPU
and every recurrent loop through libspider_b200 (fp32 activations: the
CUDA-core engine).  The logits must match the reference's
(tests/golden/cfg1_model.pt, SpiderWebLM.forward model.py:673-701) within the
fp32 tolerance, through the model's own forward and through its
``_run_recurrent_full`` driver."""
import pytest
import torch

from spider_web_moe_b200.backends import get_backend
from spider_web_moe_b200.layer import SpiderMoELayer

from helpers import rel_err
from test_oracle_model import build_cfg1_model

pytestmark = pytest.mark.gpu


def test_backend_in_full_model_matches_reference_logits(cuda_device):
    fx, cfg, model = build_cfg1_model()
    model = get_backend("spider_b200")(cfg, device=cuda_device, model=model)
    assert isinstance(model.recurrent, SpiderMoELayer)
    ids = fx["ids"].to(cuda_device)
    with torch.no_grad():
        logits = model(ids)["logits"]
    torch.cuda.synchronize()
    assert rel_err(logits, fx["logits"]) < 1e-4
    # the model's recurrent driver (all loops in one library call) gives the same block output
    with torch.no_grad():
        x0 = model._embed(ids)
        h = x0
        for layer in model.prelude:
            h = layer(h, model.rope_cos, model.rope_sin)
        loops = [h]
        for loop_idx in range(cfg.num_loops):
            loops.append(model.recurrent(loops[-1], x0, loop_idx))
        full = model._run_recurrent_full(h, x0)
    assert rel_err(full, loops[-1]) < 1e-5
