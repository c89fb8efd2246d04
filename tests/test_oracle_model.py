"""The full-model restatement (oracle/spider_lm_oracle.py) against the
reference's own SpiderWebLM forward (fixture cfg1_model: the README smoke
model, fp32, 2 x 32 token ids, logits recorded from the reference).

The fixture's parameters are re-drawn with the fixture's seeded
initialisation; the recurrent block's must equal the stored state dict
exactly, and the logits must match the reference's within fp32 rounding."""
import torch

from oracle.spider_lm_oracle import OracleSpiderWebLM, seeded_init_
from spider_web_moe_b200.config import ModelConfig

from helpers import load_golden, rel_err


def build_cfg1_model():
    fx = load_golden("cfg1_model")
    cfg = ModelConfig(**fx["cfg"]).validate()
    cfg.expert_parallel = False
    model = OracleSpiderWebLM(cfg).eval()
    seeded_init_(model, seed=0)
    return fx, cfg, model


def test_seeded_parameters_reproduce_the_fixture_block():
    fx, _, model = build_cfg1_model()
    got = model.recurrent.state_dict()
    for k, v in fx["state_dict"].items():
        assert torch.equal(got[k], v), k


def test_full_model_logits_match_the_reference():
    fx, _, model = build_cfg1_model()
    with torch.no_grad():
        logits = model(fx["ids"])["logits"]
    assert logits.shape == fx["logits"].shape
    assert rel_err(logits, fx["logits"]) < 1e-5
