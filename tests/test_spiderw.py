""".spiderw bundles (spider_web_moe_b200.spiderw) against the reference's format
tools (CPU).

tests/golden/e4_block.spiderw was written by the reference's exporter
(scripts/export_native_weights.py) from seeded block parameters and
mixed_sections.spiderw by the reference's writer; spiderw.pt holds what the
reference's loader read back from both (tests/golden/make_golden.py).
"""
import os
import struct

import numpy as np
import pytest
import torch

from spider_web_moe_b200 import spiderw as W
from spider_web_moe_b200 import synth

from helpers import GOLDEN, load_golden


def test_loader_reads_the_reference_export():
    fx = load_golden("spiderw")
    b = W.load_spiderw(os.path.join(GOLDEN, "e4_block.spiderw"))
    assert vars(b.meta) == fx["block_meta"]
    assert b.meta.tied_embeddings and not b.meta.has_csr and b.csr is None
    assert sorted(b.tensors) == sorted(fx["block_sections"])
    for k, v in fx["block_sections"].items():
        assert torch.equal(torch.from_numpy(np.array(b.tensors[k])), v), k
    with pytest.raises(KeyError):
        b.require("csr_col_idx")


def test_block_state_dict_recovers_the_parameters():
    """The bundle maps back onto the layer's parameter names; the format keeps
    no biases, so those come back as zeros."""
    fx = load_golden("spiderw")
    cfg = W.model_config(W.load_spiderw(os.path.join(GOLDEN, "e4_block.spiderw")).meta)
    sd = synth.synthetic_state_dict(cfg, seed=fx["seed"], std=fx["std"])
    got = W.block_state_dict(W.load_spiderw(os.path.join(GOLDEN, "e4_block.spiderw")))
    for k, v in got.items():
        if k.endswith(".bias") and k not in ("norm.bias",):
            assert float(v.abs().max()) == 0.0, k
        else:
            assert torch.equal(v.contiguous(), sd[k]), k
    assert set(got) <= set(sd)


def test_writer_matches_the_reference_writer_byte_for_byte(tmp_path):
    fx = load_golden("spiderw")
    meta = W.SpiderWMeta(**fx["mixed_meta"])
    tensors = {k: v.numpy() for k, v in fx["mixed_in"].items()}
    out = tmp_path / "mine.spiderw"
    W.write_spiderw(out, meta, tensors)
    assert out.read_bytes() == open(os.path.join(GOLDEN, "mixed_sections.spiderw"), "rb").read()
    b = W.load_spiderw(out)
    assert sorted(b.tensors) == sorted(fx["mixed_sections"])
    for k, v in fx["mixed_sections"].items():
        assert torch.equal(torch.from_numpy(np.array(b.tensors[k])), v), k
    assert b.meta.has_csr and sorted(b.csr) == fx["mixed_csr"]


def _section(sid, dt, payload, shape):
    dims = list(shape) + [1] * (4 - len(shape))
    return struct.pack("<IIQI", sid, dt, len(payload), len(shape)) + struct.pack("<4I", *dims) + payload


def test_bf16_sections_and_truncation(tmp_path):
    """dtype id 2 decodes as bfloat16; a section cut short ends the scan."""
    vals = torch.tensor([1.5, -2.0, 0.1, 3.0e4])
    bf = vals.bfloat16().view(torch.int16).numpy().astype("<u2").tobytes()
    meta = W.SpiderWMeta(1, 0, 1, 4, 1, 1, 1, 1, 1, 4, 0, 0)
    head = bytearray(W.HEADER_SIZE)
    head[:8] = W.MAGIC
    struct.pack_into("<12I", head, 8, *(getattr(meta, f) for f in W._META_FIELDS))
    body = _section(31, 2, bf, (4,)) + _section(30, 0, np.ones(4, np.float32).tobytes(), (4,))
    p = tmp_path / "bf16.spiderw"
    p.write_bytes(bytes(head) + body[:-3])   # the router section is truncated
    b = W.load_spiderw(p)
    assert torch.equal(torch.from_numpy(np.array(b.tensors["loop_bias"])), vals.bfloat16().float())
    assert "router" not in b.tensors
    bad = tmp_path / "bad.spiderw"
    bad.write_bytes(b"NOTSPIDR" + bytes(72))
    with pytest.raises(ValueError):
        W.load_spiderw(bad)
