"""B200-native recurrent Spider-MoE block (forward pass).

A drop-in for the reference block ``SpiderMoELayer`` (spider_moe/model.py:163)
and its ``sparse_expert_delta`` / ``expert_parallel`` helpers.  The compute
runs in hand-written sm_100a CUDA kernels behind a C ABI
(``include/spider_b200.h``); Python holds device memory, streams and
``torch.distributed``.  Submodules are imported lazily so that the config and
the synthetic-data helpers load without the CUDA library.
"""
from .config import ModelConfig, load_config  # noqa: F401

__all__ = ["ModelConfig", "load_config", "SpiderMoELayer", "sparse_expert_delta"]


def __getattr__(name):
    if name == "SpiderMoELayer":
        from .layer import SpiderMoELayer
        return SpiderMoELayer
    if name == "sparse_expert_delta":
        from .sparse_experts import sparse_expert_delta
        return sparse_expert_delta
    raise AttributeError(name)
