"""B200-native recurrent Spider-MoE block (forward pass).

A drop-in for the reference block ``SpiderMoELayer`` (spider_moe/model.py:163)
and its ``sparse_expert_delta`` / ``expert_parallel`` helpers.  The compute
runs in hand-written sm_100a CUDA kernels behind a C ABI
(``include/spider_b200.h``); Python holds device memory, streams and
``torch.distributed``.  Submodules are imported lazily so that the config and
the synthetic-data helpers load without the CUDA library.
"""
from .config import ModelConfig, load_config  # noqa: F401

__all__ = ["ModelConfig", "load_config", "SpiderMoELayer", "sparse_expert_delta", "LumenWorkspace",
           "ExpertChunkStore", "CudaGraphDecodeRunner", "load_spiderw", "write_spiderw"]

_LAZY = {
    "SpiderMoELayer": ("layer", "SpiderMoELayer"),
    "sparse_expert_delta": ("sparse_experts", "sparse_expert_delta"),
    "LumenWorkspace": ("lumen", "LumenWorkspace"),
    "ExpertChunkStore": ("dobu", "ExpertChunkStore"),
    "CudaGraphDecodeRunner": ("cuda_graph", "CudaGraphDecodeRunner"),
    "load_spiderw": ("spiderw", "load_spiderw"),
    "write_spiderw": ("spiderw", "write_spiderw"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{mod}", __name__), attr)
    raise AttributeError(name)
