"""CUDA-graph decode runner with the reference's interface
(spider_infer/cuda_graph.py:16-130: ``DecodeGraphKey``, ``CudaGraphDecodeRunner``).

A decode callable ``fn(input_ids [B, 1], request_ids) -> logits`` is captured
once per key (batch size, KV-length bucket, loop count) after three warm-up
calls and replayed afterwards; calls that cannot be replayed (not on CUDA, more
than one new token, request ids other than the captured ones) run eagerly and
count as fallbacks.  Early exit has a data-dependent active set and is not
captured, as in the reference.

Every call this package makes on the decode path is capturable: the block
kernels are enqueued on the caller's current stream, their scratch lives in
workspaces allocated before capture (during warm-up), and nothing reads device
memory back on the host.  A replay of the recurrent block therefore runs as one
graph of the library's kernels, with the programmatic-dependent-launch edges
between them preserved.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class DecodeGraphKey:
    """Graph identity: active batch size, KV length bucket, loop count."""

    batch_size: int
    length_bucket: int
    num_loops: int = 1


@dataclass
class _Captured:
    graph: torch.cuda.CUDAGraph
    ids: torch.Tensor
    logits: torch.Tensor
    request_ids: list


class CudaGraphDecodeRunner:
    """Capture and replay a static-shape decode step (reference cuda_graph.py:28-130)."""

    def __init__(self, enabled: bool = True, length_bucket_size: int = 64, warmup: int = 3):
        self.enabled = bool(enabled) and torch.cuda.is_available()
        self.length_bucket_size = int(length_bucket_size)
        self.warmup = int(warmup)
        self._cap: dict[DecodeGraphKey, _Captured] = {}
        self.hits = self.misses = self.fallbacks = 0

    def _bucket(self, length: int) -> int:
        b = self.length_bucket_size
        return -(-int(length) // b) * b

    def clear(self) -> None:
        self._cap.clear()
        self.hits = self.misses = self.fallbacks = 0

    def stats(self) -> dict:
        return {
            "enabled": self.enabled,
            "graphs": len(self._cap),
            "hits": self.hits,
            "misses": self.misses,
            "fallbacks": self.fallbacks,
            "keys": [{"batch_size": k.batch_size, "length_bucket": k.length_bucket, "num_loops": k.num_loops}
                     for k in self._cap],
        }

    def run(self, fn: Callable, input_ids: torch.Tensor, request_ids: list, cache_length: int,
            num_loops: int = 1) -> torch.Tensor:
        """fn(input_ids, request_ids) -> logits, replayed from a graph when the key was captured."""
        if not self.enabled or input_ids.device.type != "cuda" or input_ids.dim() < 2 or input_ids.shape[1] != 1:
            self.fallbacks += 1
            return fn(input_ids, request_ids)
        key = DecodeGraphKey(int(input_ids.shape[0]), self._bucket(cache_length), max(1, int(num_loops)))
        cap = self._cap.get(key)
        if cap is None:
            self.misses += 1
            for _ in range(self.warmup):  # workspaces and engines exist before capture
                fn(input_ids, request_ids)
            torch.cuda.synchronize(input_ids.device)
            ids = input_ids.clone()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                logits = fn(ids, request_ids)
            self._cap[key] = _Captured(graph, ids, logits, list(request_ids))
            graph.replay()  # the captured run produced no values: compute this call's
            return logits.clone()
        if list(request_ids) != cap.request_ids:  # page tables were captured for those requests
            self.fallbacks += 1
            return fn(input_ids, request_ids)
        self.hits += 1
        cap.ids.copy_(input_ids)
        cap.graph.replay()
        return cap.logits.clone()
