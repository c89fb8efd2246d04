"""Named backend registry (the reference's spider_infer/backends, registry.py:8-22).

``spider_b200`` builds the recurrent block on the B200 kernels; a reference
deployment registers the same builder in its own registry, under the same name.
"""
from .registry import get_backend, list_backends, register  # noqa: F401
from . import spider_b200 as _spider_b200  # noqa: F401

__all__ = ["get_backend", "list_backends", "register"]
