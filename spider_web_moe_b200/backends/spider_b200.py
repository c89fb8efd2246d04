"""``spider_b200`` backend: the recurrent Spider-MoE block on the B200 kernels.

Builder signature of the reference (spider_infer/backends/spider.py:3-6):
``build(model_config, device="cpu", **kwargs) -> nn.Module``.  Given a
``SpiderWebLM`` (``model=``) it swaps the model's ``.recurrent`` block for this
package's drop-in layer with the same weights; otherwise it returns the block.
"""
from __future__ import annotations

from .registry import register


@register("spider_b200")
def build_spider_b200(model_config, device="cuda", model=None, engine="auto", **kwargs):
    from ..layer import SpiderMoELayer

    if model is not None:
        rec = model.recurrent
        layer = SpiderMoELayer(model_config)
        layer.load_state_dict(rec.state_dict(), strict=False)
        layer.engine_name = engine
        model.recurrent = layer.to(device)
        return model.to(device).eval()
    layer = SpiderMoELayer(model_config)
    layer.engine_name = engine
    return layer.to(device).eval()
