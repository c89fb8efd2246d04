"""``spider_b200`` backend: the recurrent Spider-MoE block on the B200 kernels.

Builder signature of the reference (spider_infer/backends/spider.py:3-6):
``build(model_config, device="cpu", **kwargs) -> nn.Module``.  Given a
``SpiderWebLM`` (``model=``) it swaps the model's ``.recurrent`` block for this
package's drop-in layer with the same weights and routes the model's
recurrent drivers (all loops, early-exit decode) to the block's device
drivers; otherwise it returns the block.
"""
from __future__ import annotations

from .registry import register


def _attach_recurrent_drivers(model):
    """Route the model's recurrent drivers to the block's device drivers:
    ``_run_recurrent_full`` (model.py:445-448) runs all loops in one library
    call, ``_run_recurrent_decode`` (model.py:450-473) keeps the early-exit
    active set on the device.  Instance attributes, so the class is untouched."""
    def run_full(h, x0):
        return model.recurrent.run_recurrent_full(h, x0)

    def run_decode(h, x0, early_exit):
        return model.recurrent.run_recurrent_decode(h, x0, early_exit, model.cfg.early_exit_threshold)

    model._run_recurrent_full = run_full
    model._run_recurrent_decode = run_decode


@register("spider_b200")
def build_spider_b200(model_config, device="cuda", model=None, engine="auto", **kwargs):
    from ..layer import SpiderMoELayer

    if model is not None:
        rec = model.recurrent
        layer = SpiderMoELayer(model_config)
        layer.load_state_dict(rec.state_dict(), strict=False)
        layer.engine_name = engine
        if getattr(rec, "lumen", None) is not None and layer.lumen is not None:
            layer.lumen.j_lens = rec.lumen.j_lens  # the model's J-lens head (model.py:365-371)
        model.recurrent = layer.to(device)
        _attach_recurrent_drivers(model)
        return model.to(device).eval()
    layer = SpiderMoELayer(model_config)
    layer.engine_name = engine
    return layer.to(device).eval()
