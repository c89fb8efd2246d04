"""Model configuration for the recurrent Spider-MoE block.

Mirrors ``ModelConfig`` of the reference (spider_moe/config.py:5-52) field for
field, so a reference config object (or a YAML file in the reference format,
spider_moe/config.py:73-77) can be handed to this package unchanged.  Only the
fields the recurrent block reads matter here; the others are carried so that
``ModelConfig(**yaml["model"])`` keeps working.

Two fields are added for the B200 path and default to the reference behaviour:

* ``expert_activation``: ``"gelu"`` (reference: Linear -> erf-GELU -> Linear
  with biases, spider_moe/model.py:177-183) or ``"swiglu"`` (an extra mode:
  ``down(silu(gate(x)) * up(x))``, gate/up/down all with biases).
* ``expert_weight_format``: ``"native"`` (the module's own dtype), ``"bf16"``,
  ``"fp8"`` (e4m3 with per-output-channel fp32 scales) or ``"int4"``
  (symmetric group-wise, the format of spider_moe/quant.py:89-117).
"""
from __future__ import annotations

from dataclasses import dataclass, asdict
from pathlib import Path


@dataclass
class ModelConfig:
    vocab_size: int = 32000
    hidden_size: int = 256
    num_heads: int = 8
    num_experts: int = 8
    top_k: int = 2
    edges_per_expert: int = 3
    num_loops: int = 6
    num_prelude_layers: int = 2
    num_coda_layers: int = 2
    expert_ffn_size: int = 512
    loop_embed_size: int = 32
    residual_scale: float = 0.5
    re_inject_weight: float = 0.1
    early_exit_threshold: float = 0.85
    dropout: float = 0.0
    embedding_init_std: float = 0.02
    max_seq_len: int = 2048
    use_rope: bool = True
    rope_theta: float = 10000.0
    expert_parallel: bool = True
    offload_experts: bool = False
    offload_max_gpu_experts: int = 4
    use_lumen: bool = False
    lumen_slots: int = 8
    lumen_slot_dim: int = 0
    lumen_j_lens: bool = True
    moe_int4: bool = False
    moe_int4_group_size: int = 64
    # B200 additions (defaults reproduce the reference block).
    expert_activation: str = "gelu"
    expert_weight_format: str = "native"

    def validate(self):
        """Same checks as the reference (spider_moe/config.py:40-52) plus the B200 fields."""
        if self.hidden_size % self.num_heads:
            raise ValueError("hidden_size must be divisible by num_heads")
        if not 1 <= self.top_k <= self.num_experts:
            raise ValueError("top_k must be in [1, num_experts]")
        if not 1 <= self.edges_per_expert <= self.num_experts:
            raise ValueError("edges_per_expert must be in [1, num_experts]")
        if self.num_loops < 1:
            raise ValueError("num_loops must be >= 1")
        if self.embedding_init_std <= 0:
            raise ValueError("embedding_init_std must be > 0")
        if self.expert_activation not in ("gelu", "swiglu"):
            raise ValueError("expert_activation must be 'gelu' or 'swiglu'")
        if self.expert_weight_format not in ("native", "bf16", "fp8", "int4"):
            raise ValueError("expert_weight_format must be native|bf16|fp8|int4")
        return self

    def to_dict(self):
        return asdict(self)


def from_any(cfg) -> ModelConfig:
    """Accept this package's ModelConfig, a reference ModelConfig or a dict."""
    if isinstance(cfg, ModelConfig):
        return cfg
    if isinstance(cfg, dict):
        return ModelConfig(**cfg).validate()
    fields = ModelConfig.__dataclass_fields__
    return ModelConfig(**{k: getattr(cfg, k) for k in fields if hasattr(cfg, k)}).validate()


def load_config(path) -> ModelConfig:
    """Load the ``model:`` section of a reference-format YAML file."""
    import yaml

    raw = yaml.safe_load(Path(path).read_text()) or {}
    return ModelConfig(**raw.get("model", {})).validate()


def benchmark_configs() -> dict:
    """The five workloads the block is measured and checked on.

    cfg1: README smoke model, fp32 (the full reference LM feeds the block).
    cfg2: bf16 decode, 64 tokens.  cfg3: bf16 prefill, 8192 tokens, Zipf bias.
    cfg4: fp8 experts, 64 experts, 4096 tokens.  cfg5: int4 experts, 128
    experts, 256 tokens, Zipf bias.

    ``activation`` is the expert FFN the workload names: cfg1 is the
    reference's own model (erf-GELU, spider_moe/model.py:177-183); cfg2 and
    cfg3 are stated as SwiGLU blocks, and the quantised cfg4 / cfg5 experts
    are SwiGLU FFNs in the fp8 / int4 formats.  ``model`` holds only reference
    ``ModelConfig`` fields, so a test can run any workload in either mode.
    """
    return {
        "cfg1": dict(model=dict(vocab_size=512, hidden_size=64, num_heads=4, num_experts=4,
                                top_k=2, edges_per_expert=2, num_loops=2, expert_ffn_size=128),
                     tokens=64, dtype="fp32", wfmt="native", zipf=False, activation="gelu"),
        "cfg2": dict(model=dict(hidden_size=1024, num_heads=8, num_experts=16, top_k=2,
                                edges_per_expert=2, num_loops=6, expert_ffn_size=2048),
                     tokens=64, dtype="bf16", wfmt="bf16", zipf=False, activation="swiglu"),
        "cfg3": dict(model=dict(hidden_size=1024, num_heads=8, num_experts=16, top_k=2,
                                edges_per_expert=2, num_loops=6, expert_ffn_size=2048),
                     tokens=8192, dtype="bf16", wfmt="bf16", zipf=True, activation="swiglu"),
        "cfg4": dict(model=dict(hidden_size=2048, num_heads=8, num_experts=64, top_k=4,
                                edges_per_expert=3, num_loops=6, expert_ffn_size=1024),
                     tokens=4096, dtype="bf16", wfmt="fp8", zipf=False, activation="swiglu"),
        "cfg5": dict(model=dict(hidden_size=2048, num_heads=8, num_experts=128, top_k=8,
                                edges_per_expert=4, num_loops=4, expert_ffn_size=768,
                                moe_int4_group_size=128),
                     tokens=256, dtype="bf16", wfmt="int4", zipf=True, activation="swiglu"),
    }
