""".spiderw native weight bundles (reference: spider_infer/orbit/weight_loader.py,
docs/NATIVE_WEIGHT_FORMAT.md) and loading them into the block's device layouts.

The file format is fixed by the reference, so header, section mini-header,
section ids and dtype ids are the same; the code is this package's own:

* ``load_spiderw`` maps the file (``numpy.memmap``) and returns views of the
  sections without copying them; ``SpiderWMeta`` / ``SpiderWBundle`` have the
  reference's fields and ``require``;
* dtype id 2 is decoded as bfloat16 (the reference reads it as float16);
* ``write_spiderw`` writes what the reference's writer writes;
* ``block_state_dict`` turns a bundle into SpiderMoELayer parameter names
  (model.py:165-216) -- the format stores the router as [H, E], experts as
  up [E, H, U] / down [E, U, H] and no biases, so the transposes are views and
  the missing biases zeros;
* ``SpiderMoELayer.from_spiderw`` / ``BlockEngine.from_spiderw`` copy each
  section to the device once (pinned staging, one copy per section) and let
  the engine pack from device views, so the [E, H, U] -> [E, U, H] transposes
  run on the GPU.

Named sections (id 200) are copied out of the mapping, since their payload
follows a name of any length and need not be aligned.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

MAGIC = b"SPIDERW1"
HEADER_SIZE = 80
SECTION_HEADER = 36          # uint32 id, uint32 dtype, uint64 nbytes, uint32 rank, uint32 dims[4]
SECTION_NAMED = 200
SECTION_NAMES = {1: "token_emb", 2: "lm_head", 30: "router", 31: "loop_bias", 32: "loop_embedding",
                 33: "edge_generator", 34: "edge_value", 35: "expert_up", 36: "expert_down", 37: "moe_norm",
                 38: "exit_head", 40: "csr_row_ptr", 41: "csr_col_idx", 42: "csr_edge_w"}
SECTION_IDS = {v: k for k, v in SECTION_NAMES.items()}
_BF16 = np.dtype(np.uint16)  # bf16 bytes, widened to float32 on decode
DTYPES = {0: np.dtype(np.float32), 1: np.dtype(np.float16), 2: _BF16, 3: np.dtype(np.int32), 4: np.dtype(np.int8)}
FLAG_FP16, FLAG_CSR, FLAG_TIED = 1, 2, 4
_META_FIELDS = ("version", "flags", "vocab_size", "hidden_size", "num_heads", "num_experts", "top_k",
                "edges_per_expert", "num_loops", "expert_ffn_size", "num_prelude_layers", "num_coda_layers")


@dataclass
class SpiderWMeta:
    version: int
    flags: int
    vocab_size: int
    hidden_size: int
    num_heads: int
    num_experts: int
    top_k: int
    edges_per_expert: int
    num_loops: int
    expert_ffn_size: int
    num_prelude_layers: int
    num_coda_layers: int

    @property
    def fp16_weights(self) -> bool:
        return bool(self.flags & FLAG_FP16)

    @property
    def has_csr(self) -> bool:
        return bool(self.flags & FLAG_CSR)

    @property
    def tied_embeddings(self) -> bool:
        return bool(self.flags & FLAG_TIED)


@dataclass
class SpiderWBundle:
    meta: SpiderWMeta
    tensors: dict = field(default_factory=dict)
    csr: dict | None = None
    path: str | None = None

    def require(self, name: str) -> np.ndarray:
        if name not in self.tensors:
            raise KeyError(f"missing section {name}")
        return self.tensors[name]


def _bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def _parse(buf: np.ndarray) -> tuple[SpiderWMeta, dict]:
    raw = buf.tobytes() if buf.size < HEADER_SIZE else bytes(buf[:HEADER_SIZE])
    if len(raw) < HEADER_SIZE:
        raise ValueError("file too small for spiderw header")
    if raw[:8] != MAGIC:
        raise ValueError(f"bad magic: {raw[:8]!r}")
    meta = SpiderWMeta(*struct.unpack_from("<12I", raw, 8))
    tensors = {}
    off, end = HEADER_SIZE, buf.size
    # sections until the data ends; a truncated trailing section ends the scan
    while off + SECTION_HEADER <= end:
        sid, dt_id, nbytes, rank = struct.unpack_from("<IIQI", bytes(buf[off:off + 20]))
        dims = struct.unpack_from("<4I", bytes(buf[off + 20:off + SECTION_HEADER]))
        off += SECTION_HEADER
        dt = DTYPES.get(dt_id)
        if dt is None or off + nbytes > end:
            break
        body = buf[off:off + nbytes]
        off += int(nbytes)
        if sid == SECTION_NAMED:
            (nlen,) = struct.unpack_from("<H", bytes(body[:2]))
            name = bytes(body[2:2 + nlen]).decode("utf-8")
            body = np.array(body[2 + nlen:])
        else:
            name = SECTION_NAMES.get(sid, f"section_{sid}")
        shape = tuple(d for d in dims[:max(rank, 1)] if d > 0) or (body.size // dt.itemsize,)
        arr = body[: (body.size // dt.itemsize) * dt.itemsize].view(dt).reshape(shape)
        tensors[name] = _bf16_to_f32(arr) if dt_id == 2 else arr
    return meta, tensors


def load_spiderw(path) -> SpiderWBundle:
    """Map a .spiderw file and return its sections (views into the mapping)."""
    path = Path(path)
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    meta, tensors = _parse(buf)
    csr = None
    if meta.has_csr or all(k in tensors for k in ("csr_row_ptr", "csr_col_idx", "csr_edge_w")):
        csr = {"row_ptr": tensors.get("csr_row_ptr"), "col_idx": tensors.get("csr_col_idx"),
               "edge_w": tensors.get("csr_edge_w")}
    if meta.tied_embeddings and "lm_head" not in tensors and "token_emb" in tensors:
        tensors["lm_head"] = tensors["token_emb"]
    return SpiderWBundle(meta=meta, tensors=tensors, csr=csr, path=str(path))


def write_spiderw(path, meta: SpiderWMeta, tensors: dict, section_ids: dict | None = None) -> None:
    """Write a bundle: float32 / float16 / int32 sections as given, anything else
    as float32; known names get their section id, others a named section."""
    ids = dict(SECTION_IDS)
    ids.update(section_ids or {})
    parts = []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        codes = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int32): 3}
        if arr.dtype not in codes:
            arr = np.ascontiguousarray(arr.astype(np.float32))
        dt_id = codes[arr.dtype]
        rank = min(arr.ndim, 4)
        dims = [int(d) for d in arr.shape[:4]] + [1] * (4 - rank)
        payload = arr.tobytes()
        sid = ids.get(name)
        if sid is None:
            nb = name.encode("utf-8")
            payload = struct.pack("<H", len(nb)) + nb + payload
            sid = SECTION_NAMED
        parts += [struct.pack("<IIQI", sid, dt_id, len(payload), rank), struct.pack("<4I", *dims), payload]
    body = b"".join(parts)
    header = bytearray(HEADER_SIZE)
    header[:8] = MAGIC
    struct.pack_into("<12I", header, 8, *(int(getattr(meta, f)) for f in _META_FIELDS))
    struct.pack_into("<QQ", header, 64, 0, len(body))   # header crc unused, payload bytes
    Path(path).write_bytes(bytes(header) + body)


def model_config(meta: SpiderWMeta, **overrides):
    """This package's ModelConfig for the block a bundle describes."""
    from .config import ModelConfig

    kw = dict(vocab_size=meta.vocab_size, hidden_size=meta.hidden_size, num_heads=meta.num_heads,
              num_experts=meta.num_experts, top_k=meta.top_k, edges_per_expert=meta.edges_per_expert,
              num_loops=meta.num_loops, expert_ffn_size=meta.expert_ffn_size)
    kw.update(overrides)
    return ModelConfig(**kw).validate()


def block_state_dict(bundle: SpiderWBundle, device="cpu") -> dict:
    """SpiderMoELayer parameters (reference names) from a bundle's block sections.

    Each section is copied once to an aligned float32 host buffer and from
    there to ``device`` (pinned, for CUDA); router / expert transposes are
    views of those copies and the biases the format does not store are
    zeros."""
    m = bundle.meta
    H, E, U = m.hidden_size, m.num_experts, m.expert_ffn_size
    dev = torch.device(device)

    def put(name):
        t = torch.from_numpy(np.array(bundle.require(name), dtype=np.float32))  # one aligned host copy
        if dev.type == "cuda":
            return t.pin_memory().to(dev, non_blocking=True)
        return t

    zeros = lambda *s: torch.zeros(*s, dtype=torch.float32, device=dev)  # noqa: E731
    sd = {}
    router = put("router")
    sd["router.weight"] = router.t() if tuple(router.shape) == (H, E) and H != E else router
    lb = put("loop_bias")
    sd["loop_bias"] = lb.reshape(1, E).expand(m.num_loops, E).contiguous() if lb.dim() == 1 else lb.reshape(m.num_loops, E)
    sd["loop_embedding.weight"] = put("loop_embedding")
    gen = put("edge_generator")
    sd["edge_generator.weight"] = gen
    sd["edge_generator.bias"] = zeros(E * E)
    edge = put("edge_value").reshape(E, H, H)
    up = put("expert_up").reshape(E, H, U)
    down = put("expert_down").reshape(E, U, H)
    for i in range(E):
        sd[f"edge_value.{i}.weight"] = edge[i]
        sd[f"experts.{i}.0.weight"] = up[i].t()      # [U, H]
        sd[f"experts.{i}.0.bias"] = zeros(U)
        sd[f"experts.{i}.2.weight"] = down[i].t()    # [H, U]
        sd[f"experts.{i}.2.bias"] = zeros(H)
    norm = put("moe_norm")
    if norm.dim() == 1:
        sd["norm.weight"], sd["norm.bias"] = norm, zeros(H)
    else:
        sd["norm.weight"], sd["norm.bias"] = norm[0], norm[1]
    if "exit_head" in bundle.tensors:
        sd["exit_head.weight"] = put("exit_head").reshape(1, H)
    else:
        sd["exit_head.weight"] = zeros(1, H)
    sd["exit_head.bias"] = zeros(1)
    return sd
