"""Private-weight ingestion: the reference's quantized f12 checkpoint directory into the
layer pipeline's ring words and NTT-form plaintexts.

Format (IV1/model_tools/quantize_weights.py:60-107): a directory holding `manifest.json`
(format "quantized-private-weights-v1", 12 fractional bits, little-endian int32 storage,
59-bit semantic ring) and one NPY file per tensor, value floor(x * 4096).  A private matrix
enters the protocol as ring-59 words (two's complement of the f12 integer), the joint calls
of a decoder layer stack the rows of their matrices in call order (private_joint_matrix,
IV1/native/include/prag/joint_matrix.hpp: q|k|v and gate|up), and `Transformer` calls them as
(model.hpp:173-238): qkv joint, o, gate/up joint, down.
"""
from __future__ import annotations

import json
import os

import numpy as np

from .layout import MASK59

FORMAT = "quantized-private-weights-v1"
DOMAIN_ABS = 256 << 12          # quantize_weights.py: |w| <= 256 in f12
LAYER_CALLS = (("qkv", ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")),
               ("o", ("self_attn.o_proj",)),
               ("gate_up", ("mlp.gate_proj", "mlp.up_proj")),
               ("down", ("mlp.down_proj",)))


class WeightFormatError(ValueError):
    """The directory is not a usable quantized f12 weight set (the reference's error names)."""


class QuantizedWeights:
    """Read-only view of a quantized_f12 directory; tensors are memory-mapped on demand."""

    def __init__(self, directory: str):
        self.directory = directory
        with open(os.path.join(directory, "manifest.json")) as f:
            m = json.load(f)
        if m.get("format_version") != FORMAT or m.get("fractional_bits") != 12 or \
                m.get("stored_dtype") != "little_endian_int32" or m.get("semantic_ring_bits") != 59:
            raise WeightFormatError("E_WEIGHT_FORMAT")
        self.manifest = m
        self.tensors = {t["name"]: t for t in m.get("tensors", [])}

    def matrix(self, name: str) -> np.ndarray:
        """Signed f12 integers of tensor `name` (shape and dtype checked against the manifest)."""
        t = self.tensors.get(name)
        if t is None:
            raise WeightFormatError("MODEL_TENSOR_MISSING: " + name)
        a = np.load(os.path.join(self.directory, t["path"]), mmap_mode="r", allow_pickle=False)
        if a.dtype != np.dtype("<i4") or list(a.shape) != list(t["shape"]):
            raise WeightFormatError("MODEL_TENSOR_SHAPE_MISMATCH: " + name)
        return a

    def layer_calls(self, layer: int) -> list:
        """[(call name, [f12 matrices in row order])] for the four calls of decoder layer `layer`."""
        prefix = f"model.layers.{layer}."
        return [(call, [self.matrix(prefix + part + ".weight") for part in parts]) for call, parts in LAYER_CALLS]


def ring_words(mats, rows=None) -> np.ndarray:
    """Row-stacked ring-59 words of the given f12 matrices ([sum rows][K] int64), optionally
    only rows [lo, hi) of the stack (a shard).  Rejects values outside the f12 domain."""
    widths = {m.shape[1] for m in mats}
    if len(widths) != 1:
        raise WeightFormatError("E_JOINT_SHAPE")
    total = sum(m.shape[0] for m in mats)
    lo, hi = rows if rows is not None else (0, total)
    out = np.empty((hi - lo, widths.pop()), dtype=np.int64)
    offset, w = 0, 0
    for m in mats:
        a, b = max(lo, offset), min(hi, offset + m.shape[0])
        if a < b:
            part = np.asarray(m[a - offset:b - offset], dtype=np.int64)
            if part.size and (part.min() < -DOMAIN_ABS or part.max() > DOMAIN_ABS):
                raise WeightFormatError("E_WEIGHT_BOUND")
            out[w:w + (b - a)] = part
            w += b - a
        offset += m.shape[0]
    return out & MASK59
