"""Private-weight ingestion (bfvgpu.weights) against the reference's quantized f12 format
(IV1/model_tools/quantize_weights.py): manifest checks, int32 NPY tensors, joint row
stacking in call order (joint_matrix.hpp: q|k|v, gate|up), ring-59 words, shards, and the
packing of the stacked rows."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "privacy-rag_b200"))

from bfvgpu import layer as L  # noqa: E402
from bfvgpu import shard as S  # noqa: E402
from bfvgpu import weights as W  # noqa: E402

SHAPES = {"self_attn.q_proj": (2048, 1024), "self_attn.k_proj": (1024, 1024), "self_attn.v_proj": (1024, 1024),
          "self_attn.o_proj": (1024, 2048), "mlp.gate_proj": (3072, 1024), "mlp.up_proj": (3072, 1024),
          "mlp.down_proj": (1024, 3072)}


def write_layer(directory, layer=0, seed=0, manifest_patch=None):
    """A quantized_f12 directory holding decoder layer `layer` (random f12 values with the
    domain edges +-256*4096 and -1 planted)."""
    rng = np.random.default_rng(seed)
    tensors, mats = [], {}
    for part, shape in SHAPES.items():
        name = f"model.layers.{layer}.{part}.weight"
        a = rng.integers(-W.DOMAIN_ABS, W.DOMAIN_ABS + 1, size=shape).astype("<i4")
        a[0, 0], a[0, 1], a[-1, -1] = W.DOMAIN_ABS, -W.DOMAIN_ABS, -1
        np.save(os.path.join(directory, name + ".npy"), a)
        tensors.append({"name": name, "shape": list(shape), "path": name + ".npy"})
        mats[part] = a
    manifest = {"format_version": W.FORMAT, "fractional_bits": 12, "stored_dtype": "little_endian_int32",
                "semantic_ring_bits": 59, "tensors": tensors}
    manifest.update(manifest_patch or {})
    with open(os.path.join(directory, "manifest.json"), "w") as f:
        json.dump(manifest, f)
    return mats


def test_layer_calls_and_ring_words(tmp_path):
    mats = write_layer(str(tmp_path))
    qw = W.QuantizedWeights(str(tmp_path))
    calls = qw.layer_calls(0)
    assert [c for c, _ in calls] == ["qkv", "o", "gate_up", "down"]
    qkv = W.ring_words(calls[0][1])
    stacked = np.vstack([mats["self_attn.q_proj"], mats["self_attn.k_proj"], mats["self_attn.v_proj"]])
    assert qkv.shape == (4096, 1024)
    assert np.array_equal(qkv, stacked.astype(np.int64) & ((1 << 59) - 1))
    assert qkv[0, 1] == (1 << 59) - W.DOMAIN_ABS and qkv[-1, -1] == (1 << 59) - 1
    # a shard crossing the q/k boundary
    part = W.ring_words(calls[0][1], rows=(2000, 2100))
    assert np.array_equal(part, qkv[2000:2100])


def test_format_rejections(tmp_path):
    write_layer(str(tmp_path), manifest_patch={"fractional_bits": 16})
    with pytest.raises(W.WeightFormatError):
        W.QuantizedWeights(str(tmp_path))
    write_layer(str(tmp_path))
    qw = W.QuantizedWeights(str(tmp_path))
    with pytest.raises(W.WeightFormatError):
        qw.matrix("model.layers.1.self_attn.q_proj.weight")  # absent
    bad = np.zeros((3, 3), dtype="<i4")
    bad[1, 1] = W.DOMAIN_ABS + 1
    with pytest.raises(W.WeightFormatError):
        W.ring_words([bad])
    name = "model.layers.0.self_attn.o_proj.weight"
    np.save(os.path.join(str(tmp_path), name + ".npy"), np.zeros((1024, 2047), dtype="<i4"))
    with pytest.raises(W.WeightFormatError):
        qw.matrix(name)


def test_sharded_packing_matches_whole_call(tmp_path):
    """Each rank's rows of the gate|up call pack into exactly its groups of the whole call."""
    import torch
    write_layer(str(tmp_path), seed=3)
    qw = W.QuantizedWeights(str(tmp_path))
    mats = dict(qw.layer_calls(0))["gate_up"]
    p = L.plan("gate_up", 16, 1024, 6144)
    full = L.pack_weights_device(torch, torch.from_numpy(W.ring_words(mats)), p, 16384)
    for r in range(3):
        sp, lo, hi = S.shard_projection(p, r, 3)
        rows = (lo * p.cap, min(hi * p.cap, p.outputs))
        part = L.pack_weights_device(torch, torch.from_numpy(W.ring_words(mats, rows)), sp, 16384)
        assert torch.equal(part, full[lo:hi])
