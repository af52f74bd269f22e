"""Regenerate the golden fixtures of tests/golden/ from the reference checkout.

Run where a reference checkout exists, with PRAG_REFERENCE naming its
implementation_v1/ directory (required; there is no default path); the fixtures are
committed so hosts without a reference checkout can use them.

* art002_context.json -- the parameter known answers of IV1/artifacts/bfv_context.json
  (ART-002 primes, Q and bit sizes per level), copied as data.
* kat_linear.json -- the plaintext known answers of the reference's end-to-end probes.
  The probes compute their expected value inline as a ring-59 dot product of
  deterministic integer operands (dev_bfv_packed_probe.cpp:35-53,
  dev_bfv_merged_probe.cpp:66-97, dev_tile_long_probe.cpp:270-301 -- file lines of
  those probes); the operand generators are restated below and the expected values
  recomputed, with each case's public schedule (capacity, groups, callbacks).
* packing_kats.json -- matrix_packing decisions (the oracle's restatement of
  bfv_layout.hpp:14-27) for the Qwen3-0.6B projection shapes at B in {1,16}, the
  attention cross-term shapes and edge shapes.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("PRAG_REFERENCE", "")
MASK = (1 << 59) - 1
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "privacy-rag_b200"))


def context_fixture():
    src = os.path.join(REF, "artifacts", "bfv_context.json")
    with open(src) as f:
        ctx = json.load(f)
    out = {"source": "implementation_v1/artifacts/bfv_context.json", "polynomial_degree": ctx["polynomial_degree"],
           "plaintext_modulus": ctx["plaintext_modulus"],
           "levels": [{"chain_index": lv["chain_index"], "key_level": lv["key_level"], "primes": lv["primes"],
                       "Q": lv["Q"], "Q_bits": lv["Q_bits"]} for lv in ctx["levels"]]}
    with open(os.path.join(HERE, "art002_context.json"), "w") as f:
        json.dump(out, f, indent=1)


def whole_packed(j):
    return (((j * 13 + 7) % 101) - 50) & MASK


def client_share(j):
    return (0x1928abcdef + j * 125939) & MASK


def packed_weight(row, rows, j):
    return 0 if row in (1, rows - 1) else ((((j * (row + 3) + 5) % 17) - 8) & MASK)


def merged_whole(case_id, j):
    if case_id == 1:
        return 7 if j in (0, 8192) else 0
    return whole_packed(j)


def merged_weight(case_id, row, j):
    if case_id < 2 and row == 1:
        return 0
    if case_id == 1:
        if row == 0:
            return 11 if j == 0 else ((-11) & MASK if j == 8192 else 0)
        return 3 if j == 0 else ((-5) & MASK if j == 8192 else 0)
    return ((((j * (row + 3) + 5) % 17) - 8) & MASK)


def expected(columns, rows, whole, weight):
    out = [0] * rows
    for j in range(columns):
        w = whole(j)
        if w == 0:
            continue
        for r in range(rows):
            out[r] = (out[r] + w * weight(r, j)) & MASK
    return out


def kat_fixture():
    from bfvgpu.layout import packed_bfv_rows_per_ciphertext
    cases = []
    # dev_bfv_packed_probe.cpp:35-53
    for d, rows in ((4096, 3), (2730, 4)):
        cases.append({"probe": "dev_bfv_packed_probe", "columns": d, "rows": rows,
                      "capacity": packed_bfv_rows_per_ciphertext(d),
                      "generator": "packed", "expected": expected(d, rows, whole_packed,
                                                                   lambda r, j, rows=rows: packed_weight(r, rows, j))})
    # dev_bfv_merged_probe.cpp:66-97 (rows 3,3,1; 26 callbacks)
    for case_id, (cols, rows) in enumerate(((3, 3), (8193, 3), (19 * 8192, 1))):
        d = min(8192, cols)
        cases.append({"probe": "dev_bfv_merged_probe", "case_id": case_id, "columns": cols, "rows": rows,
                      "capacity": packed_bfv_rows_per_ciphertext(d), "generator": "merged",
                      "expected": expected(cols, rows, lambda j, c=case_id: merged_whole(c, j),
                                           lambda r, j, c=case_id: merged_weight(c, r, j))})
    # dev_tile_long_probe.cpp (rows 3,513,1; 1046 callbacks)
    for case_id, (cols, rows) in enumerate(((3, 3), (8193, 513), (19 * 8192, 1))):
        cases.append({"probe": "dev_tile_long_probe", "case_id": case_id, "columns": cols, "rows": rows,
                      "generator": "merged",
                      "expected": expected(cols, rows, lambda j, c=case_id: merged_whole(c, j),
                                           lambda r, j, c=case_id: merged_weight(c, r, j))})
    with open(os.path.join(HERE, "kat_linear.json"), "w") as f:
        json.dump({"client_share": "(0x1928abcdef + j*125939) mod 2^59", "cases": cases}, f, indent=1)


def packing_fixture():
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
    from oracle import matrix_packing  # the C restatement of bfv_layout.hpp:14-27
    shapes = [(b, k, o) for b in (1, 16) for (k, o) in ((1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072),
                                                          (3072, 1024), (1024, 4096), (1024, 6144))]
    shapes += [(16, 128, 1280), (16, 1280, 128), (1, 17, 1), (1, 8192, 155648), (3, 1000, 77)]
    out = []
    for b, k, o in shapes:
        p = matrix_packing(b, k, o)
        out.append({"b": b, "k": k, "o": o, "reduction": p.reduction, "columns": p.columns, "returns": p.returns,
                    "inputs": p.inputs})
    with open(os.path.join(HERE, "packing_kats.json"), "w") as f:
        json.dump({"rule": "implementation_v1/native/include/prag/bfv_layout.hpp:14-27", "cases": out}, f, indent=1)


if __name__ == "__main__":
    if REF and os.path.exists(REF):
        context_fixture()
    else:
        print("PRAG_REFERENCE unset or missing: art002_context.json left as committed", file=sys.stderr)
    kat_fixture()
    packing_fixture()
    print("golden fixtures written to", HERE)
