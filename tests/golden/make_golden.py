#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference tree (default /root/reference, override
with NMOE_REF_ROOT) and the reference's math.m built by `make -C oracle ref`:

    python tests/golden/make_golden.py

Outputs (committed; small):
  golden_quant.npz  -- inputs and outputs of the reference quantiser
                       (scripts/convert_qwen36.py: quantize_rows_bf16 py:195-211,
                       quantize_rows_bf16_2bit py:167-183, pack_4bit/pack_2bit) on
                       seeded rows plus hand-built edge rows (constant groups, exact
                       half-step ties, signed zeros, large magnitudes).
  golden_math.npz   -- the reference's src/math.m (compiled unchanged as C) on seeded
                       inputs: softmax (math.m:67-93), top-k (95-132), renormalise
                       (134-153), dequant matvec (236-274), sigmoid (21-28).
  golden_meta.json  -- sha256 of full expert blobs assembled with the reference's
                       EXPERT_LAYOUT (py:38-64) and write_expert_component (py:334-336)
                       from seeded bf16 weights, for q4 and q2.

Nothing at test time reads the reference tree: tests read only these files.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("NMOE_REF_ROOT", "/root/reference")
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402


def load_converter():
    path = os.path.join(REF_ROOT, "scripts", "convert_qwen36.py")
    spec = importlib.util.spec_from_file_location("nmoe_ref_convert", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def edge_rows(in_dim: int) -> np.ndarray:
    """Rows that exercise the quantiser's corner cases (all values are bf16)."""
    rows = []
    # 1. constant groups (scale == 0 -> safe_scale 1)
    rows.append(np.full(in_dim, 0.0123, np.float32))
    # 2. exact half-step ties: group spans [0, 15*0.5]; values at (j+0.5)*0.5 -> rint ties
    g = np.arange(64, dtype=np.float32) % 16
    r = np.tile((np.minimum(g, 15) * 0.5 + np.where(g % 2 == 0, 0.25, 0.0)).astype(np.float32), in_dim // 64)
    r[::64] = 0.0
    r[1::64] = 7.5
    rows.append(r)
    # 3. signed zeros and a single non-zero per group
    z = np.zeros(in_dim, np.float32)
    z[::2] = -0.0
    z[5::64] = 1.0
    rows.append(z)
    # 4. large magnitudes
    rows.append(np.linspace(-3.0e4, 3.0e4, in_dim, dtype=np.float32))
    # 5. all negative
    rows.append(-np.abs(np.sin(np.arange(in_dim, dtype=np.float32))) - 0.5)
    return O.f32_to_bf16(np.stack(rows))


def main() -> None:
    conv = load_converter()
    ref = O.ref_lib()
    if ref is None:
        raise SystemExit("build the reference math.m first: make -C oracle ref")
    rng = np.random.default_rng(20261201)

    quant = {}
    for name, in_dim in (("h2048", 2048), ("h512", 512)):
        seeded = O.randn_bf16(rng, (6, in_dim), 0.02)
        wide = O.randn_bf16(rng, (2, in_dim), 1.0)
        rows = np.concatenate([seeded, wide, edge_rows(in_dim)], axis=0)
        quant[f"{name}_rows"] = rows
        for bits, fn in ((4, conv.quantize_rows_bf16), (2, conv.quantize_rows_bf16_2bit)):
            p, s, b = fn(rows)
            quant[f"{name}_q{bits}_packed"] = np.ascontiguousarray(p, np.uint32)
            quant[f"{name}_q{bits}_scales"] = np.ascontiguousarray(s, np.uint16)
            quant[f"{name}_q{bits}_biases"] = np.ascontiguousarray(b, np.uint16)
    np.savez_compressed(os.path.join(HERE, "golden_quant.npz"), **quant)

    # Full expert blobs via the reference's own layout and writer.
    meta = {"generator": "tests/golden/make_golden.py", "seed": 7, "blobs": {}}
    brng = np.random.default_rng(7)
    gu = O.randn_bf16(brng, (1024, 2048), 0.02)
    dn = O.randn_bf16(brng, (2048, 512), 0.02)
    for bits in (4, 2):
        size = conv.EXPERT_SIZE_4BIT if bits == 4 else conv.EXPERT_SIZE_2BIT
        layout = conv.EXPERT_LAYOUT if bits == 4 else conv.EXPERT_LAYOUT_2BIT
        fn = conv.quantize_rows_bf16 if bits == 4 else conv.quantize_rows_bf16_2bit
        blob = bytearray(size)
        for i, mat in enumerate((gu[:512], gu[512:], dn)):
            w, s, b = fn(mat)
            conv.write_expert_component(blob, layout[i * 3][1], w)
            conv.write_expert_component(blob, layout[i * 3 + 1][1], s)
            conv.write_expert_component(blob, layout[i * 3 + 2][1], b)
        meta["blobs"][f"q{bits}"] = {
            "size": size,
            "sha256": hashlib.sha256(bytes(blob)).hexdigest(),
            "layout": [[n, o, z] for n, o, z in layout],
        }

    # math.m on seeded inputs.
    math = {}
    logits = rng.standard_normal((16, 256), dtype=np.float32)
    logits[1, 10] = logits[1, 200] = logits[1].max() + 1.0     # exact tie at the top
    logits[2, :] = 0.5                                          # all equal
    logits[3, 50:60] = logits[3, 50]                            # tie run
    logits[4] *= 40.0                                           # large spread
    math["logits"] = logits
    sm = logits.copy()
    for i in range(sm.shape[0]):
        row = np.ascontiguousarray(sm[i])
        ref.nmoe_cpu_softmax(row, 256)
        sm[i] = row
    math["softmax"] = sm
    topi = np.zeros((16, 8, 8), np.int64)
    topv = np.zeros((16, 8, 8), np.float32)
    renv = np.zeros((16, 8, 8), np.float32)
    for i in range(16):
        for k in range(1, 9):
            idx = np.zeros(k, np.uint64)
            vals = np.zeros(k, np.float32)
            n = ref.nmoe_cpu_topk(np.ascontiguousarray(sm[i]), 256, k, idx, vals)
            assert n == k
            topi[i, k - 1, :k] = idx
            topv[i, k - 1, :k] = vals
            rn = vals.copy()
            ref.nmoe_cpu_renormalize(rn, k)
            renv[i, k - 1, :k] = rn
    math["topk_idx"], math["topk_val"], math["renorm"] = topi, topv, renv
    xs = rng.standard_normal(2048, dtype=np.float32)
    xd = rng.standard_normal(512, dtype=np.float32)
    for bits in (4, 2):
        for name, x in (("h2048", xs), ("h512", xd)):
            p = quant[f"{name}_q{bits}_packed"]
            s = quant[f"{name}_q{bits}_scales"]
            b = quant[f"{name}_q{bits}_biases"]
            y = np.zeros(p.shape[0], np.float32)
            ref.nmoe_cpu_dequant_matvec(p, s, b, x, y, p.shape[0], x.size, bits)
            math[f"matvec_{name}_q{bits}"] = y
    math["x2048"], math["x512"] = xs, xd
    sx = np.linspace(-30, 30, 241, dtype=np.float32)
    math["sigmoid_x"] = sx
    math["sigmoid"] = np.array([ref.nmoe_cpu_sigmoid(float(v)) for v in sx], np.float32)
    np.savez_compressed(os.path.join(HERE, "golden_math.npz"), **math)

    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote golden_quant.npz, golden_math.npz, golden_meta.json")


if __name__ == "__main__":
    main()
