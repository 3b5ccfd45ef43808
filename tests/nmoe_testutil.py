"""Shared helpers for the GPU tests: upload oracle-generated layers into a Context."""
import numpy as np

import nmoe_b200 as N
from oracle import oracle as O


def upload(ctx: "N.Context", layer_idx: int, lw: "O.LayerWeights"):
    ctx.load_layer(layer_idx, lw.experts)
    ctx.set_dense(layer_idx, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_round(x: np.ndarray) -> np.ndarray:
    return O.bf16_to_f32(O.f32_to_bf16(x))


_distinct = {}


def distinct_layer(bits: int = 4) -> "O.LayerWeights":
    """One layer whose 256 expert slots all hold different packs (no e % n reuse), so a
    kernel that reads the wrong slot cannot match the oracle by accident. ~20 s of host
    work, built once per process."""
    if bits not in _distinct:
        _distinct[bits] = O.make_layer(9001 + bits, bits=bits, distinct_experts=None)
    return _distinct[bits]
