"""The CPU oracle against the reference: golden fixtures (reference quantiser and the
reference's src/math.m) and, where it was built, the live reference math library."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gq():
    return np.load(os.path.join(GOLD, "golden_quant.npz"))


@pytest.fixture(scope="module")
def gm():
    return np.load(os.path.join(GOLD, "golden_math.npz"))


@pytest.mark.parametrize("name", ["h2048", "h512"])
@pytest.mark.parametrize("bits", [4, 2])
def test_quantiser_matches_reference(gq, name, bits):
    rows = gq[f"{name}_rows"]
    p, s, b = O.quantize_rows(rows, bits)
    np.testing.assert_array_equal(p, gq[f"{name}_q{bits}_packed"])
    np.testing.assert_array_equal(s, gq[f"{name}_q{bits}_scales"])
    want_b = gq[f"{name}_q{bits}_biases"]
    # numpy's SIMD min reduction picks the sign of a zero minimum by lane order
    # (implementation-defined); +0 and -0 biases dequantise identically, so a zero
    # minimum compares by value. Every other bias compares bit-exactly.
    both_zero = ((b & 0x7FFF) == 0) & ((want_b & 0x7FFF) == 0)
    np.testing.assert_array_equal(np.where(both_zero, 0, b), np.where(both_zero, 0, want_b))
    assert both_zero.sum() <= 2 * b.shape[1]  # only the two edge rows with zero minima


@pytest.mark.parametrize("bits", [4, 2])
def test_expert_blob_matches_reference(bits):
    meta = json.load(open(os.path.join(GOLD, "golden_meta.json")))["blobs"][f"q{bits}"]
    assert O.expert_size(bits) == meta["size"]
    assert O.expert_offsets(bits) == [o for _, o, _ in meta["layout"]]
    rng = np.random.default_rng(7)
    gu = O.randn_bf16(rng, (1024, 2048), 0.02)
    dn = O.randn_bf16(rng, (2048, 512), 0.02)
    blob = O.pack_expert(gu, dn, bits)
    assert hashlib.sha256(blob.tobytes()).hexdigest() == meta["sha256"]


def test_softmax_topk_renorm_match_reference(gm):
    L = O.lib()
    logits = gm["logits"]
    for i in range(logits.shape[0]):
        p = np.ascontiguousarray(logits[i].copy())
        L.orc_softmax(p, 256)
        np.testing.assert_array_equal(p, gm["softmax"][i])
        for k in range(1, 9):
            idx = np.zeros(k, np.uint32)
            vals = np.zeros(k, np.float32)
            assert L.orc_topk(p, 256, k, idx, vals) == k
            np.testing.assert_array_equal(idx, gm["topk_idx"][i, k - 1, :k])
            np.testing.assert_array_equal(vals, gm["topk_val"][i, k - 1, :k])
            L.orc_renormalize(vals, k)
            np.testing.assert_array_equal(vals, gm["renorm"][i, k - 1, :k])


def test_sigmoid_matches_reference(gm):
    got = np.array([O.lib().orc_sigmoid_cpu(float(v)) for v in gm["sigmoid_x"]], np.float32)
    np.testing.assert_array_equal(got, gm["sigmoid"])


@pytest.mark.parametrize("name", ["h2048", "h512"])
@pytest.mark.parametrize("bits", [4, 2])
def test_dequant_matvec_matches_reference(gq, gm, name, bits):
    p = gq[f"{name}_q{bits}_packed"]
    s = gq[f"{name}_q{bits}_scales"]
    b = gq[f"{name}_q{bits}_biases"]
    x = gm["x2048" if name == "h2048" else "x512"]
    y = np.zeros(p.shape[0], np.float32)
    O.lib().orc_dequant_matvec_seq(p, s, b, x, y, p.shape[0], x.size, bits)
    np.testing.assert_array_equal(y, gm[f"matvec_{name}_q{bits}"])
    # kernel-form (lane-strided) matvecs agree to fp32 rounding
    for form in (0, 1):
        yk = np.zeros_like(y)
        O.lib().orc_dequant_matvec(p, s, b, x, yk, p.shape[0], x.size, bits, form)
        np.testing.assert_allclose(yk, y, rtol=2e-4, atol=2e-3 * np.abs(y).max())


def test_live_reference_math_when_built():
    ref = O.ref_lib()
    if ref is None:
        pytest.skip("reference math.m not built here (oracle/_ref)")
    rng = np.random.default_rng(3)
    for trial in range(50):
        lg = (rng.standard_normal(256) * rng.uniform(0.1, 20)).astype(np.float32)
        if trial % 5 == 0:
            lg[rng.integers(0, 256, 6)] = lg.max()
        a, b = lg.copy(), lg.copy()
        O.lib().orc_softmax(a, 256)
        ref.nmoe_cpu_softmax(b, 256)
        np.testing.assert_array_equal(a, b)
        k = int(rng.integers(1, 9))
        i1 = np.zeros(k, np.uint32)
        v1 = np.zeros(k, np.float32)
        i2 = np.zeros(k, np.uint64)
        v2 = np.zeros(k, np.float32)
        O.lib().orc_topk(a, 256, k, i1, v1)
        ref.nmoe_cpu_topk(b, 256, k, i2, v2)
        np.testing.assert_array_equal(i1, i2.astype(np.uint32))
        np.testing.assert_array_equal(v1, v2)


def _dequant(p, s, b, bits, in_dim):
    vpw = 32 // bits
    mask = (1 << bits) - 1
    q = np.stack([(p >> (bits * i)) & mask for i in range(vpw)], axis=-1).reshape(p.shape[0], in_dim)
    sc = np.repeat(O.bf16_to_f32(s), 64, axis=1)
    bi = np.repeat(O.bf16_to_f32(b), 64, axis=1)
    return q.astype(np.float64) * sc + bi


def _dense(d, in_dim):
    if d["dtype"] == O.DTYPE_BF16:
        return O.bf16_to_f32(d["weight"]).astype(np.float64)
    return _dequant(d["weight"], d["scales"], d["biases"], 4, in_dim)


@pytest.mark.parametrize("bits,rdt", [(4, O.DTYPE_BF16), (4, O.DTYPE_Q4), (2, O.DTYPE_Q4)])
def test_block_forward_matches_float64_restatement(bits, rdt):
    """The whole oracle block against an independent float64 numpy restatement."""
    layer = O.make_layer(11, bits=bits, router_dtype=rdt, shared_dtype=rdt, distinct_experts=4)
    rng = np.random.default_rng(5)
    x = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal(2048, dtype=np.float32)))
    hm = rng.standard_normal(2048, dtype=np.float32)
    k = 8
    r = O.block_forward(layer, k, x, hm)
    xd = x.astype(np.float64)
    logits = _dense(layer.router, 2048) @ xd
    np.testing.assert_allclose(r["logits"], logits, rtol=1e-4, atol=1e-5)
    idx, w = O.route_reference(r["logits"], k)
    np.testing.assert_array_equal(r["idx"][:k], idx)
    np.testing.assert_array_equal(r["w"][:k], w)
    silu = lambda v: v / (1 + np.exp(-v))
    sact = silu(_dense(layer.shared_gate, 2048) @ xd) * (_dense(layer.shared_up, 2048) @ xd)
    score = (_dense(layer.shared_gate_vec, 2048) @ xd)[0]
    out = hm.astype(np.float64) + (1 / (1 + np.exp(-score))) * (_dense(layer.shared_down, 512) @ sact)
    esz = O.expert_size(bits)
    off = O.expert_offsets(bits)
    for s in range(k):
        blob = layer.experts[idx[s] * esz:(idx[s] + 1) * esz]
        def comp(i, dt, n):
            return blob[off[i]:off[i] + n * np.dtype(dt).itemsize].view(dt)
        vpw = 32 // bits
        G = _dequant(comp(0, np.uint32, 512 * 2048 // vpw).reshape(512, -1), comp(1, np.uint16, 512 * 32).reshape(512, 32),
                     comp(2, np.uint16, 512 * 32).reshape(512, 32), bits, 2048)
        U = _dequant(comp(3, np.uint32, 512 * 2048 // vpw).reshape(512, -1), comp(4, np.uint16, 512 * 32).reshape(512, 32),
                     comp(5, np.uint16, 512 * 32).reshape(512, 32), bits, 2048)
        D = _dequant(comp(6, np.uint32, 2048 * 512 // vpw).reshape(2048, -1), comp(7, np.uint16, 2048 * 8).reshape(2048, 8),
                     comp(8, np.uint16, 2048 * 8).reshape(2048, 8), bits, 512)
        act = silu(G @ xd) * (U @ xd)
        out += w[s] * (D @ act)
    rel = np.linalg.norm(r["out"] - out) / np.linalg.norm(out)
    assert rel < 1e-5, rel


def test_block_forward_rejects_bad_k():
    layer = O.make_layer(1, distinct_experts=1)
    x = np.zeros(2048, np.float32)
    for k in (0, 9):
        with pytest.raises(ValueError):
            O.block_forward(layer, k, x)
