"""GatedDeltaNet decode-step core: the C oracle (a line-by-line restatement of the
reference kernels, metal/kernels.metal:1275-1346, 1780-1873) checked against an
independent vectorised numpy statement of the same math over several steps. No golden
vectors exist for this path (the reference is Metal-only), so this pins the restatement
against a second one, not against the reference itself."""
import numpy as np

from oracle import oracle as O


def numpy_step(w, inp, conv, S):
    cw = O.bf16_to_f32(w["conv_w"]).astype(np.float64)
    x = inp["qkv"].astype(np.float64)
    acc = conv[0] * cw[:, 0] + conv[1] * cw[:, 1] + conv[2] * cw[:, 2] + x * cw[:, 3]
    cv = acc / (1 + np.exp(-acc))
    conv[0], conv[1], conv[2] = conv[1].copy(), conv[2].copy(), x
    q = cv[:2048].reshape(16, 128)
    k = cv[2048:4096].reshape(16, 128)
    v = cv[4096:].reshape(32, 128)
    inv = 1 / np.sqrt(128)
    q = q / np.sqrt((q * q).mean(1, keepdims=True) + 1e-12) * inv * inv
    k = k / np.sqrt((k * k).mean(1, keepdims=True) + 1e-12) * inv
    A = np.exp(w["A_log"].astype(np.float64))
    sp = np.log1p(np.exp(inp["alpha"] + O.bf16_to_f32(w["dt_bias"])))
    g = np.exp(-A * sp)
    b = 1 / (1 + np.exp(-inp["beta"].astype(np.float64)))
    out = np.zeros((32, 128))
    for vh in range(32):
        kh = vh // 2
        Sh = S[vh] * g[vh]
        d = (v[vh] - Sh @ k[kh]) * b[vh]
        Sh = Sh + np.outer(d, k[kh])
        S[vh] = Sh
        o = Sh @ q[kh]
        o = o / np.sqrt((o * o).mean() + 1e-6)
        z = inp["z"].reshape(32, 128)[vh].astype(np.float64)
        out[vh] = o * z / (1 + np.exp(-z)) * O.bf16_to_f32(w["norm_w"])
    return out.reshape(-1)


def test_oracle_matches_numpy_over_steps():
    w = O.make_linear_attn(3)
    rng = np.random.default_rng(4)
    conv = np.zeros((3, 8192), np.float32)
    S = np.zeros((32, 128, 128), np.float32)
    conv64 = np.zeros((3, 8192))
    S64 = np.zeros((32, 128, 128))
    for step in range(4):
        inp = O.linear_attn_inputs(rng)
        out = O.linear_attn_step(w, inp, conv, S)
        ref = numpy_step(w, inp, conv64, S64)
        assert np.abs(out - ref).max() <= 2e-5 * np.abs(ref).max(), step
        assert np.abs(S - S64).max() <= 2e-5 * max(np.abs(S64).max(), 1e-6), step
        assert np.array_equal(conv, conv64.astype(np.float32))
