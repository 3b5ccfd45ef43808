"""Full-attention decode step: the C oracle (restating metal/kernels.metal:1006-1058 and
1119-1194 in the order of src/runtime.m:3040-3095) checked against an independent float64
numpy statement. No golden vectors exist (Metal only): parity against the reference
itself is unpinned; this pins the restatement against a second one."""
import numpy as np

from oracle import oracle as O


def np_prep(v, w, pos):
    v = v.astype(np.float64)
    v = v / np.sqrt((v * v).mean() + 1e-6) * (O.bf16_to_f32(w).astype(np.float64) + 1)
    t = np.arange(32)
    ang = pos * (1e7 ** (-2.0 * t / 64))
    c, s = np.cos(ang), np.sin(ang)
    v0, v1 = v[:32].copy(), v[32:64].copy()
    v[:32] = v0 * c - v1 * s
    v[32:64] = v0 * s + v1 * c
    return v


def test_oracle_matches_numpy():
    rng = np.random.default_rng(5)
    qn = O.randn_bf16(rng, (256,), 0.1)
    kn = O.randn_bf16(rng, (256,), 0.1)
    cap = 64
    kc = np.zeros((cap, 2, 256), np.float32)
    vc = np.zeros((cap, 2, 256), np.float32)
    kc64 = np.zeros((cap, 2, 256))
    vc64 = np.zeros((cap, 2, 256))
    for pos in range(12):
        q = rng.standard_normal((16, 512)).astype(np.float32)
        kn_ = rng.standard_normal((2, 256)).astype(np.float32)
        vn = rng.standard_normal((2, 256)).astype(np.float32)
        out = O.full_attn_step(q, kn_, vn, qn, kn, kc, vc, pos)
        for h in range(2):
            kc64[pos, h] = np_prep(kn_[h], kn, pos)
            vc64[pos, h] = vn[h]
        ref = np.zeros((16, 256))
        for h in range(16):
            qh = np_prep(q[h, :256], qn, pos)
            s = kc64[:pos + 1, h // 8] @ qh / 16
            p = np.exp(s - s.max())
            ref[h] = (p @ vc64[:pos + 1, h // 8]) / p.sum() / (1 + np.exp(-q[h, 256:].astype(np.float64)))
        assert np.abs(out - ref.reshape(-1)).max() <= 2e-5 * np.abs(ref).max(), pos
        assert np.abs(kc[:pos + 1] - kc64[:pos + 1]).max() <= 2e-5 * np.abs(kc64).max()
        assert np.array_equal(vc[:pos + 1], vc64[:pos + 1].astype(np.float32))


def test_oracle_bf16_cache_matches_numpy():
    """The bf16-cache step: the appended rows rounded to bf16 before
    the attention reads them; checked against the float64 statement with the same rounding
    (the k row may differ by one bf16 ulp where float32 and float64 round differently)."""
    rng = np.random.default_rng(9)
    qn = O.randn_bf16(rng, (256,), 0.1)
    kn = O.randn_bf16(rng, (256,), 0.1)
    cap = 32
    kc = np.zeros((cap, 2, 256), np.float32)
    vc = np.zeros((cap, 2, 256), np.float32)
    kc64 = np.zeros((cap, 2, 256))
    vc64 = np.zeros((cap, 2, 256))
    rnd = lambda a: O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32))).astype(np.float64)
    for pos in range(6):
        q = rng.standard_normal((16, 512)).astype(np.float32)
        kn_ = rng.standard_normal((2, 256)).astype(np.float32)
        vn = rng.standard_normal((2, 256)).astype(np.float32)
        out = O.full_attn_step(q, kn_, vn, qn, kn, kc, vc, pos, bf16_kv=True)
        for h in range(2):
            kc64[pos, h] = rnd(np_prep(kn_[h], kn, pos))
            vc64[pos, h] = rnd(vn[h])
        ref = np.zeros((16, 256))
        for h in range(16):
            qh = np_prep(q[h, :256], qn, pos)
            s = kc64[:pos + 1, h // 8] @ qh / 16
            p = np.exp(s - s.max())
            ref[h] = (p @ vc64[:pos + 1, h // 8]) / p.sum() / (1 + np.exp(-q[h, 256:].astype(np.float64)))
        assert np.abs(out - ref.reshape(-1)).max() <= 1e-4 * np.abs(ref).max(), pos
        assert np.all(np.abs(kc[:pos + 1] - kc64[:pos + 1]) <= 2.0 ** -7 * np.abs(kc64[:pos + 1]))
        assert np.array_equal(vc[:pos + 1], vc64[:pos + 1].astype(np.float32))
        assert np.array_equal(kc, O.bf16_to_f32(O.f32_to_bf16(kc)))   # the cache holds bf16 values
