"""nmoe_full_attn_step on the GPU against the oracle: consecutive positions from 0 with
the caches carried, and single steps at long positions over prefilled caches (many
split-K slices). Output within 2e-5 of its largest magnitude, the new cache rows within
2e-5 (k: RMS norm and RoPE in fp32, another order) and bit-exact (v)."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _setup(cap, seed):
    import torch
    rng = np.random.default_rng(seed)
    w = {"q_norm": O.randn_bf16(rng, (256,), 0.1), "k_norm": O.randn_bf16(rng, (256,), 0.1)}
    dw = {k: torch.from_numpy(v.view(np.int16).copy()).cuda() for k, v in w.items()}
    ws = torch.zeros(N.full_attn_workspace_bytes() // 4, dtype=torch.int32, device="cuda")
    return rng, w, dw, ws


def _step(torch, rng, w, dw, ws, kc, vc, dkc, dvc, pos, cap):
    q = rng.standard_normal((16, 512)).astype(np.float32)
    kn = rng.standard_normal((2, 256)).astype(np.float32)
    vn = rng.standard_normal((2, 256)).astype(np.float32)
    out = torch.zeros(16 * 256, device="cuda")
    N.full_attn_step(dw, torch.from_numpy(q).cuda(), torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda(),
                     dkc, dvc, pos, cap, out, ws)
    ref = O.full_attn_step(q, kn, vn, w["q_norm"], w["k_norm"], kc, vc, pos)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() <= TOL * np.abs(ref).max(), (pos, np.abs(got - ref).max())
    gk, gv = dkc.cpu().numpy(), dvc.cpu().numpy()
    assert np.abs(gk[pos] - kc[pos]).max() <= TOL * np.abs(kc[pos]).max()
    assert np.array_equal(gv[pos], vc[pos])
    assert int(ws[-64:].abs().sum().item()) == 0


def test_consecutive_positions():
    import torch
    cap = 40
    rng, w, dw, ws = _setup(cap, 1)
    kc = np.zeros((cap, 2, 256), np.float32)
    vc = np.zeros((cap, 2, 256), np.float32)
    dkc, dvc = torch.zeros(cap, 2, 256, device="cuda"), torch.zeros(cap, 2, 256, device="cuda")
    for pos in range(20):
        _step(torch, rng, w, dw, ws, kc, vc, dkc, dvc, pos, cap)


@pytest.mark.parametrize("pos", [255, 256, 4099, 30000])
def test_long_positions(pos):
    import torch
    cap = pos + 8
    rng, w, dw, ws = _setup(cap, pos)
    kc = (rng.standard_normal((cap, 2, 256)) * 0.3).astype(np.float32)
    vc = rng.standard_normal((cap, 2, 256)).astype(np.float32)
    dkc, dvc = torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda()
    _step(torch, rng, w, dw, ws, kc, vc, dkc, dvc, pos, cap)


def test_rejects_bad_position():
    import torch
    rng, w, dw, ws = _setup(8, 2)
    buf = torch.zeros(16 * 512, device="cuda")
    with pytest.raises(N.NmoeError):
        N.full_attn_step(dw, buf, buf, buf, buf, buf, 8, 8, buf, ws)


def _bf16_round(a):
    return O.bf16_to_f32(O.f32_to_bf16(np.ascontiguousarray(a, np.float32)))


def test_batched_bf16_cache():
    """nmoe_full_attn_step_batched: 5 sequences over one bf16 cache at positions that
    straddle slice boundaries (0, 63, 64, 700) and one outside the cache (zeros out, caches
    untouched); each against the oracle's bf16-cache step. The new k row within one bf16
    ulp (fp32 norm and RoPE in another order, then rounded), the new v row bit-exact."""
    import torch
    cap, positions = 768, [0, 63, 64, 700, 768]
    B = len(positions)
    rng = np.random.default_rng(77)
    w = {"q_norm": O.randn_bf16(rng, (256,), 0.1), "k_norm": O.randn_bf16(rng, (256,), 0.1)}
    dw = {k: torch.from_numpy(v.view(np.int16).copy()).cuda() for k, v in w.items()}
    kc = _bf16_round(rng.standard_normal((B, cap, 2, 256)) * 0.3)
    vc = _bf16_round(rng.standard_normal((B, cap, 2, 256)))
    q = rng.standard_normal((B, 16, 512)).astype(np.float32)
    kn = rng.standard_normal((B, 2, 256)).astype(np.float32)
    vn = rng.standard_normal((B, 2, 256)).astype(np.float32)
    dkc = torch.from_numpy(O.f32_to_bf16(kc).view(np.int16).copy()).cuda()
    dvc = torch.from_numpy(O.f32_to_bf16(vc).view(np.int16).copy()).cuda()
    ws = torch.zeros(N.full_attn_batched_workspace_bytes(B) // 4, dtype=torch.int32, device="cuda")
    out = torch.full((B, 16 * 256), 7.0, device="cuda")
    pos_d = torch.tensor(positions, dtype=torch.int32, device="cuda")
    N.full_attn_step_batched(dw, torch.from_numpy(q).cuda(), torch.from_numpy(kn).cuda(),
                             torch.from_numpy(vn).cuda(), dkc, dvc, pos_d, cap, out, ws)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    gk = O.bf16_to_f32(dkc.cpu().numpy().view(np.uint16))
    gv = O.bf16_to_f32(dvc.cpu().numpy().view(np.uint16))
    for b, pos in enumerate(positions):
        if pos >= cap:
            assert not got[b].any(), "a position outside the cache gives zeros"
            assert np.array_equal(gk[b], kc[b]) and np.array_equal(gv[b], vc[b])
            continue
        hk, hv = kc[b].copy(), vc[b].copy()
        ref = O.full_attn_step(q[b], kn[b], vn[b], w["q_norm"], w["k_norm"], hk, hv, pos, bf16_kv=True)
        assert np.abs(got[b] - ref).max() <= 1e-4 * np.abs(ref).max(), (pos, np.abs(got[b] - ref).max())
        assert np.all(np.abs(gk[b, pos] - hk[pos]) <= 2.0 ** -7 * np.abs(hk[pos])), pos
        assert np.array_equal(gv[b, pos], hv[pos]), pos
        others = np.ones(cap, bool)
        others[pos] = False
        assert np.array_equal(gk[b, others], kc[b, others]) and np.array_equal(gv[b, others], vc[b, others])
    assert int(ws[-64:].abs().sum().item()) == 0
