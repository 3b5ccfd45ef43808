"""T-token MoE block (nmoe_moe_forward_batched) on the GPU, against the CPU oracle.

The batched path is the reference block applied to every token (the reference runs
prefill token by token, src/runtime.m:3816). Parity bar: router indices bit-exact on
the GPU's own logits, outputs within 1e-2 relative L2 (bf16 tensor-core operands with
fp32 accumulation)."""
import numpy as np
import pytest

import nmoe_b200 as N
from nmoe_testutil import distinct_layer, rel_l2, upload
from oracle import oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# bf16 operands (x, dequantised weights, SwiGLU activations, per-expert down outputs)
# with fp32 accumulation: a few 1e-3 relative; the requirement is 1e-2.
OUT_TOL = 1e-2
LOGIT_TOL = 5e-5
T_MAX = 512

CONFIGS = {
    # name: (bits, router dtype, shared dtype, x dtype)
    "cfg2_q4_bf16": (4, N.DTYPE_BF16, N.DTYPE_BF16, N.DTYPE_BF16),
    "ref_q4_q4_f32": (4, N.DTYPE_Q4, N.DTYPE_Q4, N.DTYPE_F32),
    "q2_bf16": (2, N.DTYPE_BF16, N.DTYPE_BF16, N.DTYPE_BF16),
    "q2_q4_f32": (2, N.DTYPE_Q4, N.DTYPE_Q4, N.DTYPE_F32),
}

_cache = {}


def setup(name):
    if name in _cache:
        return _cache[name]
    bits, rdt, sdt, _ = CONFIGS[name]
    ctx = N.Context(quant_bits=bits, num_layers=1, router_dtype=rdt, shared_dtype=sdt, t_max=T_MAX, device=0)
    lw = O.make_layer(300, bits=bits, router_dtype=rdt, shared_dtype=sdt, distinct_experts=24)
    upload(ctx, 0, lw)
    _cache[name] = (ctx, lw)
    return ctx, lw


def make_x(seed, T, x_dtype):
    x = np.random.default_rng(seed).standard_normal((T, 2048), dtype=np.float32)
    if x_dtype == N.DTYPE_BF16:
        xb = O.f32_to_bf16(x)
        return O.bf16_to_f32(xb), torch.from_numpy(xb.view(np.int16)).cuda()
    return x, torch.from_numpy(x).cuda()


def run(ctx, T, k, xd, x_dtype, hm=None, out_dtype=N.DTYPE_F32):
    out = torch.zeros((max(T, 1), 2048), dtype=torch.float32 if out_dtype == N.DTYPE_F32 else torch.bfloat16,
                      device="cuda")
    idx = torch.full((max(T, 1), 8), 77, dtype=torch.int32, device="cuda")
    w = torch.full((max(T, 1), 8), 9.0, dtype=torch.float32, device="cuda")
    ctx.forward_batched(0, T, k, xd, out, x_dtype=x_dtype, out_dtype=out_dtype, h_mid=hm, idx_out=idx, w_out=w)
    torch.cuda.synchronize()
    lg = ctx.debug_logits(T)
    o = out.float().cpu().numpy()
    return o, idx.cpu().numpy().view(np.uint32), w.cpu().numpy(), lg


def check(lw, k, x, o, idx, w, lg, hm=None, tol=OUT_TOL):
    T = x.shape[0]
    ref_lg = np.empty_like(lg)
    ref_out = np.empty_like(o[:T])
    for t in range(T):
        r = O.block_forward(lw, k, x[t], h_mid=None if hm is None else hm[t], logits_override=lg[t])
        ref_lg[t] = r["logits"]
        ref_out[t] = r["out"]
        ridx, rw = O.route_reference(lg[t], k)
        np.testing.assert_array_equal(idx[t, :k], ridx)
        np.testing.assert_array_equal(idx[t, k:], 0)
        np.testing.assert_allclose(w[t, :k], rw, rtol=2e-6, atol=1e-7)
        np.testing.assert_array_equal(w[t, k:], 0)
    assert rel_l2(lg, ref_lg) < LOGIT_TOL, rel_l2(lg, ref_lg)
    err = rel_l2(o[:T], ref_out)
    assert err < tol, err
    return err


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("T,k", [(1, 8), (7, 1), (16, 8), (130, 4)])
def test_batched_matches_oracle(name, T, k):
    ctx, lw = setup(name)
    x_dtype = CONFIGS[name][3]
    x, xd = make_x(7 * T + k, T, x_dtype)
    o, idx, w, lg = run(ctx, T, k, xd, x_dtype)
    check(lw, k, x, o, idx, w, lg)


def test_batched_256_tokens():
    ctx, lw = setup("cfg2_q4_bf16")
    x, xd = make_x(99, 256, N.DTYPE_BF16)
    o, idx, w, lg = run(ctx, 256, 8, xd, N.DTYPE_BF16)
    check(lw, 8, x, o, idx, w, lg)


def test_one_expert_group_spans_chunks():
    """300 identical tokens route to the same k experts: every group holds 300
    positions (three 128-token items), and all rows must equal the single-token block."""
    ctx, lw = setup("cfg2_q4_bf16")
    T = 300
    x1 = np.random.default_rng(3).standard_normal(2048, dtype=np.float32)
    xb = np.repeat(O.f32_to_bf16(x1)[None, :], T, axis=0)
    xd = torch.from_numpy(xb.view(np.int16)).cuda()
    o, idx, w, lg = run(ctx, T, 8, xd, N.DTYPE_BF16)
    assert (idx == idx[0]).all()
    assert np.array_equal(o, np.repeat(o[:1], T, axis=0))
    check(lw, 8, O.bf16_to_f32(xb[:1]), o[:1], idx[:1], w[:1], lg[:1])


@pytest.mark.parametrize("name", ["cfg2_q4_bf16", "ref_q4_q4_f32"])
def test_batched_h_mid_and_bf16_out(name):
    ctx, lw = setup(name)
    x_dtype = CONFIGS[name][3]
    T = 24
    x, xd = make_x(5, T, x_dtype)
    hm = np.random.default_rng(6).standard_normal((T, 2048), dtype=np.float32)
    o, idx, w, lg = run(ctx, T, 8, xd, x_dtype, hm=torch.from_numpy(hm).cuda())
    check(lw, 8, x, o, idx, w, lg, hm=hm)
    ob, idxb, _, _ = run(ctx, T, 8, xd, x_dtype, hm=torch.from_numpy(hm).cuda(), out_dtype=N.DTYPE_BF16)
    np.testing.assert_array_equal(idxb, idx)
    assert rel_l2(ob, o) < 5e-3


def test_batched_deterministic():
    ctx, lw = setup("cfg2_q4_bf16")
    x, xd = make_x(11, 200, N.DTYPE_BF16)
    a = run(ctx, 200, 8, xd, N.DTYPE_BF16)
    b = run(ctx, 200, 8, xd, N.DTYPE_BF16)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)
    assert ctx.device_status() == (0, 0)


def test_batched_matches_decode_routing():
    """forward_batched on one token and forward (batch-1 kernel) pick the same experts."""
    ctx, lw = setup("cfg2_q4_bf16")
    x, xd = make_x(12, 1, N.DTYPE_BF16)
    o, idx, w, lg = run(ctx, 1, 8, xd, N.DTYPE_BF16)
    out1 = torch.zeros(2048, dtype=torch.float32, device="cuda")
    idx1 = torch.zeros(8, dtype=torch.int32, device="cuda")
    ctx.forward(0, 8, xd[0], out1, x_dtype=N.DTYPE_BF16, idx_out=idx1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx[0], idx1.cpu().numpy().view(np.uint32))
    assert rel_l2(o[0], out1.cpu().numpy()) < OUT_TOL


def test_batched_all_logits_tied():
    """Identical router rows: every token's logits tie, and each token selects experts
    0..k-1 with equal weights."""
    ctx = N.Context(quant_bits=4, num_layers=1, t_max=64, device=0)
    lw = O.make_layer(10, bits=4, distinct_experts=8)
    r = lw.router["weight"].copy()
    r[:] = r[9]
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    upload(ctx, 0, lw)
    x, xd = make_x(4, 40, N.DTYPE_BF16)
    o, idx, w, lg = run(ctx, 40, 8, xd, N.DTYPE_BF16)
    assert (lg == lg[:, :1]).all()
    np.testing.assert_array_equal(idx, np.tile(np.arange(8, dtype=np.uint32), (40, 1)))
    np.testing.assert_allclose(w, 1.0 / 8, rtol=1e-6)


def test_batched_argument_errors():
    ctx, lw = setup("cfg2_q4_bf16")
    x, xd = make_x(1, 4, N.DTYPE_BF16)
    out = torch.zeros((4, 2048), dtype=torch.float32, device="cuda")
    with pytest.raises(N.NmoeError) as ei:
        ctx.forward_batched(0, T_MAX + 1, 8, xd, out)
    assert ei.value.status == N.EINVAL
    with pytest.raises(N.NmoeError):
        ctx.forward_batched(0, 4, 9, xd, out)
    with pytest.raises(N.NmoeError):
        ctx.forward_batched(0, 4, 8, xd, out, out_dtype=N.DTYPE_Q4)
    ctx.forward_batched(0, 0, 8, xd, out)   # T = 0 is a no-op
    ctx2 = N.Context(quant_bits=4, num_layers=1, device=0)   # t_max 0: no batched workspace
    upload(ctx2, 0, lw)
    with pytest.raises(N.NmoeError):
        ctx2.forward_batched(0, 1, 8, xd, out)


def test_t4096_distinct_packs():
    """Config 2 at its largest size, T = 4096 (t_max 4096), on a layer whose 256 slots all
    hold different packs: every token's ids against the reference rule on the GPU's
    logits, and a 256-token sample of outputs against the oracle."""
    T = 4096
    lw = distinct_layer(4)
    ctx = N.Context(quant_bits=4, num_layers=1, t_max=T, device=0)
    upload(ctx, 0, lw)
    x, xd = make_x(4096, T, N.DTYPE_BF16)
    o, idx, w, lg = run(ctx, T, 8, xd, N.DTYPE_BF16)
    for t in range(T):
        ridx, rw = O.route_reference(lg[t], 8)
        np.testing.assert_array_equal(idx[t], ridx)
        np.testing.assert_allclose(w[t], rw, rtol=2e-6, atol=1e-7)
    assert np.unique(idx).size == 256          # every slot was read
    sample = np.random.default_rng(1).choice(T, 256, replace=False)
    ref = np.stack([O.block_forward(lw, 8, x[t], logits_override=lg[t])["out"] for t in sample])
    err = rel_l2(o[sample], ref)
    assert err < OUT_TOL, err
    assert ctx.device_status() == (N.OK, 0)
    ctx.close()
