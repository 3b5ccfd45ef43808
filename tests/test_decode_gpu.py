"""Batch-1 routed-MoE block on the GPU through the C ABI, against the CPU oracle.

Parity bar: router indices bit-exact, outputs within 1e-2
relative L2 (we assert far tighter where the arithmetic allows it).
Routing is compared on the GPU's own logits: the oracle's reference top-k
(softmax -> top-k -> renormalise of src/math.m) run on those logits must pick the
same experts in the same order."""
import numpy as np
import pytest

import nmoe_b200 as N
from nmoe_testutil import bf16_round, distinct_layer, rel_l2, upload
from oracle import oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# Output tolerance (relative L2) of the default path, whose routed-expert dot products
# run in half2 with fp32 flushes (~3e-4 typical); the requirement is 1e-2. The fp32
# expert path (NMOE_EXPERT_FP32=1) is held to 1e-4 in test_fp32_expert_path.
OUT_TOL = 2e-3

CONFIGS = {
    # name: (bits, router dtype, shared dtype, x dtype)
    "cfg0_q4_bf16": (4, N.DTYPE_BF16, N.DTYPE_BF16, N.DTYPE_BF16),
    "ref_q4_q4_f32": (4, N.DTYPE_Q4, N.DTYPE_Q4, N.DTYPE_F32),
    "cfg1_q2_bf16": (2, N.DTYPE_BF16, N.DTYPE_BF16, N.DTYPE_BF16),
    "q2_q4_f32": (2, N.DTYPE_Q4, N.DTYPE_Q4, N.DTYPE_F32),
}

_cache = {}


def setup(name, num_layers=2):
    if name in _cache:
        return _cache[name]
    bits, rdt, sdt, _ = CONFIGS[name]
    ctx = N.Context(quant_bits=bits, num_layers=num_layers, router_dtype=rdt, shared_dtype=sdt, device=0)
    layers = []
    for l in range(num_layers):
        lw = O.make_layer(100 + l, bits=bits, router_dtype=rdt, shared_dtype=sdt, distinct_experts=24)
        upload(ctx, l, lw)
        layers.append(lw)
    _cache[name] = (ctx, layers)
    return ctx, layers


def make_x(seed, x_dtype):
    x = np.random.default_rng(seed).standard_normal(2048, dtype=np.float32)
    if x_dtype == N.DTYPE_BF16:
        xb = O.f32_to_bf16(x)
        return O.bf16_to_f32(xb), torch.from_numpy(xb.view(np.int16)).cuda()
    return x, torch.from_numpy(x).cuda()


def run_gpu(ctx, layer, k, xd, x_dtype, hm=None):
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    idx = torch.full((8,), 77, dtype=torch.int32, device="cuda")
    w = torch.full((8,), 9.0, dtype=torch.float32, device="cuda")
    ctx.forward(layer, k, xd, out, x_dtype=x_dtype, h_mid=hm, idx_out=idx, w_out=w)
    lg = torch.zeros(256, dtype=torch.float32, device="cuda")
    ctx.route(layer, k, xd, x_dtype=x_dtype, logits_out=lg)
    torch.cuda.synchronize()
    return out.cpu().numpy(), idx.cpu().numpy().view(np.uint32), w.cpu().numpy(), lg.cpu().numpy()


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("k", [1, 2, 4, 6, 8])
def test_block_matches_oracle(name, k):
    ctx, layers = setup(name)
    x_dtype = CONFIGS[name][3]
    for layer in range(len(layers)):
        for trial in range(2):
            x, xd = make_x(1000 * layer + 10 * k + trial, x_dtype)
            out, idx, w, lg = run_gpu(ctx, layer, k, xd, x_dtype)
            ref = O.block_forward(layers[layer], k, x, logits_override=lg)
            # logits: fp32 arithmetic differs in order (and, on q4 rows, in the conversion-free
            # dequant, about 1e-5 relative); routing is checked on these logits below
            assert rel_l2(lg, ref["logits"]) < 5e-5
            # routing on the GPU's logits is bit-exact with the reference rule
            ridx, rw = O.route_reference(lg, k)
            np.testing.assert_array_equal(idx[:k], ridx)
            np.testing.assert_array_equal(idx[k:], 0)
            np.testing.assert_allclose(w[:k], rw, rtol=2e-6, atol=1e-7)
            np.testing.assert_array_equal(w[k:], 0)
            assert rel_l2(out, ref["out"]) < OUT_TOL, rel_l2(out, ref["out"])
            # the oracle routing on its own logits agrees unless the k-th/(k+1)-th gap is a near tie
            own = O.block_forward(layers[layer], k, x)
            if not np.array_equal(own["idx"][:k], idx[:k]):
                srt = np.sort(ref["logits"])[::-1]
                assert srt[k - 1] - srt[k] < 1e-4


@pytest.mark.parametrize("name", ["cfg0_q4_bf16", "ref_q4_q4_f32"])
def test_residual_h_mid(name):
    ctx, layers = setup(name)
    x_dtype = CONFIGS[name][3]
    x, xd = make_x(5, x_dtype)
    hm = np.random.default_rng(6).standard_normal(2048, dtype=np.float32)
    out, _, _, lg = run_gpu(ctx, 0, 8, xd, x_dtype, torch.from_numpy(hm).cuda())
    ref = O.block_forward(layers[0], 8, x, h_mid=hm, logits_override=lg)
    assert rel_l2(out, ref["out"]) < OUT_TOL


def test_tie_goes_to_lower_expert_id():
    """Two identical router rows give bit-identical logits; the lower id must win."""
    bits = 4
    ctx = N.Context(quant_bits=bits, num_layers=1, device=0)
    lw = O.make_layer(7, bits=bits, distinct_experts=8)
    r = lw.router["weight"].copy()
    r[200] = r[37]
    r[201] = r[37]
    # make the tied rows the top logits for an input aligned with them
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    upload(ctx, 0, lw)
    x = bf16_round(O.bf16_to_f32(r[37]) * 50.0)
    xd = torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda()
    for k in (1, 2, 3, 8):
        out, idx, w, lg = run_gpu(ctx, 0, k, xd, N.DTYPE_BF16)
        assert lg[37] == lg[200] == lg[201]
        assert idx[0] == 37
        if k >= 3:
            assert list(idx[:3]) == [37, 200, 201]
        ridx, _ = O.route_reference(lg, k)
        np.testing.assert_array_equal(idx[:k], ridx)


def _exact_router_layer(seed):
    """A layer whose router rows are zero except columns 0 and 1, so that with
    x = [0.25, 2^-25, 0, ...] the logits are exact sums (no rounding)."""
    lw = O.make_layer(seed, bits=4, distinct_experts=8)
    r = np.zeros_like(lw.router["weight"])
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    x = np.zeros(2048, np.float32)
    x[0], x[1] = 0.25, 2.0 ** -25
    return lw, r, x


def test_adjacent_float_logits_follow_logit_order():
    """Experts 10 and 3 get adjacent-float logits (10 the larger) that collide in the
    reference's fp32 softmax: the device keeps logit order (10 first); the reference's
    rule on the same logits picks the same sequence of probabilities (3 first)."""
    lw, r, x = _exact_router_layer(17)
    one = O.f32_to_bf16(np.array([1.0], np.float32))[0]
    two, three = O.f32_to_bf16(np.array([2.0, 3.0], np.float32))
    r[10, 0], r[10, 1] = one, three
    r[3, 0], r[3, 1] = one, two
    ctx = N.Context(quant_bits=4, num_layers=1, device=0)
    upload(ctx, 0, lw)
    xd = torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda()
    for k in (1, 2, 8):
        out, idx, w, lg = run_gpu(ctx, 0, k, xd, N.DTYPE_BF16)
        assert np.nextafter(lg[3], np.float32(1)) == lg[10]
        assert idx[0] == 10 and (k == 1 or idx[1] == 3)
        ridx, _ = O.route_reference(lg, k)
        p = lg.copy()
        O.lib().orc_softmax(p, p.size)
        np.testing.assert_array_equal(p[idx[:k]], p[ridx])
        ref = O.block_forward(lw, k, x, logits_override=lg)
        assert rel_l2(out, ref["out"]) < OUT_TOL or k == 1
    assert ctx.device_status() == (N.OK, 0)


def test_nan_logit_is_never_selected():
    """A NaN router row gives a NaN logit: it ranks below every other logit (the
    reference's strict > never prefers it), and the block output stays finite."""
    ctx = N.Context(quant_bits=4, num_layers=1, device=0)
    lw = O.make_layer(23, bits=4, distinct_experts=8)
    r = lw.router["weight"].copy()
    r[77] = 0x7FC0
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    upload(ctx, 0, lw)
    x, xd = make_x(4, N.DTYPE_BF16)
    for k in (1, 8):
        out, idx, w, lg = run_gpu(ctx, 0, k, xd, N.DTYPE_BF16)
        assert np.isnan(lg[77]) and 77 not in idx[:k]
        ridx, _ = O.route_reference(np.where(np.isnan(lg), np.float32(-np.inf), lg), k)
        np.testing.assert_array_equal(idx[:k], ridx)
        assert np.isfinite(out).all()
    assert ctx.device_status() == (N.OK, 0)


def test_all_logits_tied_picks_lowest_ids():
    """All 256 router rows identical: every logit ties, so the selection is experts
    0..k-1 (lower id first) with equal weights."""
    ctx = N.Context(quant_bits=4, num_layers=1, device=0)
    lw = O.make_layer(9, bits=4, distinct_experts=8)
    r = lw.router["weight"].copy()
    r[:] = r[5]
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    upload(ctx, 0, lw)
    x, xd = make_x(3, N.DTYPE_BF16)
    for k in (1, 3, 8):
        out, idx, w, lg = run_gpu(ctx, 0, k, xd, N.DTYPE_BF16)
        assert (lg == lg[0]).all()
        assert list(idx[:k]) == list(range(k))
        np.testing.assert_allclose(w[:k], 1.0 / k, rtol=1e-6)
        ridx, _ = O.route_reference(lg, k)
        np.testing.assert_array_equal(idx[:k], ridx)


def test_argument_errors():
    ctx, _ = setup("cfg0_q4_bf16")
    x, xd = make_x(1, N.DTYPE_BF16)
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    for k in (0, 9):
        with pytest.raises(N.NmoeError) as ei:
            ctx.forward(0, k, xd, out)
        assert ei.value.status == N.EINVAL
    with pytest.raises(N.NmoeError) as ei:
        ctx.forward(5, 8, xd, out)
    assert ei.value.status == N.EINVAL
    with pytest.raises(N.NmoeError) as ei:
        ctx.forward(0, 8, xd, out, x_dtype=N.DTYPE_Q4)
    assert ei.value.status == N.EINVAL
    with pytest.raises(N.NmoeError) as ei:
        ctx.load_layer(0, np.zeros(100, np.uint8))
    assert ei.value.status == N.ESIZE
    fresh = N.Context(quant_bits=4, num_layers=1, device=0)
    with pytest.raises(N.NmoeError) as ei:   # weights never uploaded
        fresh.forward(0, 8, xd, out)
    assert ei.value.status == N.EINVAL


def test_k_max_bound():
    ctx = N.Context(quant_bits=4, num_layers=1, k_max=4, device=0)
    lw = O.make_layer(3, distinct_experts=4)
    upload(ctx, 0, lw)
    x, xd = make_x(2, N.DTYPE_BF16)
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    ctx.forward(0, 4, xd, out)
    with pytest.raises(N.NmoeError):
        ctx.forward(0, 5, xd, out)


def test_out_of_range_expert_sets_device_error():
    """num_experts < 256: a routed id beyond the uploaded experts raises the device error
    word and contributes nothing (the reference's invalid-slot rule, src/runtime.m:2980)."""
    ne = 16
    ctx = N.Context(quant_bits=4, num_layers=1, num_experts=ne, device=0)
    lw = O.make_layer(9, distinct_experts=4)
    r = lw.router["weight"].copy()
    upload_lw = O.LayerWeights(4, lw.experts[:ne * O.expert_size(4)].copy(), ne, lw.router, lw.shared_gate,
                               lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    upload(ctx, 0, upload_lw)
    assert ctx.device_status() == (N.OK, 0)
    x = bf16_round(O.bf16_to_f32(r[100]) * 50.0)   # expert 100 wins
    xd = torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda()
    out, idx, w, lg = run_gpu(ctx, 0, 1, xd, N.DTYPE_BF16)
    assert idx[0] == 100
    rc, code = ctx.device_status()
    assert rc == N.EDEVICE and code == 1
    assert ctx.device_status() == (N.OK, 0)   # cleared
    assert np.isfinite(out).all()


def test_load_layer_file(tmp_path):
    bits = 2
    ctx = N.Context(quant_bits=bits, num_layers=1, device=0)
    lw = O.make_layer(21, bits=bits, distinct_experts=4)
    p = tmp_path / "layer_00.bin"
    lw.experts.tofile(p)
    ctx.load_layer_file(0, str(p))
    ctx.set_dense(0, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    x, xd = make_x(4, N.DTYPE_BF16)
    out, idx, w, lg = run_gpu(ctx, 0, 8, xd, N.DTYPE_BF16)
    ref = O.block_forward(lw, 8, x, logits_override=lg)
    assert rel_l2(out, ref["out"]) < OUT_TOL
    (tmp_path / "short.bin").write_bytes(b"\0" * 1000)
    with pytest.raises(N.NmoeError) as ei:
        ctx.load_layer_file(0, str(tmp_path / "short.bin"))
    assert ei.value.status == N.ESIZE


def test_repeated_calls_agree_and_counters_reset():
    """Back-to-back calls reuse the launch-tag exchange (epoch / done counter) and the
    output initialisation: same ids, same outputs up to the order of the fp32 adds that
    combine the CTAs' split-K partials."""
    ctx, layers = setup("cfg0_q4_bf16")
    x, xd = make_x(31, N.DTYPE_BF16)
    hm = torch.randn(2048, device="cuda")
    runs = [run_gpu(ctx, 0, 8, xd, N.DTYPE_BF16, hm) for _ in range(4)]
    for o, idx, w, lg in runs[1:]:
        np.testing.assert_array_equal(runs[0][1], idx)
        np.testing.assert_array_equal(runs[0][3], lg)
        assert rel_l2(o, runs[0][0]) < 1e-6
    assert ctx.device_status() == (N.OK, 0)
    trail = ctx.debug_trail(1024)
    assert not (trail >= 100).any()   # no bounded wait gave up


def test_timeline_records_only_the_last_call(monkeypatch):
    """NMOE_TIMELINE=1: a full forward stamps every phase; a routing-only call after it
    leaves the routed phases unstamped instead of keeping the previous call's stamps."""
    lw = O.make_layer(91, bits=4, distinct_experts=8)
    monkeypatch.setenv("NMOE_TIMELINE", "1")
    ct = N.Context(quant_bits=4, num_layers=1, device=0)
    monkeypatch.delenv("NMOE_TIMELINE")
    upload(ct, 0, lw)
    G = ct.decode_grid()
    assert 1 <= G <= 256
    x, xd = make_x(12, N.DTYPE_BF16)
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    ct.forward(0, 8, xd, out)
    ph = ct.timeline_phases()
    for name in ("x staged", "logits seen", "first unit landed", "routed units done", "end"):
        assert name in ph, name
    assert ph["end"][1] >= ph["logits seen"][1] >= 0
    ct.route(0, 8, xd)
    tl = ct.debug_timeline()
    assert tl.shape == (G, N.TIMELINE_WIDTH)
    assert (tl[:, 11] == 0).all() and (tl[:, 5] == 0).all()
    assert (tl[:, 7] != 0).all()
    assert ct.device_status() == (N.OK, 0)
    ct.close()


def test_bounded_wait_timeout_reports_and_recovers(monkeypatch):
    """The logits wait is pointed at a tag that no CTA writes (NMOE_TEST_STALL_WAIT) with a
    1 ms budget: the bounded wait expires, the call returns, the host reads NMOE_ETIMEOUT
    from the device error word, and the device stays usable."""
    lw = O.make_layer(77, bits=4, distinct_experts=8)
    monkeypatch.setenv("NMOE_WAIT_TIMEOUT_MS", "1")
    monkeypatch.setenv("NMOE_TEST_STALL_WAIT", "1")
    ct = N.Context(quant_bits=4, num_layers=1, device=0)
    monkeypatch.delenv("NMOE_WAIT_TIMEOUT_MS")
    monkeypatch.delenv("NMOE_TEST_STALL_WAIT")
    upload(ct, 0, lw)
    x, xd = make_x(8, N.DTYPE_BF16)
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    ct.forward(0, 8, xd, out)
    rc, code = ct.device_status()
    assert rc == N.ETIMEOUT and code == 2
    ct.close()
    cn = N.Context(quant_bits=4, num_layers=1, device=0)
    upload(cn, 0, lw)
    o, idx, w, lg = run_gpu(cn, 0, 8, xd, N.DTYPE_BF16)
    ref = O.block_forward(lw, 8, x, logits_override=lg)
    assert rel_l2(o, ref["out"]) < OUT_TOL
    assert cn.device_status() == (N.OK, 0)


@pytest.mark.parametrize("name", ["cfg0_q4_bf16", "ref_q4_q4_f32", "cfg1_q2_bf16"])
def test_fp32_expert_path(monkeypatch, name):
    """NMOE_EXPERT_FP32=1 selects fp32 routed-expert dot products: 1e-4 bar."""
    bits, rdt, sdt, x_dtype = CONFIGS[name]
    lw = O.make_layer(66, bits=bits, router_dtype=rdt, shared_dtype=sdt, distinct_experts=12)
    monkeypatch.setenv("NMOE_EXPERT_FP32", "1")
    ctx = N.Context(quant_bits=bits, num_layers=1, router_dtype=rdt, shared_dtype=sdt, device=0)
    monkeypatch.delenv("NMOE_EXPERT_FP32")
    upload(ctx, 0, lw)
    for t in range(3):
        x, xd = make_x(500 + t, x_dtype)
        out, idx, w, lg = run_gpu(ctx, 0, 8, xd, x_dtype)
        ref = O.block_forward(lw, 8, x, logits_override=lg)
        np.testing.assert_array_equal(idx, ref["idx"])
        assert rel_l2(out, ref["out"]) < 1e-4, rel_l2(out, ref["out"])


@pytest.mark.parametrize("bits", [4, 2])
def test_distinct_packs_in_every_slot(bits):
    """Every one of the 256 slots holds its own pack: 24 tokens (192 routed picks) must
    match the oracle, so each unit's copies read the slot the router chose."""
    lw = distinct_layer(bits)
    ctx = N.Context(quant_bits=bits, num_layers=1, device=0)
    upload(ctx, 0, lw)
    seen = set()
    for t in range(24):
        x, xd = make_x(7000 + t, N.DTYPE_BF16)
        out, idx, w, lg = run_gpu(ctx, 0, 8, xd, N.DTYPE_BF16)
        ref = O.block_forward(lw, 8, x, logits_override=lg)
        np.testing.assert_array_equal(idx, ref["idx"])
        assert rel_l2(out, ref["out"]) < OUT_TOL, rel_l2(out, ref["out"])
        seen.update(idx.tolist())
    assert len(seen) > 100
    assert ctx.device_status() == (N.OK, 0)
    ctx.close()
