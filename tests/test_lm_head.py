"""LM head (final RMSNorm + vocab GEMV + top-1): the CPU oracle pinned against the
reference's own math (src/math.m compiled unchanged) and the reference kernels' top-1 rule
(metal/kernels.metal:1562-1597, 1599-1713); no GPU needed."""
import numpy as np
import pytest

from oracle import oracle as O

FMAX = np.finfo(np.float32).max


def test_rms_norm_matches_reference_cpu_form():
    R = O.ref_lib()
    if R is None:
        pytest.skip("reference math.m not built here")
    rng = np.random.default_rng(3)
    for add_one in (0, 1):
        x = (rng.standard_normal(2048) * 3).astype(np.float32)
        w = O.f32_to_bf16(rng.standard_normal(2048).astype(np.float32) * 0.2)
        ref = np.empty(2048, np.float32)
        R.nmoe_cpu_rms_norm(x, w.ctypes.data, ref, 2048, 1e-6, add_one)
        got = O.rms_norm(x, w, 1e-6, bool(add_one))
        np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("vals,want", [
    ([1.0, 3.0, 3.0, 2.0], 1),                       # tie -> lower index
    ([np.nan, 0.5, np.nan, 0.5], 1),                # NaN never wins
    ([np.nan, np.nan], 0),                          # nothing qualifies -> 0
    ([-np.inf, -FMAX, -np.inf], 0),                 # -inf and -FLT_MAX never win
    ([-np.inf, -3.0e38, -np.inf], 1),
    ([-0.0, 0.0, -1.0], 0),                         # -0 == +0 -> lower index
    ([0.0, -0.0], 0),
    ([1.0, np.inf, np.inf], 1),
    ([np.float32(1.0), np.nextafter(np.float32(1.0), np.float32(2.0))], 1),   # adjacent floats
])
def test_top1_rule(vals, want):
    assert O.argmax_top1(np.array(vals, np.float32)) == want


@pytest.mark.parametrize("dtype", [O.DTYPE_Q4, O.DTYPE_BF16])
def test_head_logits_follow_reference_matvec(dtype):
    """Oracle head logits = the reference's sequential CPU dequant matvec (src/math.m:236-274)
    within fp32 reordering, and token = the rule applied to them."""
    head = O.make_lm_head(5, 3000, dtype)
    rng = np.random.default_rng(6)
    x = rng.standard_normal(2048).astype(np.float32)
    nw = O.f32_to_bf16(rng.standard_normal(2048).astype(np.float32) * 0.1)
    tok, logits = O.lm_head_argmax(head, x, nw)
    xn = O.rms_norm(x, nw)
    if dtype == O.DTYPE_Q4:
        R = O.ref_lib()
        if R is None:
            pytest.skip("reference math.m not built here")
        ref = np.empty(head.vocab, np.float32)
        R.nmoe_cpu_dequant_matvec(head.weight, head.scales, head.biases, xn, ref, head.vocab, 2048, 4)
    else:
        ref = (O.bf16_to_f32(head.weight).astype(np.float64) @ xn.astype(np.float64)).astype(np.float32)
    np.testing.assert_allclose(logits, ref, rtol=0, atol=2e-5 * np.abs(ref).max())
    assert tok == O.argmax_top1(logits)
    assert tok == int(np.argmax(ref)) or abs(ref[tok] - ref.max()) < 1e-5 * np.abs(ref).max()
