"""LM head on the GPU (nmoe_lm_head_argmax) against the CPU oracle: logits within the
stated tolerance, the token by the reference's top-1 rule, edge cases of that rule
(ties, NaN, ragged vocab), and the workspace left zeroed after every call."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu
VOCAB = 248320   # src/runtime.m:1911
# Logits tolerance: max |gpu - oracle| <= LOGIT_ATOL_FRAC * max |oracle logit|. The GPU sums
# each 64-column group as scale * sum(q x) + bias * sum(x) (the reference sums
# fma(q, scale, bias) * x column by column), so only fp32 rounding differs.
LOGIT_ATOL_FRAC = 3e-6


def _torch():
    import torch
    return torch


def _dev_head(head):
    torch = _torch()
    d = {"weight": torch.from_numpy(head.weight.view(np.int32) if head.weight.dtype == np.uint32
                                    else head.weight.view(np.int16)).cuda()}
    if head.scales is not None:
        d["scales"] = torch.from_numpy(head.scales.view(np.int16)).cuda()
        d["biases"] = torch.from_numpy(head.biases.view(np.int16)).cuda()
    return d


def _run(head, dh, x, nw=None, x_dtype=N.DTYPE_F32, want_logits=True, ws=None):
    torch = _torch()
    if x_dtype == N.DTYPE_F32:
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    else:
        xd = torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda()
    nwd = None if nw is None else torch.from_numpy(nw.view(np.int16)).cuda()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    if ws is None:
        ws = torch.zeros(N.lm_head_workspace_bytes() // 8, dtype=torch.int64, device="cuda")
    lg = torch.empty(head.vocab, dtype=torch.float32, device="cuda") if want_logits else None
    N.lm_head_argmax(dh, head.dtype, head.vocab, xd, tok, ws, x_dtype=x_dtype, norm_weight=nwd, logits_out=lg)
    torch.cuda.synchronize()
    assert int(ws.abs().sum().item()) == 0, "workspace not left zeroed"
    return int(tok.item()) & 0xFFFFFFFF, (None if lg is None else lg.cpu().numpy())


def _check(head, x, nw, tok, lg):
    xin = x if nw is None else x
    otok, ol = O.lm_head_argmax(head, xin, nw)
    scale = np.abs(ol).max()
    err = np.abs(lg - ol).max()
    assert err <= LOGIT_ATOL_FRAC * scale, (err, scale)
    assert tok == O.argmax_top1(lg)            # the rule, bit-exact on the GPU's own logits
    srt = np.sort(ol[~np.isnan(ol)])
    if srt.size >= 2 and srt[-1] - srt[-2] > 2 * LOGIT_ATOL_FRAC * scale:
        assert tok == otok
    return err / scale


@pytest.mark.parametrize("dtype", [N.DTYPE_Q4, N.DTYPE_BF16])
@pytest.mark.parametrize("vocab", [1, 17, 1000, 4099])
def test_small_vocab_with_norm(dtype, vocab):
    head = O.make_lm_head(11 + vocab, vocab, dtype)
    rng = np.random.default_rng(vocab)
    x = (rng.standard_normal(2048) * 2).astype(np.float32)
    nw = O.f32_to_bf16(rng.standard_normal(2048).astype(np.float32) * 0.1)
    tok, lg = _run(head, _dev_head(head), x, nw)
    _check(head, x, nw, tok, lg)


@pytest.mark.parametrize("dtype", [N.DTYPE_Q4, N.DTYPE_BF16])
def test_full_vocab(dtype):
    head = O.make_lm_head(77, VOCAB, dtype)
    dh = _dev_head(head)
    for seed in range(3):
        rng = np.random.default_rng(100 + seed)
        x = rng.standard_normal(2048).astype(np.float32)
        nw = O.f32_to_bf16(rng.standard_normal(2048).astype(np.float32) * 0.1)
        tok, lg = _run(head, dh, x, nw)
        _check(head, x, nw, tok, lg)
        tok2, _ = _run(head, dh, x, nw, want_logits=False)   # token-only call: same token
        assert tok2 == tok


def test_bf16_input_and_no_norm():
    head = O.make_lm_head(5, 5000, N.DTYPE_Q4)
    x = O.bf16_to_f32(O.f32_to_bf16(np.random.default_rng(1).standard_normal(2048).astype(np.float32)))
    tok, lg = _run(head, _dev_head(head), x, None, x_dtype=N.DTYPE_BF16)
    _check(head, x, None, tok, lg)


def test_duplicate_rows_tie_to_lowest_index():
    head = O.make_lm_head(8, 3000, N.DTYPE_Q4)
    x = np.random.default_rng(2).standard_normal(2048).astype(np.float32)
    _, ol = O.lm_head_argmax(head, x)
    top = int(np.argmax(ol))
    for dst in (top + 1 if top + 1 < 3000 else 0, 2999, 5):   # copies of the winning row
        head.weight[dst] = head.weight[top]
        head.scales[dst] = head.scales[top]
        head.biases[dst] = head.biases[top]
    tok, lg = _run(head, _dev_head(head), x)
    dups = [i for i in range(3000) if lg[i] == lg[top]]
    assert len(dups) >= 4   # identical rows give bit-identical logits
    assert tok == O.argmax_top1(lg)
    if lg[top] == np.nanmax(lg):
        assert tok == min(dups)


def test_nan_rows_never_win_and_all_nan_gives_zero():
    head = O.make_lm_head(9, 2000, N.DTYPE_Q4)
    x = np.random.default_rng(3).standard_normal(2048).astype(np.float32)
    _, ol = O.lm_head_argmax(head, x)
    top = int(np.argmax(ol))
    head.scales[top, 0] = 0x7FC0   # bf16 NaN scale: the winning row's logit becomes NaN
    tok, lg = _run(head, _dev_head(head), x)
    assert np.isnan(lg[top]) and tok != top and tok == O.argmax_top1(lg)
    xn = x.copy()
    xn[7] = np.nan                  # every logit NaN
    tok, lg = _run(head, _dev_head(head), xn)
    assert np.isnan(lg).all() and tok == 0


def test_workspace_reuse_across_calls():
    torch = _torch()
    head = O.make_lm_head(12, 6000, N.DTYPE_Q4)
    dh = _dev_head(head)
    ws = torch.zeros(N.lm_head_workspace_bytes() // 8, dtype=torch.int64, device="cuda")
    for seed in range(4):
        x = np.random.default_rng(40 + seed).standard_normal(2048).astype(np.float32)
        tok, lg = _run(head, dh, x, ws=ws)
        _check(head, x, None, tok, lg)


def test_rejects_bad_arguments():
    torch = _torch()
    head = O.make_lm_head(1, 32, N.DTYPE_Q4)
    dh = _dev_head(head)
    x = torch.zeros(2048, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(N.NmoeError):
        N.lm_head_argmax(dh, N.DTYPE_Q2, 32, x, tok, ws)
    with pytest.raises(N.NmoeError):
        N.lm_head_argmax({"weight": dh["weight"]}, N.DTYPE_Q4, 32, x, tok, ws)
    with pytest.raises(N.NmoeError):
        N.lm_head_argmax(dh, N.DTYPE_Q4, 0, x, tok, ws)
