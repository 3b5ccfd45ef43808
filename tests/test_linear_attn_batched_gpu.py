"""nmoe_linear_attn_step_batched: 3 sequences with their own weights-shared states and
inputs over 3 steps, each against the oracle's single-sequence step: conv state bit-exact,
recurrent state and output within 2e-5 of the largest magnitude."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-5


def test_batched_steps_match_oracle():
    import torch
    B = 3
    w = O.make_linear_attn(4)
    dw = {k: torch.from_numpy(v.view(np.int16).copy() if v.dtype == np.uint16 else v.copy()).cuda()
          for k, v in w.items()}
    rng = np.random.default_rng(41)
    conv = [np.zeros((3, 8192), np.float32) for _ in range(B)]
    S = [(rng.standard_normal((32, 128, 128)) * 0.05 * b).astype(np.float32) for b in range(B)]
    dconv = torch.from_numpy(np.stack(conv)).cuda()
    dS = torch.from_numpy(np.stack(S)).cuda()
    out = torch.zeros(B, 4096, device="cuda")
    for step in range(3):
        inps = [O.linear_attn_inputs(rng) for _ in range(B)]
        di = {k: torch.from_numpy(np.stack([i[k] for i in inps])).cuda() for k in inps[0]}
        N.linear_attn_step_batched(dw, di["qkv"], di["z"], di["alpha"], di["beta"], dconv, dS, out)
        torch.cuda.synchronize()
        got, gS, gc = out.cpu().numpy(), dS.cpu().numpy(), dconv.cpu().numpy()
        for b in range(B):
            ref = O.linear_attn_step(w, inps[b], conv[b], S[b])
            assert np.abs(got[b] - ref).max() <= TOL * np.abs(ref).max(), (step, b)
            assert np.abs(gS[b] - S[b]).max() <= TOL * max(np.abs(S[b]).max(), 1e-6), (step, b)
            assert np.array_equal(gc[b], conv[b]), (step, b)
