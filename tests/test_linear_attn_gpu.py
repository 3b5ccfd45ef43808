"""nmoe_linear_attn_step on the GPU against the oracle over several steps with the
recurrent states carried: conv state bit-exact (pure copies), recurrent state and output
within 2e-5 of the largest magnitude (fp32, sums in another order)."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _dev(a, torch):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda()
    return torch.from_numpy(a.copy()).cuda()


@pytest.mark.parametrize("seed", [1, 2])
def test_steps_match_oracle(seed):
    import torch
    w = O.make_linear_attn(seed)
    dw = {k: _dev(v, torch) for k, v in w.items()}
    rng = np.random.default_rng(100 + seed)
    conv = np.zeros((3, 8192), np.float32)
    S = (rng.standard_normal((32, 128, 128)) * 0.05).astype(np.float32) if seed == 2 else np.zeros((32, 128, 128), np.float32)
    dconv, dS = _dev(conv, torch), _dev(S, torch)
    out = torch.zeros(4096, device="cuda")
    for step in range(6):
        inp = O.linear_attn_inputs(rng)
        di = {k: _dev(v, torch) for k, v in inp.items()}
        N.linear_attn_step(dw, di["qkv"], di["z"], di["alpha"], di["beta"], dconv, dS, out)
        ref = O.linear_attn_step(w, inp, conv, S)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.abs(got - ref).max() <= TOL * np.abs(ref).max(), (step, np.abs(got - ref).max())
        gS = dS.cpu().numpy()
        assert np.abs(gS - S).max() <= TOL * max(np.abs(S).max(), 1e-6), step
        assert np.array_equal(dconv.cpu().numpy(), conv), step


def test_rejects_null_and_misaligned():
    import torch
    w = O.make_linear_attn(1)
    dw = {k: _dev(v, torch) for k, v in w.items()}
    buf = torch.zeros(32 * 128 * 128 + 8, device="cuda")
    with pytest.raises(N.NmoeError):
        N.linear_attn_step(dw, buf, buf, buf, buf, buf, buf.data_ptr() + 4, buf)
    with pytest.raises(N.NmoeError):
        N.linear_attn_step(dw, None, buf, buf, buf, buf, buf, buf)
