"""nmoe_moe_forward_static: the batch-1 block for callers that cannot allocate device
memory when they call (their memory belongs to a preallocated pool, or cudaMalloc's
implicit synchronisation is not allowed where they run). It keeps its scratch in an
array compiled into the library. Checked through the C ABI against nmoe_moe_forward on
the same weights and inputs, on two calls in a row (the second reuses the scratch the
first left behind). Collected last on purpose."""
import numpy as np
import pytest

import nmoe_b200 as N
from nmoe_testutil import rel_l2, upload
from oracle import oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _dev(d):
    out = {"weight": torch.from_numpy(d["weight"].view(np.uint8).copy()).cuda()}
    if d.get("scales") is not None:
        out["scales"] = torch.from_numpy(d["scales"].view(np.uint8).copy()).cuda()
        out["biases"] = torch.from_numpy(d["biases"].view(np.uint8).copy()).cuda()
    return out


@pytest.mark.parametrize("bits,rdt,xdt", [(4, N.DTYPE_BF16, N.DTYPE_BF16), (2, N.DTYPE_Q4, N.DTYPE_F32)])
def test_static_forward_matches_context_forward(bits, rdt, xdt):
    lw = O.make_layer(4242, bits=bits, router_dtype=rdt, shared_dtype=rdt, distinct_experts=12)
    ctx = N.Context(quant_bits=bits, num_layers=1, router_dtype=rdt, shared_dtype=rdt, device=0)
    upload(ctx, 0, lw)
    experts = torch.from_numpy(lw.experts).cuda()
    dense = {n: _dev(getattr(lw, n)) for n in ("router", "shared_gate", "shared_up", "shared_down", "shared_gate_vec")}
    rng = np.random.default_rng(3)
    for call in range(2):
        xf = rng.standard_normal(2048, dtype=np.float32)
        xd = (torch.from_numpy(O.f32_to_bf16(xf).view(np.int16)) if xdt == N.DTYPE_BF16 else torch.from_numpy(xf)).cuda()
        hm = torch.randn(2048, device="cuda")
        k = 8 if call == 0 else 5
        o1 = torch.zeros(2048, device="cuda")
        i1 = torch.zeros(8, dtype=torch.int32, device="cuda")
        w1 = torch.zeros(8, device="cuda")
        ctx.forward(0, k, xd, o1, x_dtype=xdt, h_mid=hm, idx_out=i1, w_out=w1)
        o2 = torch.full((2048,), 7.0, device="cuda")
        i2 = torch.full((8,), 99, dtype=torch.int32, device="cuda")
        w2 = torch.full((8,), 3.0, device="cuda")
        N.forward_static(experts, 256, bits, dense, rdt, rdt, k, xd, o2, x_dtype=xdt, h_mid=hm, idx_out=i2, w_out=w2)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(i1.cpu().numpy(), i2.cpu().numpy())
        # the two paths compute the router logits in different fp32 orders (~1e-5 relative)
        np.testing.assert_allclose(w1.cpu().numpy(), w2.cpu().numpy(), rtol=1e-4, atol=1e-6)
        # the context path's routed-expert dots run in half2 (see test_decode_gpu.OUT_TOL)
        assert rel_l2(o2.cpu().numpy(), o1.cpu().numpy()) < 2e-3


@pytest.mark.parametrize("bits,rdt,xdt", [(4, N.DTYPE_BF16, N.DTYPE_BF16), (2, N.DTYPE_Q4, N.DTYPE_F32)])
def test_static_forward_matches_oracle(bits, rdt, xdt):
    """The static path runs fp32 kernels: held to 1e-4 against the CPU oracle, on the
    routing the oracle derives from the GPU's logits (ids must agree exactly)."""
    lw = O.make_layer(5151, bits=bits, router_dtype=rdt, shared_dtype=rdt, distinct_experts=12)
    ctx = N.Context(quant_bits=bits, num_layers=1, router_dtype=rdt, shared_dtype=rdt, device=0)
    upload(ctx, 0, lw)
    experts = torch.from_numpy(lw.experts).cuda()
    dense = {n: _dev(getattr(lw, n)) for n in ("router", "shared_gate", "shared_up", "shared_down", "shared_gate_vec")}
    rng = np.random.default_rng(8)
    for call in range(2):
        xf = rng.standard_normal(2048, dtype=np.float32)
        if xdt == N.DTYPE_BF16:
            xb = O.f32_to_bf16(xf)
            xf = O.bf16_to_f32(xb)
            xd = torch.from_numpy(xb.view(np.int16)).cuda()
        else:
            xd = torch.from_numpy(xf).cuda()
        hm = np.random.default_rng(9 + call).standard_normal(2048, dtype=np.float32)
        k = 8 if call == 0 else 3
        lg = torch.zeros(256, device="cuda")
        ctx.route(0, k, xd, x_dtype=xdt, logits_out=lg)
        out = torch.zeros(2048, device="cuda")
        idx = torch.zeros(8, dtype=torch.int32, device="cuda")
        N.forward_static(experts, 256, bits, dense, rdt, rdt, k, xd, out, x_dtype=xdt,
                         h_mid=torch.from_numpy(hm).cuda(), idx_out=idx)
        torch.cuda.synchronize()
        ref = O.block_forward(lw, k, xf, h_mid=hm, logits_override=lg.cpu().numpy())
        np.testing.assert_array_equal(idx.cpu().numpy()[:k].view(np.uint32), ref["idx"][:k])
        assert rel_l2(out.cpu().numpy(), ref["out"]) < 1e-4, rel_l2(out.cpu().numpy(), ref["out"])
        assert N.static_status() == (N.OK, 0)


def test_static_status_reports_out_of_range_expert():
    """A routed id >= num_experts contributes nothing and leaves the device error word set;
    nmoe_moe_static_status reads it (NMOE_EDEVICE, code 1) and clears it."""
    lw = O.make_layer(77, bits=4, distinct_experts=8)
    r = lw.router["weight"].copy()
    r[250] = r[3]                       # experts 250 and 3 tie at the top: both are picked
    lw.router = {"dtype": N.DTYPE_BF16, "weight": r}
    ne = 200                            # ... but only experts 0..199 exist
    esz = O.expert_size(4)
    experts = torch.from_numpy(lw.experts[: ne * esz].copy()).cuda()
    dense = {n: _dev(getattr(lw, n)) for n in ("router", "shared_gate", "shared_up", "shared_down", "shared_gate_vec")}
    x = O.f32_to_bf16(O.bf16_to_f32(r[3]) * 50.0)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.zeros(2048, device="cuda")
    idx = torch.zeros(8, dtype=torch.int32, device="cuda")
    N.forward_static(experts, ne, 4, dense, N.DTYPE_BF16, N.DTYPE_BF16, 2, xd, out, idx_out=idx)
    torch.cuda.synchronize()
    assert sorted(idx.cpu().numpy()[:2].tolist()) == [3, 250]
    assert N.static_status() == (N.EDEVICE, 1)
    assert N.static_status() == (N.OK, 0)
    assert np.isfinite(out.cpu().numpy()).all()
    assert N.lib().nmoe_moe_static_scratch_bytes() == 19712


def test_static_forward_rejects_k_beyond_scratch():
    x = torch.zeros(2048, dtype=torch.int16, device="cuda")
    out = torch.zeros(2048, device="cuda")
    dummy = {"weight": x}
    dense = {n: dummy for n in ("router", "shared_gate", "shared_up", "shared_down", "shared_gate_vec")}
    for k in (0, 9):
        with pytest.raises(N.NmoeError) as ei:
            N.forward_static(x, 256, 4, dense, N.DTYPE_BF16, N.DTYPE_BF16, k, x, out)
        assert ei.value.status == N.EINVAL and "8" in str(ei.value)
