"""Checked layer loads on the GPU: the device CRC-32C of every expert blob equals the host
values (library and bitwise oracle), a mismatch refuses the layer, and the file variant
reads the same image."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [4, 2])
def test_device_crcs_match_host(bits):
    lw = O.make_layer(21 + bits, bits=bits, distinct_experts=8)
    img = lw.experts.view(np.uint8).copy()
    esz = N.expert_size(bits)
    img[5 * esz + 12345] ^= 0x40          # expert 5 differs from its pool twin 13
    host = N.expert_crcs(img, bits)
    ctx = N.Context(quant_bits=bits, num_layers=1)
    got = ctx.load_layer_checked(0, img, expected=host)
    assert np.array_equal(got, host)
    assert got[5] != got[13] and got[6] == got[14]
    for e in (0, 5, 255):
        assert host[e] == O.crc32c(img[e * esz:(e + 1) * esz])
    ctx.close()


def test_mismatch_refuses_the_layer(tmp_path):
    lw = O.make_layer(31, bits=4, distinct_experts=4)
    img = lw.experts.view(np.uint8)
    want = N.expert_crcs(img, 4)
    bad = want.copy()
    bad[77] ^= 1
    ctx = N.Context(quant_bits=4, num_layers=1)
    with pytest.raises(N.NmoeError) as ei:
        ctx.load_layer_checked(0, img, expected=bad)
    assert ei.value.status == N.ECHECKSUM and "expert 77" in str(ei.value)
    # nothing was loaded: a forward on the layer is refused
    ctx.set_dense(0, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    import torch
    x = torch.zeros(2048, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(2048, dtype=torch.float32, device="cuda")
    with pytest.raises(N.NmoeError):
        ctx.forward(0, 8, x, out)
    # the file variant: same CRCs, and a good manifest loads
    path = tmp_path / "layer_00.bin"
    img.tofile(path)
    got = ctx.load_layer_file_checked(0, str(path), expected=want)
    assert np.array_equal(got, want)
    ctx.forward(0, 8, x, out)
    torch.cuda.synchronize()
    ctx.close()
