"""Whole decode step (nmoe_decoder_step) against the oracle's restatement of
NMOEProcessToken over several tokens fed back autoregressively: 4 layers (3 linear
attention + 1 full attention, the model's pattern), the fp32 routed-expert path, vocab
512. The last hidden state within 1e-3 relative L2; the token equal to the oracle's
wherever the oracle's top-2 logit gap exceeds the logits' error bound."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O
from nmoe_testutil import upload

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("head_dtype", [N.DTYPE_Q4, N.DTYPE_BF16])
def test_decode_steps_match_oracle(head_dtype):
    import torch
    L, V = 4, 512
    layers, g = O.make_decoder_weights(3, L, V, head_dtype=head_dtype, embed_dtype=head_dtype)
    moe = [O.make_layer(20 + l, distinct_experts=4) for l in range(L)]
    ctx = N.Context(quant_bits=4, num_layers=L, flags=N.FLAG_EXPERT_FP32)
    for l in range(L):
        upload(ctx, l, moe[l])
    dec = N.Decoder(ctx, L, k=8, max_positions=16)
    for l in range(L):
        dec.set_layer(l, layers[l])
    dec.set_globals(g)
    ref = O.DecoderOracle(layers, g, moe, max_positions=16)
    tok = torch.tensor([5], dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    hid = torch.zeros(2048, device="cuda")
    t_host = 5
    for pos in range(5):
        dec.step(tok, pos, nxt, hid)
        otok, oh, ologits = ref.step(t_host, pos)
        torch.cuda.synchronize()
        gh = hid.cpu().numpy()
        rel = np.linalg.norm(gh - oh) / np.linalg.norm(oh)
        assert rel <= 1e-3, (pos, rel)
        gt = int(nxt.item())
        top2 = np.sort(ologits)[-2:]
        if top2[1] - top2[0] > 2e-3 * np.abs(ologits).max():
            assert gt == otok, (pos, gt, otok)
        # feed the oracle's token to both, so that the two stay on one sequence
        t_host = otok
        tok.fill_(otok)
    dec.close()
    ctx.close()


def test_unset_layer_is_refused():
    import torch
    ctx = N.Context(quant_bits=4, num_layers=4)
    dec = N.Decoder(ctx, 4, max_positions=4)
    t = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(N.NmoeError):
        dec.step(t, 0, t)
    dec.close()
    ctx.close()
