"""Expert-parallel forward_batched on 2 GPUs (one process per GPU, token rows exchanged by
NVLink peer stores), against the single-GPU path on the same tokens; and the collective
refusal of ranks whose t_max differ. Needs >= 2 GPUs."""
import os
import subprocess
import sys

import numpy as np
import pytest

import nmoe_b200 as N
from nmoe_testutil import rel_l2, upload
from oracle import oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("counts", [(40, 24), (17, 0)])
def test_ep_two_gpus_matches_single_gpu(tmp_path, counts):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, HERE)
    import ep_worker
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_worker.py"), str(r), "2", str(counts[r]),
                               str(tmp_path)], env=env) for r in range(2)]
    try:
        rcs = [p.wait(timeout=300) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert rcs == [0, 0]
    # single GPU, all tokens
    ctx = N.Context(quant_bits=4, num_layers=1, t_max=64, device=0)
    lw = O.make_layer(300, bits=4, distinct_experts=24)
    upload(ctx, 0, lw)
    for r in range(2):
        T = counts[r]
        if T == 0:
            continue
        xb = ep_worker.tokens(r, T)
        xd = torch.from_numpy(xb.view(np.int16)).cuda()
        out = torch.zeros((T, 2048), dtype=torch.float32, device="cuda")
        idx = torch.zeros((T, 8), dtype=torch.int32, device="cuda")
        ctx.forward_batched(0, T, 8, xd, out, idx_out=idx)
        torch.cuda.synchronize()
        for call in range(2):
            np.testing.assert_array_equal(np.load(tmp_path / f"idx{r}_{call}.npy"), idx.cpu().numpy())
            got = np.load(tmp_path / f"out{r}_{call}.npy")
            assert rel_l2(got, out.cpu().numpy()) < 1e-3, (r, call)


def test_ep_mismatched_t_max_is_refused(tmp_path):
    """The receive slabs have one capacity on every rank: ranks created with different
    t_max all fail with NMOE_EINVAL instead of one of them overrunning another's slab."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_worker.py"), str(r), "2", "8", str(tmp_path),
                               "mismatch"], env=env) for r in range(2)]
    try:
        rcs = [p.wait(timeout=300) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert rcs == [0, 0]
