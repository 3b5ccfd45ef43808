"""One rank of the expert-parallel GPU test (tests/test_ep_gpu.py): creates a
world_size-W context on GPU `rank`, runs forward_batched on this rank's tokens and saves
the outputs."""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(HERE, ".."), os.path.join(HERE, "..", "nano-metal-moe-qwen36_b200")]

import torch  # noqa: E402

import nmoe_b200 as N  # noqa: E402
from nmoe_testutil import upload  # noqa: E402
from oracle import oracle as O  # noqa: E402


def tokens(rank, T):
    x = np.random.default_rng(500 + rank).standard_normal((T, 2048), dtype=np.float32)
    return O.f32_to_bf16(x)


def main():
    rank, world, T, workdir = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    idfile = os.path.join(workdir, "nccl.id")
    if rank == 0:
        with open(idfile + ".tmp", "wb") as f:
            f.write(N.nccl_unique_id())
        os.replace(idfile + ".tmp", idfile)
    t0 = time.time()
    while not os.path.exists(idfile):
        if time.time() - t0 > 60:
            raise SystemExit("no NCCL id")
        time.sleep(0.05)
    uid = open(idfile, "rb").read()
    torch.cuda.set_device(rank)
    if len(sys.argv) > 5 and sys.argv[5] == "mismatch":
        # rank 1 asks for a different t_max: every rank must refuse the context
        try:
            N.Context(quant_bits=4, num_layers=1, t_max=64 if rank == 0 else 32, device=rank, world_size=world,
                      rank=rank, nccl_unique_id=uid)
        except N.NmoeError as ex:
            assert ex.status == N.EINVAL and "t_max" in str(ex), ex
            return
        raise SystemExit("a context with mismatched t_max was created")
    ctx = N.Context(quant_bits=4, num_layers=1, t_max=64, device=rank, world_size=world, rank=rank,
                    nccl_unique_id=uid)
    lw = O.make_layer(300, bits=4, distinct_experts=24)
    upload(ctx, 0, lw)
    xb = tokens(rank, T)
    xd = torch.from_numpy(xb.view(np.int16)).cuda()
    for call in range(2):
        out = torch.zeros((max(T, 1), 2048), dtype=torch.float32, device="cuda")
        idx = torch.zeros((max(T, 1), 8), dtype=torch.int32, device="cuda")
        ctx.forward_batched(0, T, 8, xd, out, idx_out=idx)
        torch.cuda.synchronize()
        np.save(os.path.join(workdir, f"out{rank}_{call}.npy"), out.cpu().numpy()[:T])
        np.save(os.path.join(workdir, f"idx{rank}_{call}.npy"), idx.cpu().numpy()[:T])
    assert ctx.device_status() == (0, 0)
    ctx.close()


if __name__ == "__main__":
    main()
