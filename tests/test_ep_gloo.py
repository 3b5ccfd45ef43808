"""Expert-parallel dispatch and combine on two CPU ranks (gloo), against the
single-process routed sum.

This mirrors the plan nmoe_moe_forward_batched follows when world_size > 1: every rank
routes its own tokens over all 256 experts; (token, slot) rows are ordered by global
expert, so each destination rank's rows form one contiguous segment; ranks exchange the
per-expert counts, then the rows; each rank applies its own experts (32 per rank at 8
GPUs, 128 here) to the rows it received, in (source rank, local expert) order; the
outputs go back to their source ranks in the order they were sent, and the source
combines sum_s w_s * down_s. Gate/up/down use the oracle's expert functions, so the EP
result must equal the local one exactly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

W, T, K, E = 2, 6, 4, 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expert(lw, e, x):
    L = O.lib()
    blob = np.ascontiguousarray(lw.experts[e * O.expert_size(lw.bits):(e + 1) * O.expert_size(lw.bits)])
    act = np.zeros(512, np.float32)
    out = np.zeros(2048, np.float32)
    L.orc_expert_gate_up(blob, lw.bits, np.ascontiguousarray(x, np.float32), act)
    L.orc_expert_down(blob, lw.bits, act, out)
    return out


def _worker(rank, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=W)
        lw = O.make_layer(11, bits=4, distinct_experts=6)
        x = np.random.default_rng(100 + rank).standard_normal((T, 2048), dtype=np.float32)
        nl = E // W
        # route (oracle logits) and order (token, slot) rows by global expert, then token
        idx, w = np.zeros((T, K), np.int64), np.zeros((T, K), np.float32)
        for t in range(T):
            r = O.block_forward(lw, K, x[t])
            idx[t], w[t] = r["idx"][:K], r["w"][:K]
        rows = sorted(((int(idx[t, s]), t, s) for t in range(T) for s in range(K)))
        pos = {(t, s): p for p, (_, t, s) in enumerate(rows)}
        cnt = np.bincount([e for e, _, _ in rows], minlength=E).astype(np.int64)
        # exchange counts: rank p gets cnt[p*nl:(p+1)*nl] from every source
        rcnt = [torch.zeros(nl, dtype=torch.int64) for _ in range(W)]
        for p in range(W):
            if p == rank:
                rcnt[p] = torch.from_numpy(cnt[p * nl:(p + 1) * nl].copy())
        reqs = []
        for p in range(W):
            if p != rank:
                reqs.append(dist.isend(torch.from_numpy(cnt[p * nl:(p + 1) * nl].copy()), p))
                reqs.append(dist.irecv(rcnt[p], p))
        for r_ in reqs:
            r_.wait()
        scnt = [int(cnt[p * nl:(p + 1) * nl].sum()) for p in range(W)]
        soff = np.concatenate([[0], np.cumsum(scnt)])
        send = np.stack([x[t] for _, t, _ in rows])
        recv = [None] * W
        reqs = []
        for p in range(W):
            n_in = int(rcnt[p].sum())
            recv[p] = torch.zeros((n_in, 2048), dtype=torch.float32)
            if p == rank:
                recv[p] = torch.from_numpy(send[soff[p]:soff[p + 1]].copy())
            else:
                reqs.append(dist.isend(torch.from_numpy(send[soff[p]:soff[p + 1]].copy()), p))
                reqs.append(dist.irecv(recv[p], p))
        for r_ in reqs:
            r_.wait()
        # apply this rank's experts in (source, local expert) order
        back = []
        for p in range(W):
            y = np.zeros((recv[p].shape[0], 2048), np.float32)
            i = 0
            for j in range(nl):
                for _ in range(int(rcnt[p][j])):
                    y[i] = _expert(lw, rank * nl + j, recv[p][i].numpy())
                    i += 1
            back.append(torch.from_numpy(y))
        # return outputs; they arrive in send order
        ret = [None] * W
        reqs = []
        for p in range(W):
            ret[p] = torch.zeros((scnt[p], 2048), dtype=torch.float32)
            if p == rank:
                ret[p] = back[p]
            else:
                reqs.append(dist.isend(back[p], p))
                reqs.append(dist.irecv(ret[p], p))
        for r_ in reqs:
            r_.wait()
        yall = torch.cat(ret).numpy()
        ep = np.zeros((T, 2048), np.float32)
        local = np.zeros((T, 2048), np.float32)
        for t in range(T):
            for s in range(K):
                ep[t] += w[t, s] * yall[pos[(t, s)]]
                local[t] += w[t, s] * _expert(lw, int(idx[t, s]), x[t])
        q.put((rank, float(np.abs(ep - local).max()), sorted(set(scnt))))
        dist.destroy_process_group()
    except Exception as ex:  # surface worker failures to the test
        q.put((rank, repr(ex), None))


def test_ep_dispatch_combine_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(W)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(W)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, _ in res:
        assert isinstance(err, float), err
        assert err == 0.0, (rank, err)
