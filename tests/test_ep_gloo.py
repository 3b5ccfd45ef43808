"""Expert-parallel dispatch and combine on two CPU ranks (gloo), against the
single-process routed sum.

This mirrors the plan nmoe_moe_forward_batched follows when world_size > 1 (the device
does it with NVLink peer stores; here fixed-size gloo messages stand in for them): every
rank routes its own tokens over all 256 experts; (token, slot) rows are ordered by global
expert, so each destination rank's rows form one contiguous segment; each rank writes its
segment into slab `rank` (fixed capacity C = T_max * K rows, so no sizes are exchanged
first) of the destination's receive buffer, together with its per-expert counts and the
segment's first position; the destination applies its own experts (128 per rank here, 32
at 8 GPUs) to every slab in (source rank, local expert) order and writes each output back
into the source's return buffer at the position the row left from; the source combines
sum_s w_s * down_s. Gate/up/down use the oracle's expert functions, so the EP result must
equal the local one exactly. Rank 1 has fewer tokens than rank 0."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

W, K, E = 2, 4, 256
T_RANK = (6, 3)
C = max(T_RANK) * K   # slab capacity: every token could send all K rows to one rank


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
        T = T_RANK[rank]
        lw = O.make_layer(11, bits=4, distinct_experts=6)
        x = np.random.default_rng(100 + rank).standard_normal((T, 2048), dtype=np.float32)
        nl = E // W
        idx, w = np.zeros((T, K), np.int64), np.zeros((T, K), np.float32)
        for t in range(T):
            r = O.block_forward(lw, K, x[t])
            idx[t], w[t] = r["idx"][:K], r["w"][:K]
        rows = sorted(((int(idx[t, s]), t, s) for t in range(T) for s in range(K)))
        pos = {(t, s): p for p, (_, t, s) in enumerate(rows)}
        cnt = np.bincount([e for e, _, _ in rows], minlength=E).astype(np.int64)
        off = np.concatenate([[0], np.cumsum(cnt)])          # first position of each expert's rows

        def exchange(msgs):   # one fixed-size message to every rank (self included)
            got = [None] * W
            reqs = []
            for p in range(W):
                if p == rank:
                    got[p] = msgs[p].clone()
                else:
                    got[p] = torch.zeros_like(msgs[p])
                    reqs.append(dist.isend(msgs[p], p))
                    reqs.append(dist.irecv(got[p], p))
            for r_ in reqs:
                r_.wait()
            return got

        # dispatch: slab for destination p = rows of experts [p*nl, (p+1)*nl), then counts, offset
        msgs = []
        for p in range(W):
            slab = np.zeros((C, 2048), np.float32)
            for e, t, s in rows:
                if e // nl == p:
                    slab[pos[(t, s)] - off[p * nl]] = x[t]
            meta = np.concatenate([cnt[p * nl:(p + 1) * nl], [off[p * nl]]]).astype(np.float32)
            msgs.append(torch.from_numpy(np.concatenate([slab.ravel(), meta])))
        recv = exchange(msgs)
        # this rank's experts over every source's slab, in (source, local expert) order;
        # outputs written into a return message at the source's positions
        back = []
        for r in range(W):
            m = recv[r].numpy()
            slab = m[: C * 2048].reshape(C, 2048)
            rc = m[C * 2048: C * 2048 + nl].astype(np.int64)
            first = int(m[-1])
            ret = np.zeros((C, 2048), np.float32)
            i = 0
            for j in range(nl):
                for _ in range(int(rc[j])):
                    ret[first + i] = _expert(lw, rank * nl + j, slab[i])
                    i += 1
            back.append(torch.from_numpy(ret.ravel()))
        rets = exchange(back)
        yret = sum(r.numpy().reshape(C, 2048) for r in rets)   # owners write disjoint positions
        ep = np.zeros((T, 2048), np.float32)
        local = np.zeros((T, 2048), np.float32)
        for t in range(T):
            for s in range(K):
                ep[t] += w[t, s] * yret[pos[(t, s)]]
                local[t] += w[t, s] * _expert(lw, int(idx[t, s]), x[t])
        q.put((rank, float(np.abs(ep - local).max()) if T else 0.0, int(cnt.sum())))
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
