"""CPU, multi-process (gloo): the token-ownership plan of the sharded forward.

Each rank computes its own view of the plan through the C ABI (host only);
the ranks then check with gloo collectives that their independent views
agree: local tokens partition the video tokens, what rank s sends to q is
what q expects from s, and an emulated exchange (gloo send/recv standing in
for the NCCL exchange) delivers exactly the listed tokens.  A second test
kills one rank before the exchange and checks the survivors fail with an
error instead of hanging (process-group timeout).
"""
import os
import socket

import numpy as np
import pytest

from tests.conftest import ROOT

CASES = [([6, 45, 80], [4, 3, 4], 0), ([2, 12, 20], [1, 8, 8], 1), ([3, 7, 11], [2, 3, 4], 1)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, q):
    import sys
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from seedvr2_ncnn_b200 import abi

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=30))
        for shape, window, mode in CASES:
            for shifted in (0, 1):
                _check_case(dist, torch, abi, rank, world, shape, window, mode, T, shifted)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, f"error: {e!r}"))


def _check_case(dist, torch, abi, rank, world, shape, window, mode, T, shifted):
    s = abi.shard(shape, T, window, mode, rank, world, shifted)
    nv = int(np.prod(shape))
    local = torch.from_numpy(s["local_tokens"].astype(np.int64))
    # 1. local tokens partition [0, nv)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([len(local)]))
    mx = int(max(x.item() for x in sizes))
    padded = torch.full((mx,), -1, dtype=torch.int64)
    padded[:len(local)] = local
    allp = [torch.zeros(mx, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(allp, padded)
    every = torch.cat([a[a >= 0] for a in allp]).sort().values
    assert torch.equal(every, torch.arange(nv)), "local tokens do not partition the video tokens"
    assert max(x.item() for x in sizes) - min(x.item() for x in sizes) <= 1, "token ranges are not balanced"
    # 2. send counts of s->q equal recv counts of q<-s
    sc = torch.from_numpy(s["send_counts"].astype(np.int64))
    rc = torch.from_numpy(s["recv_counts"].astype(np.int64))
    all_sc = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(all_sc, sc)
    for src in range(world):
        assert all_sc[src][rank].item() == rc[src].item(), (src, rank)
    # 3. emulated exchange: rows = (token id, 3*id+1); received rows must be the listed tokens
    pos = {int(g): i for i, g in enumerate(s["local_tokens"])}
    rows = torch.stack([local, 3 * local + 1], 1)
    so = np.concatenate([[0], np.cumsum(s["send_counts"])])
    ro = np.concatenate([[0], np.cumsum(s["recv_counts"])])
    recv = torch.zeros((int(rc.sum()), 2), dtype=torch.int64)
    reqs = []
    for p in range(world):
        if p == rank:
            continue
        if s["send_counts"][p]:
            idx = [pos[int(g)] for g in s["send_tokens"][so[p]:so[p + 1]]]
            reqs.append(dist.isend(rows[idx].contiguous(), p))
        if s["recv_counts"][p]:
            buf = torch.zeros((int(s["recv_counts"][p]), 2), dtype=torch.int64)
            reqs.append((dist.irecv(buf, p), buf, p))
    for r in reqs:
        if isinstance(r, tuple):
            r[0].wait()
            p = r[2]
            recv[ro[p]:ro[p + 1]] = r[1]
        else:
            r.wait()
    expect = torch.from_numpy(s["recv_tokens"].astype(np.int64))
    assert torch.equal(recv[:, 0], expect) and torch.equal(recv[:, 1], 3 * expect + 1)
    assert not set(s["recv_tokens"].tolist()) & set(s["local_tokens"].tolist())


def _run(world, fn, *args):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, msg = q.get(timeout=120)
        out[r] = msg
    for p in procs:
        p.join(timeout=60)
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_shard_plans_agree_across_ranks(world):
    out = _run(world, _worker, 58)
    assert all(v == "ok" for v in out.values()), out


def _dying_worker(rank, world, port, q):
    import sys
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))  # this rank leaves between steps, before the exchange
        q.close()
        q.join_thread()  # flush the message before the hard exit
        os._exit(0)
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, f"raised {type(e).__name__}"))


def test_peer_that_leaves_is_reported_not_hung():
    out = _run(2, _dying_worker)
    assert out[1] == "left"
    assert out[0].startswith("raised"), out
