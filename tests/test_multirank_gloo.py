"""Multi-rank host logic on CPU gloo ranks (world 2 and 3): every rank derives the same harmony
plan from all-gathered counts, and the plan-driven chunk exchange moves each (src, expert, dst)
chunk into the receiver's expert-major layout and back.  No kernels run here."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, E, q):
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from dsca_moe_b200.engine import default_expert_to_gpu, exchange_chunks, plan_harmony, plan_layout
    from oracle import oracle as O

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        g = np.random.default_rng(100 + rank)
        T = 200
        ids = g.integers(0, E, size=T)
        ids[: T // 3] = 1  # a hot expert on every rank
        counts = torch.from_numpy(np.bincount(ids, minlength=E).astype(np.int32))
        meta = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(meta, counts)
        meta = torch.stack(meta).numpy()
        e2g = default_expert_to_gpu(E, world)
        S = plan_harmony(meta, e2g, 5)
        assert np.array_equal(S, O.harmony_schedule(meta, e2g, 5))
        lay = plan_layout(S, rank)
        # send buffer in the plan's order; row = [src rank, token, expert, 0...]
        lists = O.expert_token_lists(ids, E)
        rows, exps, splits = O.send_order(S, rank, lists)
        d = 8
        send = torch.zeros(len(rows), d)
        send[:, 0] = rank
        send[:, 1] = torch.from_numpy(rows).float()
        send[:, 2] = torch.from_numpy(exps).float()
        recv = torch.full((int(lay.recv_splits.sum()), d), -1.0)
        exchange_chunks(S, lay, rank, send, recv)
        # receiver: group gi (expert e) rows come from src 0..G-1 in order, every row of expert e
        for gi, e in enumerate(lay.group_expert):
            blk = recv[lay.group_offsets[gi]:lay.group_offsets[gi + 1]]
            assert torch.all(blk[:, 2] == e)
            srcs = blk[:, 0].numpy()
            assert np.all(np.diff(srcs) >= 0)
            for src in range(world):
                assert int((srcs == src).sum()) == int(S[src, e, rank])
        # computing "expert outputs" = rows + 1000 and returning them restores the send layout
        out = recv.clone()
        out[:, 3] = 1000.0 + out[:, 1]
        ret = torch.zeros_like(send)
        exchange_chunks(S, lay, rank, ret, out, reverse=True)
        assert torch.equal(ret[:, :3], send[:, :3])
        assert torch.equal(ret[:, 3], 1000.0 + send[:, 1])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - report to the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,E", [(2, 8), (3, 7), (4, 60)])
def test_plan_and_exchange_on_gloo(world, E):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, E, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res
