"""Tensor-parallel host logic without a GPU: the communicator id is made by
rank 0 and shared over a torch.distributed group (two gloo ranks here), and
the NCCL entry points load at run time."""
import os

import pytest


def _worker(rank, ws, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=60))
    try:
        cid = ltx_b200.share_comm_id()
        got = [None] * ws
        dist.all_gather_object(got, cid)
        if rank == 0:
            q.put((len(cid), all(g == cid for g in got)))
    finally:
        dist.destroy_process_group()


def test_comm_id_shared_over_two_gloo_ranks():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    n, same = q.get(timeout=5)
    assert n == 128 and same


def test_comm_unique_ids_differ():
    import ltx_b200
    assert ltx_b200.comm_unique_id() != ltx_b200.comm_unique_id()


def _leaver(rank, ws, port, q, step1_done):
    """Rank 1 leaves between steps; rank 0's next collective must end with an
    error within the process group's short timeout instead of hanging."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)                       # step 1: both ranks
    if rank == 1:
        step1_done.wait(30)                  # rank 0 has finished step 1 too: nothing is in flight
        os._exit(0)                          # leaves without a goodbye
    step1_done.set()
    import time
    t0 = time.time()
    try:
        dist.all_reduce(t)                   # step 2: the peer is gone
        q.put(("no error", time.time() - t0))
    except Exception as e:                   # noqa: BLE001 - any error is the detection
        q.put((type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()                          # the result is in the pipe before the process ends
    os._exit(0)


def test_lost_rank_is_detected_by_the_next_collective():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    step1_done = ctx.Event()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q, step1_done)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    kind, waited = q.get(timeout=5)
    assert kind != "no error" and waited < 30, (kind, waited)


def test_cfg_tp_layout():
    """Ranks [0, n/2) run the conditional pass, [n/2, n) the unconditional one; rank r
    pairs with r + n/2 and each half is one tensor-parallel group."""
    import ltx_b200
    assert ltx_b200.cfg_tp_layout(2, 1) == (1, 1, 0, [1], [0, 1])
    assert ltx_b200.cfg_tp_layout(8, 5) == (1, 4, 1, [4, 5, 6, 7], [1, 5])
    assert ltx_b200.cfg_tp_layout(4, 0) == (0, 2, 0, [0, 1], [0, 2])
    for n in (1, 3):
        with pytest.raises(ValueError):
            ltx_b200.cfg_tp_layout(n, 0)


class _FakeCtx:
    """Records the communicator calls init_cfg_tensor_parallel makes."""
    def __init__(self):
        self.calls = []

    def init_comm(self, cid, n, r):
        self.calls.append(("tp", cid, n, r))

    def init_cfg_comm(self, cid, cfg_rank):
        self.calls.append(("cfg", cid, cfg_rank))


def _cfg_layout_worker(rank, ws, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=60))
    try:
        ctx = _FakeCtx()
        got = ltx_b200.init_cfg_tensor_parallel(ctx)
        allc = [None] * ws
        dist.all_gather_object(allc, (got, ctx.calls))
        if rank == 0:
            q.put(allc)
    finally:
        dist.destroy_process_group()


def test_cfg_tensor_parallel_groups_over_four_gloo_ranks():
    """Four ranks: two tensor-parallel halves {0,1} and {2,3}, CFG pairs {0,2} and
    {1,3}; every member of a group receives the same fresh id, the groups' ids differ."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cfg_layout_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    allc = q.get(timeout=5)
    assert [a[0] for a in allc] == [(0, 2, 0), (0, 2, 1), (1, 2, 0), (1, 2, 1)]
    tp = [c[0] for c in (a[1] for a in allc)]
    cfg = [c[1] for c in (a[1] for a in allc)]
    assert [(t[0], t[2], t[3]) for t in tp] == [("tp", 2, 0), ("tp", 2, 1), ("tp", 2, 0), ("tp", 2, 1)]
    assert tp[0][1] == tp[1][1] and tp[2][1] == tp[3][1] and tp[0][1] != tp[2][1]
    assert [(c[0], c[2]) for c in cfg] == [("cfg", 0), ("cfg", 0), ("cfg", 1), ("cfg", 1)]
    assert cfg[0][1] == cfg[2][1] and cfg[1][1] == cfg[3][1] and cfg[0][1] != cfg[1][1]
