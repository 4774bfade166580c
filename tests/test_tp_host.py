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
