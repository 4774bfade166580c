"""Seam crossfade on the device (ltx_seam_blend, ltx_chunk_assemble) against
the oracle's Blender, bit-exact (crates/ltx-chunk/src/blend.rs), and the
chunk-parallel seam exchange over NCCL when the box has two GPUs."""
import os

import numpy as np
import pytest
import torch

from oracle import chunks as oc

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("frames,fv,offset", [(8, 1024, 0), (16, 4 * 24 * 16 * 128 // 4, 0), (6, 333, 0),
                                               (3, 1000, 1), (1, 7, 0), (2, 128 * 384, 3)])
def test_seam_blend_bit_exact(frames, fv, offset):
    import ltx_b200
    ctx = ltx_b200.Context(0)
    g = torch.Generator().manual_seed(frames * 7 + fv)
    old = torch.randn(frames * fv + offset, generator=g) * 3
    new = torch.randn(frames * fv + offset, generator=g) * 3
    o_d, n_d = old.cuda(), new.cuda()
    # offset > 0 makes the pointers unaligned for float4 (scalar path)
    o_v, n_v = o_d[offset:].view(frames, fv), n_d[offset:].view(frames, fv)
    dst = torch.full((frames, fv), float("nan"), device="cuda")
    ltx_b200.seam_blend(ctx, o_v, n_v, dst)
    # in place on the incoming head, as the chunk-parallel path uses it
    ltx_b200.seam_blend(ctx, o_v, n_v, n_v)
    ctx.synchronize()
    want = np.stack([oc.blend_frame(old[offset:].view(frames, fv)[i].numpy(), new[offset:].view(frames, fv)[i].numpy(),
                                    oc.crossfade_weight(i, frames)) for i in range(frames)])
    assert np.array_equal(_bits(dst.cpu().numpy()), _bits(want))
    assert np.array_equal(_bits(n_v.cpu().numpy()), _bits(want))
    ctx.close()


@pytest.mark.parametrize("total,chunk_len,overlap,fv", [
    (26, 17, 8, 64), (28, 17, 8, 64), (40, 17, 8, 50), (100, 17, 8, 64), (18, 17, 8, 16),
    (17, 17, 8, 64), (5, 17, 8, 4), (226, 121, 16, 1024),
    # latent frames of the config-4 clip: 16 latent frames a chunk, 2 shared, 24x16 tokens x 128 channels
    (30, 17, 8, 24 * 16 * 128 // 8),
])
def test_chunk_assemble_matches_blender(total, chunk_len, overlap, fv):
    import ltx_b200
    ctx = ltx_b200.Context(0)
    plan = ltx_b200.chunk_plan(total, chunk_len, overlap)
    assert plan == oc.plan(total, chunk_len, overlap)
    rng = np.random.default_rng(total + fv)
    frames = [rng.standard_normal((e - s, fv), dtype=np.float32) for s, e, _ in plan]
    dev = [torch.from_numpy(f).cuda() for f in frames]
    dst = torch.full((total, fv), float("nan"), device="cuda")
    ltx_b200.chunk_assemble(ctx, dev, plan, dst)
    ctx.synchronize()
    want = oc.assemble(frames, plan, chunk_len, overlap)
    assert np.array_equal(_bits(dst.cpu().numpy()), _bits(want))
    ctx.close()


def test_chunk_assemble_rejects_bad_plans():
    import ltx_b200
    ctx = ltx_b200.Context(0)
    a = torch.zeros(17, 4, device="cuda")
    dst = torch.zeros(40, 4, device="cuda")
    for bad in ([(1, 17, 0)], [(0, 17, 0), (9, 26, 7)], [(0, 17, 0), (9, 26, 8), (12, 29, 14)]):
        with pytest.raises(ltx_b200.LtxError) as e:
            ltx_b200.chunk_assemble(ctx, [a] * len(bad), bad, dst)
        assert e.value.kind == "INVALID_ARG"
    ctx.close()


def _nccl_worker(rank, ws, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    from ltx_b200 import chunks as cp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = ltx_b200.Context(rank)
        total, chunk_len, overlap, fv = 2 * 121 - 16, 121, 16, 4096
        plan = ltx_b200.chunk_plan(total, chunk_len, overlap)
        asg = cp.assign(len(plan), ws)
        rng = np.random.default_rng(9)
        frames = [rng.standard_normal((e - s, fv), dtype=np.float32) for s, e, _ in plan]
        data = {n: torch.from_numpy(frames[n]).cuda() for n in asg[rank]}
        recv = cp.exchange_seams(plan, asg, rank, data)
        cp.blend_seams(ctx, plan, recv, data)
        clip = cp.gather_clip(plan, asg, rank, data, (total, fv))
        torch.cuda.synchronize()
        if rank == 0:
            want = oc.assemble(frames, plan, chunk_len, overlap)
            q.put(bool(np.array_equal(_bits(clip.cpu().numpy()), _bits(want))))
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_chunk_parallel_nccl_two_gpus():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True
