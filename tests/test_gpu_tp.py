"""Tensor-parallel model (heads and FFN units split over two GPUs, a sum over
ranks after each row-split projection) against the same model on one GPU.
The sum runs every way the library has: fused into the GEMM over NVLink peer
memory (the default), the same with sequence-parallel norms
(LTX_TP_SEQ_NORMS=1), and as an NCCL allreduce (LTX_TP_EXCHANGE=nccl).

Needs two GPUs; each rank is a spawned process.  The whole model on one GPU
is the reference: same seed, same synthetic FP8 + LoRA weights (every shard
count generates the full tensors, then keeps its part), same inputs.  The
ranks' sums come in a different order than the single GPU's fused epilogue,
so the comparison is by relative L2, not bits.
"""
import json
import os

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def _cfg(heads, head_dim, layers):
    from dit_checkpoint import small_config
    return small_config(heads=heads, head_dim=head_dim, layers=layers)


def _worker(rank, ws, port, cfg, T_frames, q, exchange="peer"):
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    from oracle import sampler
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if exchange == "nccl":
        os.environ["LTX_TP_EXCHANGE"] = "nccl"
    if exchange == "peer_sp":   # sequence-parallel norms (inner dimension 4096)
        os.environ["LTX_TP_SEQ_NORMS"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=90))
    try:
        ctx = ltx_b200.Context(rank)
        ltx_b200.init_tensor_parallel(ctx)
        cj = json.dumps(cfg)
        model = ltx_b200.VideoTransformer.init_random(ctx, cj, seed=21, lora_rank=8, lora_strength=0.8)
        F, Hh, W, S = T_frames, 8, 8, 40
        rng = np.random.default_rng(4)
        Tt = F * Hh * W
        T = 2 * Tt
        C, Dc = cfg["in_channels"], cfg["cross_attention_dim"]
        lat = rng.standard_normal((1, T, C)).astype(np.float32)
        ts = np.concatenate([np.full(Tt, 0.6, np.float32), np.zeros(Tt, np.float32)])[None]
        pos = np.concatenate([sampler.target_positions(F, Hh, W), sampler.reference_positions(F, Hh, W)], axis=2)
        ctxt = rng.standard_normal((1, S, Dc)).astype(np.float32)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        out = torch.empty(lat.shape, device="cuda")
        model.forward(dev(lat), dev(ts), dev(pos), dev(ctxt), out)
        # one guided Euler step on the replicated latent
        clean = np.concatenate([np.zeros((Tt, C), np.float32), rng.standard_normal((Tt, C)).astype(np.float32)])
        mask = np.concatenate([np.ones(Tt, np.float32), np.zeros(Tt, np.float32)])
        unc = rng.standard_normal((S, Dc)).astype(np.float32)
        lat_s = dev(lat[0])
        model.denoise_step(lat_s, dev(clean), dev(mask), dev(pos), dev(ctxt[0]), dev(unc), 0.8, 0.6, 3.0, 0.7)
        ctx.synchronize()
        ctx.comm_check()
        used = ctx.tp_exchange()
        got_f, got_s = out.cpu().numpy(), lat_s.cpu().numpy()
        outs = [None] * ws
        dist.all_gather_object(outs, (got_f, got_s))
        if rank == 0:
            # the whole model on this GPU, no communicator
            ctx1 = ltx_b200.Context(0)
            m1 = ltx_b200.VideoTransformer.init_random(ctx1, cj, seed=21, lora_rank=8, lora_strength=0.8)
            ref = torch.empty(lat.shape, device="cuda")
            m1.forward(dev(lat), dev(ts), dev(pos), dev(ctxt), ref)
            lat1 = dev(lat[0])
            m1.denoise_step(lat1, dev(clean), dev(mask), dev(pos), dev(ctxt[0]), dev(unc), 0.8, 0.6, 3.0, 0.7)
            ctx1.synchronize()
            ref_f, ref_s = ref.cpu().numpy(), lat1.cpu().numpy()
            same_ranks = all(np.array_equal(o[0], outs[0][0]) and np.array_equal(o[1], outs[0][1]) for o in outs)
            q.put((same_ranks, used, _rel_l2(got_f, ref_f), _rel_l2(got_s - lat[0], ref_s - lat[0])))
            m1.close()
            ctx1.close()
        model.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("heads,head_dim,layers,frames,exchange",
                         [(4, 128, 2, 2, "peer"), (32, 128, 1, 1, "peer"), (4, 128, 2, 2, "nccl"),
                          (32, 128, 2, 1, "peer_sp")])
def test_tensor_parallel_two_gpus_matches_one(heads, head_dim, layers, frames, exchange):
    import socket
    import torch.multiprocessing as mp
    cfg = _cfg(heads, head_dim, layers)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_worker, args=(r, 2, port, cfg, frames, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same, used, err_f, err_s = q.get(timeout=5)
    print(f"\nTP x2 ({heads} heads, {layers} layers, {used}): forward rel-L2 {err_f:.2e}, "
          f"step update rel-L2 {err_s:.2e}")
    assert used == exchange.split("_")[0]
    assert same, "ranks disagree on the replicated output"
    assert err_f < 1e-2 and err_s < 1e-2


def _cfg_pair_worker(rank, ws, port, cfg, q):
    """CFG-parallel pair: rank 0 runs the conditional pass, rank 1 the unconditional
    one; every step all-gathers the two velocities and both ranks update the latent."""
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    from oracle import sampler
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=90))
    try:
        ctx = ltx_b200.Context(rank)
        assert ltx_b200.init_cfg_tensor_parallel(ctx) == (rank, 1, 0)
        cj = json.dumps(cfg)
        model = ltx_b200.VideoTransformer.init_random(ctx, cj, seed=23, lora_rank=8, lora_strength=0.8)
        F, Hh, W, S = 2, 8, 8, 40
        rng = np.random.default_rng(6)
        Tt = F * Hh * W
        T = 2 * Tt
        C, Dc = cfg["in_channels"], cfg["cross_attention_dim"]
        lat = rng.standard_normal((T, C)).astype(np.float32)
        pos = np.concatenate([sampler.target_positions(F, Hh, W), sampler.reference_positions(F, Hh, W)], axis=2)
        ctxt = rng.standard_normal((S, Dc)).astype(np.float32)
        unc = rng.standard_normal((S, Dc)).astype(np.float32)
        clean = np.concatenate([np.zeros((Tt, C), np.float32), rng.standard_normal((Tt, C)).astype(np.float32)])
        mask = np.concatenate([np.ones(Tt, np.float32), np.zeros(Tt, np.float32)])
        sig = np.array([1.0, 0.9, 0.7, 0.4], np.float32)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()

        def run(m):
            step = dev(lat)
            m.denoise_step(step, dev(clean), dev(mask), dev(pos), dev(ctxt), dev(unc), 0.8, 0.6, 3.0, 0.7)
            loop = dev(lat)
            m.denoise_loop(loop, dev(clean), dev(mask), dev(pos), dev(ctxt), dev(unc), sig, 3.0, 0.7)
            return step, loop

        step, loop = run(model)
        ctx.synchronize()
        ctx.comm_check()
        got = (step.cpu().numpy(), loop.cpu().numpy())
        outs = [None] * ws
        dist.all_gather_object(outs, got)
        if rank == 0:
            ctx1 = ltx_b200.Context(0)   # both passes as one batch-2 forward, no communicator
            m1 = ltx_b200.VideoTransformer.init_random(ctx1, cj, seed=23, lora_rank=8, lora_strength=0.8)
            r_step, r_loop = run(m1)
            ctx1.synchronize()
            ref = (r_step.cpu().numpy(), r_loop.cpu().numpy())
            same_ranks = all(np.array_equal(o[i], outs[0][i]) for o in outs for i in range(2))
            bits = all(np.array_equal(got[i], ref[i]) for i in range(2))
            q.put((same_ranks, bits, _rel_l2(got[0] - lat, ref[0] - lat), _rel_l2(got[1] - lat, ref[1] - lat)))
            m1.close()
            ctx1.close()
        model.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_cfg_pair_two_gpus_matches_batch2():
    """The pair's two batch-1 passes and the single GPU's batch-2 forward compute the
    same rows (every kernel is row-wise or per batch row), so the step and a 3-step
    loop match the single GPU's; the bar is rel-L2 <= 1e-5 of the update, and the run
    reports whether the bits agree."""
    import socket
    import torch.multiprocessing as mp
    cfg = _cfg(4, 128, 2)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_cfg_pair_worker, args=(r, 2, port, cfg, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same, bits, err_step, err_loop = q.get(timeout=5)
    print(f"\nCFG pair x2: step update rel-L2 {err_step:.2e}, 3-step loop rel-L2 {err_loop:.2e}, bit-identical {bits}")
    assert same, "the pair's ranks disagree on the latent"
    assert err_step < 1e-5 and err_loop < 1e-5


def _cfg_tp_worker(rank, ws, port, cfg, q):
    """CFG-parallel x tensor-parallel on four GPUs: ranks {0,1} run the conditional
    pass split over two GPUs, {2,3} the unconditional one; the pairs {0,2}, {1,3}
    all-gather the velocities."""
    import torch.distributed as dist
    from datetime import timedelta
    import ltx_b200
    from oracle import sampler
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=90))
    try:
        ctx = ltx_b200.Context(rank)
        layout = ltx_b200.init_cfg_tensor_parallel(ctx)
        cj = json.dumps(cfg)
        model = ltx_b200.VideoTransformer.init_random(ctx, cj, seed=29, lora_rank=8, lora_strength=0.8)
        F, Hh, W, S = 2, 8, 8, 40
        rng = np.random.default_rng(8)
        Tt = F * Hh * W
        T = 2 * Tt
        C, Dc = cfg["in_channels"], cfg["cross_attention_dim"]
        lat = rng.standard_normal((T, C)).astype(np.float32)
        pos = np.concatenate([sampler.target_positions(F, Hh, W), sampler.reference_positions(F, Hh, W)], axis=2)
        ctxt = rng.standard_normal((S, Dc)).astype(np.float32)
        unc = rng.standard_normal((S, Dc)).astype(np.float32)
        clean = np.concatenate([np.zeros((Tt, C), np.float32), rng.standard_normal((Tt, C)).astype(np.float32)])
        mask = np.concatenate([np.ones(Tt, np.float32), np.zeros(Tt, np.float32)])
        sig = np.array([1.0, 0.8, 0.5], np.float32)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()

        def run(m):
            loop = dev(lat)
            m.denoise_loop(loop, dev(clean), dev(mask), dev(pos), dev(ctxt), dev(unc), sig, 3.0, 0.7)
            return loop

        got = run(model)
        ctx.synchronize()
        ctx.comm_check()
        used = ctx.tp_exchange()
        got = got.cpu().numpy()
        outs = [None] * ws
        dist.all_gather_object(outs, (layout, used, got))
        if rank == 0:
            ctx1 = ltx_b200.Context(0)
            m1 = ltx_b200.VideoTransformer.init_random(ctx1, cj, seed=29, lora_rank=8, lora_strength=0.8)
            ref = run(m1)
            ctx1.synchronize()
            ref = ref.cpu().numpy()
            same = all(np.array_equal(o[2], outs[0][2]) for o in outs)
            q.put(([o[0] for o in outs], [o[1] for o in outs], same, _rel_l2(got - lat, ref - lat)))
            m1.close()
            ctx1.close()
        model.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_cfg_x_tensor_parallel_four_gpus_matches_one():
    import socket
    import torch.multiprocessing as mp
    cfg = _cfg(4, 128, 2)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_cfg_tp_worker, args=(r, 4, port, cfg, q)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    layouts, used, same, err = q.get(timeout=5)
    print(f"\nCFG x TP (2 x 2): 2-step loop update rel-L2 {err:.2e}, exchanges {used}")
    assert layouts == [(0, 2, 0), (0, 2, 1), (1, 2, 0), (1, 2, 1)]
    assert used == ["peer"] * 4
    assert same, "the four ranks disagree on the latent"
    assert err < 1e-2


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_tensor_parallel_four_gpus_matches_one():
    """Heads and FFN units split four ways (inner dimension 4096: the fused exchange
    with sequence-parallel norms, the default from 4 ranks) against one GPU."""
    import socket
    import torch.multiprocessing as mp
    cfg = _cfg(32, 128, 1)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_worker, args=(r, 4, port, cfg, 1, q, "peer")) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same, used, err_f, err_s = q.get(timeout=5)
    print(f"\nTP x4 (32 heads, 1 layer, {used}): forward rel-L2 {err_f:.2e}, step update rel-L2 {err_s:.2e}")
    assert used == "peer"
    assert same, "ranks disagree on the replicated output"
    assert err_f < 1e-2 and err_s < 1e-2
