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


# ── seam keyframes: ImageKeyframeCondition on the device, the sequential chunk loop ──

def test_apply_keyframe_bit_exact():
    """ltx_apply_keyframe against oracle/sampler.apply_keyframe (Burn's clean*keep + img*frame,
    mask*keep + frame*(1-strength)): bit-exact, -0.0 values included."""
    import ltx_b200
    from oracle import sampler as osam
    ctx = ltx_b200.Context(0)
    rng = np.random.default_rng(4)
    T, C, tpf = 6 * 20, 7, 20
    for frame, strength in ((0, 0.95), (3, 0.3), (5, 1.0), (2, 0.0)):
        clean = rng.standard_normal((1, T, C)).astype(np.float32)
        clean[0, :3, 0] = -0.0
        mask = rng.choice(np.array([0.0, 1.0, -0.0, 0.25], np.float32), size=(1, T, 1))
        img = rng.standard_normal((1, C, 1, 4, 5)).astype(np.float32)
        img[0, 0, 0, 0, :2] = -0.0
        st = osam.LatentState(np.zeros((1, T, C), np.float32), mask, None, clean)
        exp = osam.apply_keyframe(st, img, frame, tpf, strength)
        cd, md = torch.from_numpy(clean[0].copy()).cuda(), torch.from_numpy(mask[0, :, 0].copy()).cuda()
        ltx_b200.apply_keyframe(ctx, cd, md, torch.from_numpy(img[0]).cuda(), frame, strength)
        ctx.synchronize()
        assert np.array_equal(cd.cpu().numpy().view(np.uint32), exp.clean_latent[0].view(np.uint32))
        assert np.array_equal(md.cpu().numpy().view(np.uint32), exp.denoise_mask[0, :, 0].view(np.uint32))
    z = torch.zeros(T, C, device="cuda")
    m = torch.zeros(T, device="cuda")
    for frame, strength, kind in ((0, 1.5, "STRENGTH"), (0, float("nan"), "STRENGTH"), (6, 0.9, "SHAPE")):
        with pytest.raises(ltx_b200.LtxError) as e:
            ltx_b200.apply_keyframe(ctx, z, m, torch.zeros(C, tpf, device="cuda"), frame, strength)
        assert e.value.kind == kind
    ctx.close()


def test_sequential_chunks_with_seam_keyframes_match_oracle(tmp_path):
    """Two overlapping chunks (4 latent frames each, 1 shared) through denoise_sequential:
    chunk 1's first latent frame is conditioned (strength 0.95) on chunk 0's final latent at
    that clip frame, then denoised.  Against the oracle running the same loop on its own
    chunk-0 output: rel-L2 <= 1e-2 per chunk."""
    import ltx_b200
    from ltx_b200 import chunks as lc
    from dit_checkpoint import small_config, write_checkpoint
    from oracle import dit, sampler as osam
    from oracle.weight_store import KeyMap, WeightStore as OracleStore
    cfg = small_config(heads=2, head_dim=128, layers=2)
    ck = str(tmp_path / "seq.safetensors")
    write_checkpoint(ck, cfg, seed=17)
    ctx = ltx_b200.Context(0)
    st = ltx_b200.WeightStore(ctx, [ck], ltx_b200.KEYMAP_TRANSFORMER)
    model = ltx_b200.VideoTransformer.load(ctx, st)
    o = OracleStore([ck], KeyMap.transformer())
    params = dit.load_params({k: o.read(k) for k in o.keys()})
    c = dit.DiTConfig.from_json(cfg)
    F, Hh, W, S, C = 4, 4, 8, 24, 128
    tpf, Tt = Hh * W, F * Hh * W
    plan = [(0, 4, 0), (3, 7, 1)]
    sig = [float(x) for x in osam.scheduler_execute(8, Tt)[:3]]
    rng = np.random.default_rng(8)
    o_states, d_states = [], []
    for n in range(2):
        init = osam.LatentState(rng.standard_normal((1, Tt, C)).astype(np.float32), np.ones((1, Tt, 1), np.float32),
                                osam.target_positions(F, Hh, W), np.zeros((1, Tt, C), np.float32))
        s = osam.apply_reference(init, rng.standard_normal((1, C, F, Hh, W)).astype(np.float32), strength=1.0)
        cc = rng.standard_normal((1, S, cfg["cross_attention_dim"])).astype(np.float32)
        cu = rng.standard_normal((1, S, cfg["cross_attention_dim"])).astype(np.float32)
        o_states.append((s, cc, cu))
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        d_states.append({"latent": dev(s.latent[0]), "clean": dev(s.clean_latent[0]), "mask": dev(s.denoise_mask[0, :, 0]),
                         "positions": dev(s.positions), "ctx_cond": dev(cc[0]), "ctx_uncond": dev(cu[0])})
    got = lc.denoise_sequential(ctx, model, d_states, plan, tpf, sig, 3.0, 0.7, target_tokens=Tt)
    ctx.synchronize()
    got = [g.cpu().numpy() for g in got]

    def model_x0(latent, ts, pos, ctx_):
        with torch.no_grad():
            v = dit.model_forward(params, c, torch.from_numpy(latent), torch.from_numpy(ts), torch.from_numpy(pos),
                                  torch.from_numpy(ctx_)).numpy()
        return osam.velocity_to_x0(latent, ts, v)

    exp = []
    for n, (s, cc, cu) in enumerate(o_states):
        if n > 0:
            (idx, strength), = oc.seam_cond_plan(8 * plan[n][2])[0]
            src = plan[n][0] - plan[n - 1][0] + idx // 8
            tok = exp[n - 1][src * tpf:(src + 1) * tpf]                      # [tpf, C]
            image = osam.unpatchify(tok[None], 1, 1, tpf)                  # [1, C, 1, 1, tpf]
            s = osam.apply_keyframe(s, image, idx // 8, tpf, strength)
        exp.append(osam.euler_loop(sig, s, Tt, model_x0, cc, cu, cfg_scale=3.0, rescale_scale=0.7).latent[0])
    for n in range(2):
        err = float(np.linalg.norm(got[n] - exp[n]) / np.linalg.norm(exp[n]))
        print(f"\nchunk {n} with seam keyframes: rel-L2 {err:.2e}")
        assert np.isfinite(got[n]).all() and err < 1e-2
    # the keyframe moved chunk 1's first latent frame toward chunk 0's output there
    model.close()
    st.close()
    ctx.close()
