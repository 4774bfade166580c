"""Temporal chunk planner and seam crossfade: host side (no GPU).

1. The oracle (oracle/chunks.py) against the known answers of the reference's
   own tests (crates/ltx-chunk/src/plan.rs tests, blend.rs tests).
2. The library's ltx_chunk_plan / ltx_crossfade_weight against the oracle,
   bit-exact, over a sweep of clip lengths, chunk lengths and overlaps,
   including the ChunkError variants.
3. The chunk-parallel host logic (ltx_b200.chunks) on two gloo ranks: the seam
   exchange and the clip gather move the right frames, so that blending the
   received tails reproduces the reference Blender's clip.
"""
import os

import numpy as np
import pytest

from oracle import chunks as oc


# ── 1. oracle pinned to the reference's tests ───────────────────────────────

@pytest.mark.parametrize("args,kind", [
    ((0, 9, 0), "ZeroTotal"),                          # plan.rs tests: zero_total_is_error
    ((10, 10, 0), "ChunkLenNotOnGrid"),                # chunk_len_not_on_grid_is_error
    ((10, 2, 0), "ChunkLenNotOnGrid"),
    ((50, 17, 4), "OverlapNotMultipleOf8"),            # overlap_not_multiple_of_8_is_error
    ((50, 17, 17), "OverlapNotSmallerThanChunkLen"),   # overlap_ge_chunk_len_is_error
    ((50, 17, 16), "StrideSmallerThanOverlap"),        # stride_smaller_than_overlap_is_error
])
def test_oracle_plan_errors(args, kind):
    with pytest.raises(oc.ChunkError) as e:
        oc.plan(*args)
    assert e.value.kind == kind


def test_oracle_plan_known_answers():
    assert oc.plan(17, 17, 8) == [(0, 17, 0)]                     # single_chunk_total_eq_chunk_len
    assert oc.plan(5, 17, 8) == [(0, 5, 0)]                       # single_chunk_total_less_than_chunk_len
    assert oc.plan(17, 17, 0) == [(0, 17, 0)]                     # single_chunk_zero_overlap
    assert oc.plan(18, 17, 8) == [(0, 17, 0), (1, 18, 16)]        # two_chunks_last_anchored
    p = oc.plan(35, 17, 8)                                        # three_chunks_exact_fit
    assert [c[0] for c in p] == [0, 9, 18] and p[2][1] == 35 and p[2][2] == 8
    assert oc.plan(28, 17, 8) == [(0, 17, 0), (11, 28, 6)]        # anchored_last_prunes_three_chunk_overlap
    assert oc.plan(40, 17, 8) == [(0, 17, 0), (9, 26, 8), (23, 40, 3)]  # ..._keeps_earlier_non_intersecting
    p = oc.plan(200, 33, 8)                                       # many_chunks_full_coverage
    assert p[-1][1] == 200 and p[0][2] == 0 and all(c[2] == 8 for c in p[1:-1])
    p = oc.plan(100, 17, 0)                                       # zero_overlap_no_blend_zones
    assert all(c[2] == 0 for c in p[:-1])


def _check_plan_properties(p, total, chunk_len):
    for f in range(total):
        cover = sum(1 for s, e, _ in p if s <= f < e)
        assert 1 <= cover <= 2, (f, p)
    assert all(a[0] < b[0] for a, b in zip(p, p[1:]))
    assert all((e - s) == (total if total <= chunk_len else chunk_len) for s, e, _ in p)


def test_oracle_plan_coverage_sweep():
    for chunk_len in (9, 17, 33, 49, 121):
        for overlap in range(0, chunk_len // 2 + 1, 8):
            for total in list(range(1, 3 * chunk_len)) + [200, 481]:
                _check_plan_properties(oc.plan(total, chunk_len, overlap), total, chunk_len)


def test_oracle_smoothstep_and_weights():
    assert abs(oc.smoothstep(0.0)) < 1e-10 and abs(oc.smoothstep(1.0) - 1) < 1e-10   # smoothstep_endpoints
    assert abs(oc.smoothstep(0.5) - 0.5) < 1e-10                                      # smoothstep_midpoint
    assert oc.smoothstep(-0.5) == 0.0 and oc.smoothstep(1.5) == 1.0                  # smoothstep_clamps_outside
    assert abs(oc.crossfade_weight(0, 8)) < 1e-6 and abs(oc.crossfade_weight(8, 8) - 1) < 1e-6
    for i in range(16):                                                               # weights_sum_to_one
        w = oc.crossfade_weight(i, 16)
        assert abs(w + (np.float32(1) - w) - 1) < 1e-6
    assert oc.crossfade_weight(3, 0) == 1.0


def test_oracle_blender_constant_and_ramp():
    # constant_signal_reconstructs_exactly: two chunks of 1.0, 17 frames, overlap 8 -> 26 frames of 1.0
    b = oc.Blender(17, 8, 4)
    out = []
    for nxt in (8, 0):
        for _ in range(17):
            b.push_frame(np.ones(4, np.float32))
        b.finish_chunk(17, nxt)
        out += b.drain()
    out += b.flush()
    assert len(out) == 26 and all(np.all(np.abs(f - 1) < 1e-6) for f in out)
    # ramp_signal_reconstructs_exactly: chunk 0 frame i -> i, chunk 1 frame i -> 9 + i
    b = oc.Blender(17, 8, 4)
    out = []
    for base, nxt in ((0, 8), (9, 0)):
        for i in range(17):
            b.push_frame(np.full(4, base + i, np.float32))
        b.finish_chunk(17, nxt)
        out += b.drain()
    out += b.flush()
    assert len(out) == 26
    for g, f in enumerate(out):
        assert np.all(np.abs(f - g) < 1e-4), (g, f)


def test_oracle_assemble_planned_ramp():
    # blend.rs planned_ramp_handles_anchored_totals: global ramp survives every plan
    for total in (17, 18, 26, 28, 35, 40, 57, 100):
        p = oc.plan(total, 17, 8)
        frames = [np.arange(s, e, dtype=np.float32).reshape(-1, 1) for s, e, _ in p]
        clip = oc.assemble(frames, p, 17, 8)
        assert clip.shape == (total, 1)
        assert np.all(np.abs(clip[:, 0] - np.arange(total)) < 1e-4)


# ── 2. the library's host functions against the oracle ──────────────────────

def test_capi_plan_matches_oracle():
    import ltx_b200
    n = 0
    for chunk_len in (1, 9, 17, 25, 33, 49, 121):
        for overlap in (0, 4, 8, 16, 24, 32, 48, 56, 64, 120, 121):
            for total in (0, 1, 5, 9, 17, 18, 26, 28, 35, 40, 57, 100, 121, 200, 241, 481, 1000):
                try:
                    want = oc.plan(total, chunk_len, overlap)
                except oc.ChunkError as e:
                    with pytest.raises(ltx_b200.LtxError) as got:
                        ltx_b200.chunk_plan(total, chunk_len, overlap)
                    assert got.value.kind == "CHUNK_PLAN" and e.kind in str(got.value), (total, chunk_len, overlap)
                    continue
                assert ltx_b200.chunk_plan(total, chunk_len, overlap) == want, (total, chunk_len, overlap)
                n += 1
    assert n > 300


def test_capi_crossfade_weight_bit_exact():
    import ltx_b200
    for ov in range(0, 130):
        for i in range(0, ov + 2):
            assert np.float32(ltx_b200.crossfade_weight(i, ov)).tobytes() == oc.crossfade_weight(i, ov).tobytes()


# ── 3. chunk-parallel host logic on two gloo ranks ──────────────────────────

def _gloo_worker(rank, ws, port, total, chunk_len, overlap, fsize, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=60))
    try:
        from ltx_b200 import chunks as cp
        plan = oc.plan(total, chunk_len, overlap)
        asg = cp.assign(len(plan), ws)
        rng = np.random.default_rng(5)
        all_frames = [rng.standard_normal((e - s, fsize), dtype=np.float32) for s, e, _ in plan]
        data = {n: torch.from_numpy(all_frames[n].copy()) for n in asg[rank]}
        recv = cp.exchange_seams(plan, asg, rank, data)
        # the device blend (ltx_seam_blend) is checked on the GPU; here the oracle plays it
        for n, tail in recv.items():
            ro = plan[n][2]
            for i in range(ro):
                w = oc.crossfade_weight(i, ro)
                data[n][i] = torch.from_numpy(oc.blend_frame(tail[i].numpy(), data[n][i].numpy(), w))
        clip = cp.gather_clip(plan, asg, rank, data, (total, fsize))
        if rank == 0:
            want = oc.assemble(all_frames, plan, chunk_len, overlap)
            q.put(bool(np.array_equal(clip.numpy().view(np.uint32), want.view(np.uint32))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total,chunk_len,overlap", [(121 * 2 - 16, 121, 16), (40, 17, 8), (100, 17, 8)])
def test_chunk_parallel_gloo_two_ranks(total, chunk_len, overlap):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, total, chunk_len, overlap, 6, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def test_assign_contiguous():
    from ltx_b200 import chunks as cp
    assert cp.assign(8, 8) == [[i] for i in range(8)]
    assert cp.assign(5, 2) == [[0, 1, 2], [3, 4]]
    assert cp.assign(1, 2) == [[0], []]
    p = oc.plan(100, 17, 8)
    assert [cp.emitted_range(p, n) for n in range(len(p))][0] == (0, p[1][0])


# ── seam keyframes (crates/ltx-chunk/src/seam.rs, ltx-sampler conditioning.rs) ──

def test_seam_cond_plan_oracle_matches_reference_tests():
    """seam.rs's own tests: one conditioning at chunk-local 0 (latent-aligned), strength 0.95,
    blend tail overlap - 1 (so conditioning + tail == overlap), ZeroOverlapForSeam at 0."""
    from oracle import chunks as oc
    for overlap in (8, 16, 24, 32):
        conds, tail = oc.seam_cond_plan(overlap)
        assert conds == [(0, np.float32(0.95))] and tail == overlap - 1 and len(conds) + tail == overlap
        assert all(i % 8 == 0 for i, _ in conds)
    with pytest.raises(oc.ChunkError) as e:
        oc.seam_cond_plan(0)
    assert e.value.kind == "ZeroOverlapForSeam"


def test_seam_cond_plan_c_abi_matches_oracle():
    import ltx_b200
    from oracle import chunks as oc
    for overlap in (1, 8, 16, 40):
        idx, strength, tail = ltx_b200.seam_cond_plan(overlap)
        (o_idx, o_s), = oc.seam_cond_plan(overlap)[0]
        assert (idx, np.float32(strength), tail) == (o_idx, o_s, oc.seam_cond_plan(overlap)[1])
    with pytest.raises(ltx_b200.LtxError) as e:
        ltx_b200.seam_cond_plan(0)
    assert e.value.kind == "CHUNK_PLAN" and "ZeroOverlapForSeam" in str(e.value)


def test_keyframe_oracle_matches_reference_tests():
    """conditioning.rs keyframe_condition_writes_only_its_frame and
    keyframe_condition_rejects_strength_outside_unit_range."""
    from oracle import sampler as os_
    st = os_.LatentState(np.zeros((1, 6, 2), np.float32), np.ones((1, 6, 1), np.float32),
                         np.zeros((1, 3, 6, 2), np.float32), np.full((1, 6, 2), -1.0, np.float32))
    img = np.array([1.0, 3.0, 2.0, 4.0], np.float32).reshape(1, 2, 1, 1, 2)
    out = os_.apply_keyframe(st, img, 1, 2, 0.95)
    assert out.clean_latent.reshape(-1).tolist() == [-1, -1, -1, -1, 1, 2, 3, 4, -1, -1, -1, -1]
    np.testing.assert_allclose(out.denoise_mask.reshape(-1), [1, 1, 0.05, 0.05, 1, 1], atol=1e-6)
    for s in (-0.1, 1.5, float("nan")):
        with pytest.raises(os_.SamplerError) as e:
            os_.apply_keyframe(st, np.zeros((1, 2, 1, 1, 2), np.float32), 0, 2, s)
        assert e.value.kind == "InvalidStrength"
