"""Chunk-parallel generation across ranks: one temporal chunk per GPU.

The reference generates a clip's temporal chunks one after another
(crates/ltx-pipeline/src/lib.rs:270-353) and crossfades consecutive chunks
over their shared frames (crates/ltx-chunk/src/blend.rs).  With seam
keyframes off (PipelineConfig::seam_keyframes = false, lib.rs:28-39) the
chunks do not depend on one another, so here each rank denoises its own
chunks (seed = base + chunk index, lib.rs:374-377) and the only exchange is
the seam: the frames a chunk shares with the next one travel once, to the
rank that owns the next chunk, which blends them into its head with
ltx_seam_blend.  After that every clip frame is final on exactly one rank.

Ownership: chunk n is the clip frames [start_n, end_n); frames
[start_n, start_n + real_overlap_n) are its seam with chunk n-1 (blended on
the owner of chunk n); frames [start_{n+1}, end_n) go to chunk n+1.  So the
owner of chunk n emits [start_n, start_{n+1}) (or [start_n, end_n) for the
last chunk), as Blender::finish_chunk emits them (blend.rs:151-182).

Collectives: one point-to-point send/recv per seam whose two chunks sit on
different ranks (NCCL on device tensors, gloo on CPU tensors); every rank
takes the same steps in the same order.

With seam keyframes on (the reference's default) chunk n depends on chunk
n-1's output, so the chunks run one after another: denoise_sequential.
"""
from __future__ import annotations


def assign(n_chunks: int, world_size: int):
    """Contiguous blocks of chunks per rank: [[chunk indices of rank 0], ...]."""
    per, extra = divmod(n_chunks, world_size)
    out, c = [], 0
    for r in range(world_size):
        k = per + (1 if r < extra else 0)
        out.append(list(range(c, c + k)))
        c += k
    return out


def owner_of(chunk: int, assignment) -> int:
    for r, cs in enumerate(assignment):
        if chunk in cs:
            return r
    raise ValueError(f"chunk {chunk} has no owner")


def emitted_range(chunks, n: int):
    """Clip frames [a, b) that chunk n's owner holds final after the seam blends."""
    start, end, _ = chunks[n]
    return start, (chunks[n + 1][0] if n + 1 < len(chunks) else end)


def exchange_seams(chunks, assignment, rank: int, chunk_data: dict, group=None):
    """Sends each owned chunk's tail to the owner of the next chunk and returns
    {n: tail of chunk n-1} for every owned chunk n > 0.

    chunk_data maps owned chunk index -> tensor [len_n, ...] (frames first).
    Tails of chunks on the same rank are sliced locally (no copy over the
    link).  Uses torch.distributed point-to-point ops; all sends and receives
    of a rank are issued together and waited on before returning."""
    import torch
    import torch.distributed as dist
    ops, recv = [], {}
    for n in range(1, len(chunks)):
        src, dst = owner_of(n - 1, assignment), owner_of(n, assignment)
        ro = chunks[n][2]
        if ro == 0:
            continue
        prev_start = chunks[n - 1][0]
        off = chunks[n][0] - prev_start          # tail of chunk n-1 starts at chunk n's start
        if src == rank and dst == rank:
            recv[n] = chunk_data[n - 1][off:off + ro]
        elif src == rank:
            ops.append(dist.P2POp(dist.isend, chunk_data[n - 1][off:off + ro].contiguous(), dst, group))
        elif dst == rank:
            like = chunk_data[n]
            buf = torch.empty((ro,) + tuple(like.shape[1:]), dtype=like.dtype, device=like.device)
            recv[n] = buf
            ops.append(dist.P2POp(dist.irecv, buf, src, group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return recv


def blend_seams(ctx, chunks, recv: dict, chunk_data: dict):
    """Blends every received tail into the head of its chunk in place, on the device
    (ltx_seam_blend: w = crossfade_weight(i, real_overlap), new = fma(w, head, (1-w)*tail))."""
    from . import seam_blend
    for n, tail in recv.items():
        ro = chunks[n][2]
        head = chunk_data[n][:ro]
        seam_blend(ctx, tail, head, head)


def gather_clip(chunks, assignment, rank: int, chunk_data: dict, total_shape, root: int = 0, group=None):
    """Collects every chunk's emitted frames on `root` (after blend_seams) into one
    tensor of total_shape [total_frames, ...]; returns it on root, None elsewhere."""
    import torch
    import torch.distributed as dist
    like = next(iter(chunk_data.values()))
    clip = torch.empty(total_shape, dtype=like.dtype, device=like.device) if rank == root else None
    ops = []
    for n in range(len(chunks)):
        a, b = emitted_range(chunks, n)
        if b <= a:
            continue
        o = owner_of(n, assignment)
        s = chunks[n][0]
        if o == rank == root:
            clip[a:b].copy_(chunk_data[n][a - s:b - s])
        elif o == rank:
            ops.append(dist.P2POp(dist.isend, chunk_data[n][a - s:b - s].contiguous(), root, group))
        elif rank == root:
            ops.append(dist.P2POp(dist.irecv, clip[a:b], o, group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return clip


def denoise_sequential(ctx, model, states, latent_plan, tokens_per_frame, sigmas, cfg_scale=3.0, rescale_scale=0.7,
                       target_tokens=None, seam_keyframes=True):
    """The reference's default chunk loop (PipelineConfig::seam_keyframes = true,
    crates/ltx-pipeline/src/lib.rs:28-39, 300-311): before chunk n > 0 is
    denoised it is conditioned on chunk n-1's output at the seam
    (keyframes_from_previous, lib.rs:493-548): seam_cond_plan (crates/ltx-chunk/
    src/seam.rs:110-125) names one frame at chunk-local index 0 with strength
    0.95, applied as ImageKeyframeCondition (crates/ltx-sampler/src/
    conditioning.rs:127-205).  The reference encodes chunk n-1's decoded pixel
    frame with the VAE; here the keyframe is chunk n-1's final latent frame at
    the same clip position, applied in latent space (ltx_apply_keyframe), so
    no VAE is needed.

    states: one dict per chunk of device tensors latent [T, C], clean [T, C],
    mask [T], positions, ctx_cond, ctx_uncond (the chunk's sampler state;
    clean and mask are modified); latent_plan: [(start, end, real_overlap)] in
    latent frames.  Returns each chunk's final target tokens [target_tokens, C]."""
    import torch
    from . import apply_keyframe, seam_cond_plan, unpatchify
    outs = []
    for n, st in enumerate(states):
        T, C = st["latent"].shape
        tt = T if target_tokens is None else target_tokens
        ro = latent_plan[n][2]
        if seam_keyframes and n > 0 and ro > 0:
            idx, strength, _ = seam_cond_plan(8 * ro)          # pixel overlap: 8 frames per latent frame
            src = latent_plan[n][0] - latent_plan[n - 1][0] + idx // 8   # that clip frame in chunk n-1
            tok = outs[n - 1][src * tokens_per_frame:(src + 1) * tokens_per_frame]
            image = torch.empty(C, tokens_per_frame, dtype=tok.dtype, device=tok.device)
            unpatchify(ctx, tok.contiguous(), image.view(1, C, 1, 1, tokens_per_frame))   # [tpf, C] -> [C, 1, 1, tpf]
            apply_keyframe(ctx, st["clean"], st["mask"], image, idx // 8, strength)
        out = torch.empty(tt, C, dtype=st["latent"].dtype, device=st["latent"].device)
        lat = st["latent"].clone()
        model.denoise_loop(lat, st["clean"], st["mask"], st["positions"], st["ctx_cond"], st["ctx_uncond"], sigmas,
                           cfg_scale, rescale_scale, target_tokens=tt, out=out)
        outs.append(out)
    return outs
