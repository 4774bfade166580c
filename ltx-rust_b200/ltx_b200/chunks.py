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
