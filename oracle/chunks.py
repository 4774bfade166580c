"""CPU restatement of the reference's temporal chunk planner and seam blender.

TEST INFRASTRUCTURE ONLY: the checker for the library's ltx_chunk_plan,
ltx_seam_blend and ltx_chunk_assemble.  Nothing in the product imports it.

Follows, line by line:
  plan                      crates/ltx-chunk/src/plan.rs:56-160
  on_frame_grid             plan.rs:163-168 (LTX-2 temporal scale 8)
  smoothstep                crates/ltx-chunk/src/blend.rs:32-36
  crossfade_weight          blend.rs:49-56
  Blender                   blend.rs:67-298 (new, push_frame, finish_chunk, drain, flush)
  the pipeline's driving    crates/ltx-pipeline/src/lib.rs:270-353 (push every frame,
                            finish_chunk(len, next.real_overlap), drain, flush at the end)
  seam_cond_plan            crates/ltx-chunk/src/seam.rs:110-125 (one keyframe at the seam)

Pinned against the known answers in plan.rs / blend.rs's own tests
(tests/test_chunks_host.py).
"""
import numpy as np


class ChunkError(ValueError):
    """ChunkError (crates/ltx-chunk/src/error.rs:7-30); .kind is the variant name."""

    def __init__(self, kind, msg=""):
        super().__init__(f"{kind}: {msg}")
        self.kind = kind


DEFAULT_KEYFRAME_STRENGTH = np.float32(0.95)   # seam.rs:60


def seam_cond_plan(overlap):
    """seam_cond_plan (seam.rs:110-125): ([(chunk_local_idx, strength)], blend_tail_len)."""
    if overlap == 0:
        raise ChunkError("ZeroOverlapForSeam", "overlap must be non-zero for a seam conditioning plan")
    return [(0, DEFAULT_KEYFRAME_STRENGTH)], overlap - 1


def _sat_sub(a, b):
    return a - b if a > b else 0


def on_frame_grid(frames):
    return frames >= 1 and (frames - 1) % 8 == 0


def plan(total, chunk_len, overlap):
    """[(start, end, real_overlap), ...] as plan() (plan.rs:56-160)."""
    if total == 0:
        raise ChunkError("ZeroTotal")
    if not on_frame_grid(chunk_len):
        raise ChunkError("ChunkLenNotOnGrid", str(chunk_len))
    if overlap >= chunk_len:
        raise ChunkError("OverlapNotSmallerThanChunkLen", f"{overlap} >= {chunk_len}")
    if overlap % 8 != 0:
        raise ChunkError("OverlapNotMultipleOf8", str(overlap))
    stride = _sat_sub(chunk_len, overlap)
    if stride < overlap:
        raise ChunkError("StrideSmallerThanOverlap", f"{stride} < {overlap}")
    if total <= chunk_len:
        return [(0, total, 0)]
    starts, s = [], 0
    while True:
        if s + chunk_len >= total:
            break
        starts.append(s)
        s += stride
    last = _sat_sub(total, chunk_len)
    if not starts or starts[-1] != last:
        starts.append(last)
    while len(starts) >= 3:
        fi = len(starts) - 1
        if starts[fi] < starts[fi - 2] + chunk_len:
            del starts[fi - 1]
        else:
            break
    out = []
    for i, st in enumerate(starts):
        end = total if i == len(starts) - 1 else st + chunk_len
        ro = 0 if i == 0 else _sat_sub(min(starts[i - 1] + chunk_len, total), st)
        out.append((st, end, ro))
    return out


def smoothstep(t):
    """t² (3 − 2t) in f64, clamped to [0, 1]: t * t * 2.mul_add(-t, 3) (blend.rs:32-36).
    2·(−t) is exact in f64, so fma(2, −t, 3) and 3 − 2t round once, identically."""
    t = min(max(float(t), 0.0), 1.0)
    return t * t * (3.0 - 2.0 * t)


def crossfade_weight(offset, overlap_len):
    """f32 of smoothstep(offset / overlap_len); 1.0 for overlap_len 0 (blend.rs:49-56)."""
    if overlap_len == 0:
        return np.float32(1.0)
    return np.float32(smoothstep(float(offset) / float(overlap_len)))


def blend_frame(old, new, w_new):
    """blend_with_pending (blend.rs:284-298): w_new.mul_add(new, (1 - w_new) * old), f32."""
    from oracle.weight_store import lib
    old = np.ascontiguousarray(old, np.float32)
    new = np.ascontiguousarray(new, np.float32)
    out = np.empty_like(old)
    lib().oracle_crossfade_blend(old.ctypes.data, new.ctypes.data, float(w_new), old.size, out.ctypes.data)
    return out


class Blender:
    """Streaming crossfade blender (blend.rs:67-298), the state machine as the reference keeps it."""

    def __init__(self, chunk_len, overlap, frame_size):
        if not on_frame_grid(chunk_len):
            raise ChunkError("ChunkLenNotOnGrid", str(chunk_len))
        if overlap % 8 != 0:
            raise ChunkError("OverlapNotMultipleOf8", str(overlap))
        if overlap >= chunk_len:
            raise ChunkError("OverlapNotSmallerThanChunkLen")
        if chunk_len - overlap < overlap:
            raise ChunkError("StrideSmallerThanOverlap")
        self.chunk_len, self.frame_size = chunk_len, frame_size
        self.pending, self.current, self.ready = [], [], []
        self.first = True

    def push_frame(self, frame):
        frame = np.asarray(frame, np.float32).reshape(-1)
        if frame.size != self.frame_size:
            raise ChunkError("PixelsWrongLen")
        if len(self.current) >= self.chunk_len:
            raise ChunkError("ChunkAlreadyFull")
        self.current.append(frame.copy())

    def finish_chunk(self, expected_len, next_overlap):
        if len(self.current) != expected_len:
            raise ChunkError("ChunkFrameCount")
        if next_overlap > expected_len:
            raise ChunkError("RetainedOverlapTooLarge")
        emit_until = _sat_sub(expected_len, next_overlap)
        if not self.first and len(self.pending) > emit_until:
            raise ChunkError("RetainedOverlapTooLarge")
        for i in range(expected_len):
            frame = self.current[i]
            if not self.first and i < len(self.pending):
                self.ready.append(blend_frame(self.pending[i], frame, crossfade_weight(i, len(self.pending))))
            elif i < emit_until:
                self.ready.append(frame.copy())
        self.pending = [f.copy() for f in self.current[expected_len - next_overlap:]] if next_overlap else []
        self.current = []
        self.first = False

    def drain(self):
        out, self.ready = self.ready, []
        return out

    def flush(self):
        self.ready.extend(self.pending)
        self.pending = []
        return self.drain()


def assemble(chunk_frames, chunks, chunk_len, overlap):
    """The clip the pipeline writes (lib.rs:270-353): every chunk's frames pushed in
    order, finish_chunk(len, next.real_overlap), drained, then flushed.
    chunk_frames[n] is [len_n, frame_size] f32.  Returns [total, frame_size]."""
    frame_size = int(np.asarray(chunk_frames[0]).reshape(len(chunk_frames[0]), -1).shape[1])
    b = Blender(chunk_len, overlap, frame_size)
    out = []
    for n, (st, en, _ro) in enumerate(chunks):
        frames = np.asarray(chunk_frames[n], np.float32).reshape(en - st, -1)
        for f in frames:
            b.push_frame(f)
        nxt = chunks[n + 1][2] if n + 1 < len(chunks) else 0
        b.finish_chunk(en - st, nxt)
        out.extend(b.drain())
    out.extend(b.flush())
    return np.stack(out)
