// Temporal chunks of a clip: the chunk planner (host) and the smoothstep
// crossfade across chunk seams (device).
//   plan                crates/ltx-chunk/src/plan.rs:56-160
//   smoothstep          crates/ltx-chunk/src/blend.rs:32-36
//   crossfade_weight    blend.rs:49-56
//   Blender seams       blend.rs:151-182 (finish_chunk), 284-298 (blend_with_pending)
//   driving the blender crates/ltx-pipeline/src/lib.rs:270-353
//
// The blend is an HBM-bound streaming op (two f32 reads, one f32 write per
// value); frames are contiguous runs of frame_values floats, so a pixel frame
// and a latent frame (H*W tokens x C channels) are blended the same way.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <vector>

#include "internal.hpp"

namespace {

// u32 saturating arithmetic as the reference's saturating_add/sub.
inline uint32_t sat_add(uint32_t a, uint32_t b) { return a > UINT32_MAX - b ? UINT32_MAX : a + b; }
inline uint32_t sat_sub(uint32_t a, uint32_t b) { return a > b ? a - b : 0; }

// smoothstep(offset / overlap) in f64 with the reference's operation order
// t * t * fma(2, -t, 3), then narrowed to f32.  The explicit intrinsics keep
// the compiler from contracting or reassociating (identical on host and
// device: f64 division, multiply and fma are correctly rounded on both).
__host__ __device__ inline float crossfade(uint32_t offset, uint32_t overlap) {
    if (overlap == 0) return 1.0f;
#ifdef __CUDA_ARCH__
    double t = __ddiv_rn((double)offset, (double)overlap);
    t = fmin(fmax(t, 0.0), 1.0);
    return (float)__dmul_rn(__dmul_rn(t, t), __fma_rn(2.0, -t, 3.0));
#else
    double t = (double)offset / (double)overlap;
    t = t < 0.0 ? 0.0 : (t > 1.0 ? 1.0 : t);
    const double tt = t * t;
    const double q = std::fma(2.0, -t, 3.0);
    return (float)(tt * q);
#endif
}

// dst[f][j] = fma(w_f, in[f][j], (1 - w_f) * out[f][j]) for f < frames.
// blockIdx.y is the frame; float4 path when every pointer is 16-byte aligned
// and frame_values % 4 == 0.  dst may alias either input: each value is read
// and written by the same thread.
template <bool VEC>
__global__ void __launch_bounds__(256) seam_blend_kernel(const float *outgoing, const float *incoming,
                                                         float *dst,
                                                         uint32_t frames, int64_t frame_values) {
    const uint32_t f = blockIdx.y;
    if (f >= frames) return;
    const float w_new = crossfade(f, frames);
    const float w_old = 1.0f - w_new;
    const int64_t base = (int64_t)f * frame_values;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if constexpr (VEC) {
        const int64_t n4 = frame_values / 4;
        const float4 *o4 = reinterpret_cast<const float4 *>(outgoing + base);
        const float4 *i4 = reinterpret_cast<const float4 *>(incoming + base);
        float4 *d4 = reinterpret_cast<float4 *>(dst + base);
        for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += stride) {
            const float4 a = __ldcs(o4 + v), b = __ldcs(i4 + v);
            float4 r;
            r.x = __fmaf_rn(w_new, b.x, __fmul_rn(w_old, a.x));
            r.y = __fmaf_rn(w_new, b.y, __fmul_rn(w_old, a.y));
            r.z = __fmaf_rn(w_new, b.z, __fmul_rn(w_old, a.z));
            r.w = __fmaf_rn(w_new, b.w, __fmul_rn(w_old, a.w));
            __stcs(d4 + v, r);
        }
    } else {
        for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < frame_values; v += stride)
            dst[base + v] = __fmaf_rn(w_new, incoming[base + v], __fmul_rn(w_old, outgoing[base + v]));
    }
}

cudaError_t launch_seam_blend(cudaStream_t st, int sms, const float *outgoing, const float *incoming, float *dst,
                              uint32_t frames, int64_t frame_values) {
    if (frames == 0 || frame_values == 0) return cudaSuccess;
    const bool vec = frame_values % 4 == 0 && ((uintptr_t)outgoing | (uintptr_t)incoming | (uintptr_t)dst) % 16 == 0;
    const int64_t per_thread = vec ? 4 : 1;
    int64_t blocks_x = (frame_values / per_thread + 255) / 256;
    // enough blocks in total to cover the SMs a few times, capped per frame
    const int64_t cap = ((int64_t)sms * 8 + frames - 1) / frames;
    if (blocks_x > cap) blocks_x = cap;
    if (blocks_x < 1) blocks_x = 1;
    // blockIdx.y carries the frame: the grid's y limit is 65535 frames
    if (frames > 65535) return cudaErrorInvalidValue;
    dim3 grid((unsigned)blocks_x, frames);
    if (vec)
        seam_blend_kernel<true><<<grid, 256, 0, st>>>(outgoing, incoming, dst, frames, frame_values);
    else
        seam_blend_kernel<false><<<grid, 256, 0, st>>>(outgoing, incoming, dst, frames, frame_values);
    return cudaGetLastError();
}

}  // namespace

extern "C" float ltx_crossfade_weight(uint32_t offset, uint32_t overlap_len) { return crossfade(offset, overlap_len); }

// seam_cond_plan (crates/ltx-chunk/src/seam.rs:110-125): one keyframe at the
// seam (chunk-local 0, latent-aligned), strength DEFAULT_KEYFRAME_STRENGTH.
extern "C" int ltx_seam_cond_plan(uint32_t overlap, uint32_t *chunk_local_idx, float *strength,
                                  uint32_t *blend_tail_len) {
    if (!chunk_local_idx || !strength || !blend_tail_len)
        return ltx::host_fail(LTX_ERR_INVALID_ARG, "ltx_seam_cond_plan: null output");
    if (overlap == 0)
        return ltx::host_fail(LTX_ERR_CHUNK_PLAN, "ZeroOverlapForSeam: overlap must be non-zero for a seam conditioning plan");
    *chunk_local_idx = 0;
    *strength = 0.95f;   // DEFAULT_KEYFRAME_STRENGTH (seam.rs:60)
    *blend_tail_len = overlap - 1;
    return LTX_OK;
}

extern "C" int ltx_chunk_plan(uint32_t total, uint32_t chunk_len, uint32_t overlap, ltx_chunk *chunks_out,
                              int32_t max_chunks, int32_t *n_chunks) {
    using ltx::host_fail;
    if (!n_chunks || max_chunks < 0 || (max_chunks > 0 && !chunks_out))
        return host_fail(LTX_ERR_INVALID_ARG, "ltx_chunk_plan: null output or negative max_chunks");
    *n_chunks = 0;
    // the checks, their order and their messages as plan() (plan.rs:56-86, error.rs:7-30)
    if (total == 0) return host_fail(LTX_ERR_CHUNK_PLAN, "ZeroTotal: total frame count must be non-zero");
    if (chunk_len == 0 || (chunk_len - 1) % 8 != 0)
        return host_fail(LTX_ERR_CHUNK_PLAN, "ChunkLenNotOnGrid: chunk_len %u is not 8k+1", chunk_len);
    if (overlap >= chunk_len)
        return host_fail(LTX_ERR_CHUNK_PLAN, "OverlapNotSmallerThanChunkLen: overlap %u must be less than chunk_len %u",
                         overlap, chunk_len);
    if (overlap % 8 != 0)
        return host_fail(LTX_ERR_CHUNK_PLAN, "OverlapNotMultipleOf8: overlap %u is not a multiple of 8", overlap);
    const uint32_t stride = sat_sub(chunk_len, overlap);
    if (stride < overlap)
        return host_fail(LTX_ERR_CHUNK_PLAN, "StrideSmallerThanOverlap: stride (chunk_len - overlap = %u) must be >= "
                         "overlap %u", stride, overlap);

    std::vector<ltx_chunk> out;
    if (total <= chunk_len) {
        out.push_back({0, total, 0});
    } else {
        std::vector<uint32_t> starts;
        for (uint32_t s = 0;; s = sat_add(s, stride)) {
            if (sat_add(s, chunk_len) >= total) break;
            starts.push_back(s);
        }
        const uint32_t last = sat_sub(total, chunk_len);
        if (starts.empty() || starts.back() != last) starts.push_back(last);
        // drop the middle candidate while the anchored chunk reaches into the
        // chunk two places back (keeps every frame in at most two chunks)
        while (starts.size() >= 3) {
            const size_t fi = starts.size() - 1;
            if (starts[fi] < sat_add(starts[fi - 2], chunk_len))
                starts.erase(starts.begin() + (fi - 1));
            else
                break;
        }
        for (size_t i = 0; i < starts.size(); ++i) {
            const uint32_t end = i + 1 == starts.size() ? total : sat_add(starts[i], chunk_len);
            uint32_t ro = 0;
            if (i > 0) {
                uint32_t prev_end = sat_add(starts[i - 1], chunk_len);
                if (prev_end > total) prev_end = total;
                ro = sat_sub(prev_end, starts[i]);
            }
            out.push_back({starts[i], end, ro});
        }
    }
    *n_chunks = (int32_t)out.size();
    if ((int64_t)out.size() > max_chunks)
        return host_fail(LTX_ERR_INVALID_ARG, "ltx_chunk_plan: %zu chunks do not fit in max_chunks %d", out.size(),
                         max_chunks);
    for (size_t i = 0; i < out.size(); ++i) chunks_out[i] = out[i];
    return LTX_OK;
}

extern "C" int ltx_seam_blend(ltx_ctx *ctx, const float *outgoing_dev, const float *incoming_dev,
                              uint32_t overlap_frames, int64_t frame_values, float *dst_dev) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!outgoing_dev || !incoming_dev || !dst_dev || frame_values < 0)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_seam_blend: null pointer or negative frame size");
    if (overlap_frames > 65535)
        return ltx::fail(ctx, LTX_ERR_UNSUPPORTED, "ltx_seam_blend: %u overlap frames (max 65535)", overlap_frames);
    cudaError_t e = launch_seam_blend(ctx->stream, ctx->sm_count, outgoing_dev, incoming_dev, dst_dev,
                                      overlap_frames, frame_values);
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_seam_blend");
}

extern "C" int ltx_chunk_assemble(ltx_ctx *ctx, const float *const *chunk_dev, const ltx_chunk *chunks,
                                  int32_t n_chunks, int64_t frame_values, float *dst_dev) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!chunk_dev || !chunks || n_chunks <= 0 || frame_values < 0 || !dst_dev)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_chunk_assemble: bad arguments");
    // validate the plan's shape: contiguous coverage with seams no wider than
    // the overlap of the two chunks that form them
    for (int32_t n = 0; n < n_chunks; ++n) {
        const ltx_chunk c = chunks[n];
        if (!chunk_dev[n] || c.end <= c.start)
            return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_chunk_assemble: chunk %d is empty or null", n);
        if (n == 0 ? (c.start != 0 || c.real_overlap != 0)
                   : (c.start + c.real_overlap != chunks[n - 1].end || c.start <= chunks[n - 1].start ||
                      c.real_overlap > c.end - c.start))
            return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_chunk_assemble: chunk %d does not follow the plan", n);
        if (n >= 2 && c.start < chunks[n - 2].end)
            return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_chunk_assemble: frame in three chunks at chunk %d", n);
        if (c.real_overlap > 65535)
            return ltx::fail(ctx, LTX_ERR_UNSUPPORTED, "ltx_chunk_assemble: seam of %u frames", c.real_overlap);
    }
    const size_t fbytes = (size_t)frame_values * sizeof(float);
    for (int32_t n = 0; n < n_chunks; ++n) {
        const ltx_chunk c = chunks[n];
        // seam with the previous chunk: frames [start, start + real_overlap)
        if (c.real_overlap > 0) {
            const ltx_chunk p = chunks[n - 1];
            const float *old_tail = chunk_dev[n - 1] + (int64_t)(c.start - p.start) * frame_values;
            cudaError_t e = launch_seam_blend(ctx->stream, ctx->sm_count, old_tail, chunk_dev[n],
                                              dst_dev + (int64_t)c.start * frame_values, c.real_overlap,
                                              frame_values);
            if (e != cudaSuccess) return ltx::cuda_fail(ctx, e, "ltx_chunk_assemble: seam blend");
        }
        // frames only this chunk covers: [start + real_overlap, next.start or end)
        const uint32_t from = c.start + c.real_overlap;
        const uint32_t to = n + 1 < n_chunks ? chunks[n + 1].start : c.end;
        if (to > from && fbytes > 0) {
            cudaError_t e = cudaMemcpyAsync(dst_dev + (int64_t)from * frame_values,
                                            chunk_dev[n] + (int64_t)(from - c.start) * frame_values,
                                            (size_t)(to - from) * fbytes, cudaMemcpyDeviceToDevice, ctx->stream);
            if (e != cudaSuccess) return ltx::cuda_fail(ctx, e, "ltx_chunk_assemble: copy");
        }
    }
    return LTX_OK;
}
