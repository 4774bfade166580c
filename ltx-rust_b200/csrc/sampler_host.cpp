// Host-side ltx-sampler pieces of the denoise loop: the sigma schedule and the
// token position grids, with the reference's exact f32 operation order.
//   LTX2Scheduler::execute       crates/ltx-sampler/src/scheduler.rs:67-125
//   make_target_positions        crates/ltx-sampler/src/patchifier.rs:101-118, 222-264
//   make_reference_positions     patchifier.rs:131-161, 267-332
//   time_coords_s                patchifier.rs:183-194
#include <cmath>
#include <cstdint>
#include <vector>

#include "../../include/ltx_b200.h"

namespace {

// u32 saturating arithmetic as in time_coords_s.
inline uint32_t sat_add(uint32_t a, uint32_t b) { return a > UINT32_MAX - b ? UINT32_MAX : a + b; }
inline uint32_t sat_sub(uint32_t a, uint32_t b) { return a > b ? a - b : 0; }
inline uint32_t sat_mul(uint32_t a, uint32_t b) {
    const uint64_t r = (uint64_t)a * b;
    return r > UINT32_MAX ? UINT32_MAX : (uint32_t)r;
}

void time_coords(uint32_t frame, uint32_t time_scale, float fps, float &s, float &e) {
    const uint32_t start = sat_sub(sat_add(sat_mul(frame, time_scale), 1), time_scale);
    const uint32_t end = sat_sub(sat_add(sat_mul(sat_add(frame, 1), time_scale), 1), time_scale);
    s = (float)start / fps;
    e = (float)end / fps;
}

}  // namespace

extern "C" int ltx_scheduler_execute(int32_t steps, uint64_t num_tokens, float max_shift, float base_shift,
                                     int32_t stretch, float terminal, float *sigmas_out) {
    if (steps < 0 || !sigmas_out) return LTX_ERR_INVALID_ARG;
    const int n = steps;
    const float denom = (float)n;
    std::vector<float> s(n + 1);
    for (int i = 0; i <= n; ++i) s[i] = denom == 0.0f ? 1.0f : 1.0f - (float)i / denom;
    const float tokens = (float)num_tokens;
    const float mm = (max_shift - base_shift) / (4096.0f - 1024.0f);
    const float b_off = std::fma(mm, -1024.0f, base_shift);
    const float shift = std::fma(mm, tokens, b_off);
    const float e = std::exp(shift);
    for (auto &v : s)
        if (v != 0.0f) v = e / std::fma(e, 1.0f, 1.0f / v - 1.0f);
    if (stretch) {
        int last = -1;
        for (int i = 0; i <= n; ++i)
            if (s[i] != 0.0f) last = i;
        if (last >= 0) {
            const float sf = (1.0f - s[last]) / (1.0f - terminal);
            for (int i = 0; i <= n; ++i)
                if (s[i] != 0.0f) s[i] = 1.0f - (1.0f - s[i]) / sf;
        }
    }
    for (int i = 0; i <= n; ++i) sigmas_out[i] = s[i];
    return LTX_OK;
}

extern "C" int ltx_target_positions(uint32_t frames, uint32_t height, uint32_t width, uint32_t batch,
                                    uint32_t scale_t, uint32_t scale_h, uint32_t scale_w, float fps,
                                    float *out_host) {
    if (!out_host || scale_t == 0 || scale_h == 0 || scale_w == 0) return LTX_ERR_INVALID_ARG;
    const uint64_t hw = (uint64_t)height * width, T = frames * hw;
    for (uint32_t b = 0; b < batch; ++b) {
        float *o = out_host + (uint64_t)b * 3 * T * 2;
        for (uint64_t t = 0; t < T; ++t) {
            const uint32_t f = (uint32_t)(t / hw), rem = (uint32_t)(t % hw);
            const uint32_t h = rem / width, w = rem % width;
            time_coords(f, scale_t, fps, o[t * 2], o[t * 2 + 1]);
            o[(T + t) * 2] = (float)sat_mul(h, scale_h);
            o[(T + t) * 2 + 1] = (float)sat_mul(h + 1, scale_h);
            o[(2 * T + t) * 2] = (float)sat_mul(w, scale_w);
            o[(2 * T + t) * 2 + 1] = (float)sat_mul(w + 1, scale_w);
        }
    }
    return LTX_OK;
}

extern "C" int ltx_reference_positions(uint32_t frames, uint32_t height, uint32_t width, uint32_t batch,
                                       uint32_t first_latent_frame, uint32_t scale_t, uint32_t scale_h,
                                       uint32_t scale_w, float fps, uint32_t temporal_scale_factor,
                                       uint32_t downscale_factor, float *out_host) {
    if (!out_host || scale_t == 0 || scale_h == 0 || scale_w == 0 || temporal_scale_factor == 0)
        return LTX_ERR_INVALID_ARG;
    const uint64_t hw = (uint64_t)height * width, T = frames * hw;
    const float ref_fps = fps / (float)temporal_scale_factor;
    const float shift_s = (float)sat_sub(temporal_scale_factor, 1) / fps;
    const float ds = (float)downscale_factor;
    for (uint32_t b = 0; b < batch; ++b) {
        float *o = out_host + (uint64_t)b * 3 * T * 2;
        for (uint64_t t = 0; t < T; ++t) {
            const uint32_t f = (uint32_t)(t / hw), rem = (uint32_t)(t % hw);
            const uint32_t h = rem / width, w = rem % width;
            float s, e;
            time_coords(f + first_latent_frame, scale_t, ref_fps, s, e);
            o[t * 2] = std::fmax(s - shift_s, 0.0f);
            o[t * 2 + 1] = std::fmax(e - shift_s, 0.0f);
            o[(T + t) * 2] = (float)sat_mul(h, scale_h) * ds;
            o[(T + t) * 2 + 1] = (float)sat_mul(h + 1, scale_h) * ds;
            o[(2 * T + t) * 2] = (float)sat_mul(w, scale_w) * ds;
            o[(2 * T + t) * 2 + 1] = (float)sat_mul(w + 1, scale_w) * ds;
        }
    }
    return LTX_OK;
}
