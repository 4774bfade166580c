"""numpy float32 restatement of the ltx-sampler pieces on the denoise-step path.

TEST INFRASTRUCTURE ONLY (checker for the CUDA sampler kernels and the C++
host loop; never imported by the product library).

  LTX2Scheduler::execute       crates/ltx-sampler/src/scheduler.rs:67-125
  patchify / unpatchify        crates/ltx-sampler/src/patchifier.rs:50-89
  target / reference positions patchifier.rs:101-161, 183-332
  VideoReferenceCondition      crates/ltx-sampler/src/conditioning.rs:63-106
  ImageKeyframeCondition       conditioning.rs:127-205
  apply_noise                  crates/ltx-sampler/src/noiser.rs:91-106
  GuidedDenoiser::apply        crates/ltx-sampler/src/guidance.rs:102-195
  post_process / euler_step    crates/ltx-sampler/src/loop_.rs:37-65
  euler_denoising_loop         loop_.rs:93-149, clear_conditioning :162-185

Parity: the scheduler is pinned by the known values of scheduler.rs:205-216;
CFG and Euler by the toy-model tests of guidance.rs:222-281 and
loop_.rs:203-357.  The reference has no golden vector from upstream for the
CFG rescale or the Euler update; for those the reference's Rust code itself
is the specification restated here.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


class SamplerError(Exception):
    def __init__(self, kind, msg=""):
        super().__init__(f"{kind}: {msg}")
        self.kind = kind


def scheduler_execute(steps: int, num_tokens: int, max_shift=2.05, base_shift=0.95,
                      stretch=True, terminal=0.1):
    """LTX2Scheduler::execute, f32 arithmetic with the reference's FMA placement."""
    n = int(steps)
    denom = f32(n)
    sig = [f32(1.0) if denom == 0 else f32(f32(1.0) - f32(f32(i) / denom)) for i in range(n + 1)]
    tokens = f32(num_tokens)
    mm = f32(f32(f32(max_shift) - f32(base_shift)) / f32(f32(4096.0) - f32(1024.0)))
    b_off = _fma(mm, f32(-1024.0), f32(base_shift))
    shift = _fma(mm, tokens, b_off)
    e = _expf(shift)
    out = []
    for s in sig:
        if s != 0:
            s = f32(e / _fma(e, f32(1.0), f32(f32(f32(1.0) / s) - f32(1.0))))
        out.append(s)
    if stretch:
        nz = [i for i, v in enumerate(out) if v != 0]
        if nz:
            last = out[nz[-1]]
            sf = f32(f32(f32(1.0) - last) / f32(f32(1.0) - f32(terminal)))
            for i in nz:
                out[i] = f32(f32(1.0) - f32(f32(f32(1.0) - out[i]) / sf))
    return np.array(out, dtype=np.float32)


def _fma(a, b, c):
    """f32 fused multiply-add with one rounding (Rust f32::mul_add), through C fmaf."""
    from oracle.weight_store import lib
    return f32(lib().oracle_fmaf(float(a), float(b), float(c)))


def _expf(x):
    """Rust f32::exp, through C expf."""
    from oracle.weight_store import lib
    return f32(lib().oracle_expf(float(x)))


def patchify(latent):
    """[B,C,F,H,W] -> [B,F*H*W,C] (patchifier.rs:50-60)."""
    B, C, F, H, W = latent.shape
    return np.ascontiguousarray(latent.transpose(0, 2, 3, 4, 1).reshape(B, F * H * W, C))


def unpatchify(tokens, F, H, W):
    B, T, C = tokens.shape
    if T != F * H * W:
        raise SamplerError("Shape")
    return np.ascontiguousarray(tokens.reshape(B, F, H, W, C).transpose(0, 4, 1, 2, 3))


def _time_coords_s(frame, time_scale, fps):
    """patchifier.rs:183-194 (u32 saturating arithmetic)."""
    start = max(frame * time_scale + 1 - time_scale, 0)
    end = max((frame + 1) * time_scale + 1 - time_scale, 0)
    return f32(f32(start) / f32(fps)), f32(f32(end) / f32(fps))


def target_positions(F, H, W, batch=1, scale=(8, 32, 32), fps=24.0):
    """make_target_positions -> [B,3,T,2] f32 (patchifier.rs:101-118, 222-264)."""
    ts, hs, ws = scale
    T = F * H * W
    out = np.zeros((3, T, 2), np.float32)
    for t in range(T):
        f, rem = divmod(t, H * W)
        h, w = divmod(rem, W)
        out[0, t] = _time_coords_s(f, ts, fps)
        out[1, t] = (h * hs, (h + 1) * hs)
        out[2, t] = (w * ws, (w + 1) * ws)
    return np.broadcast_to(out, (batch, 3, T, 2)).copy()


def reference_positions(F, H, W, batch=1, first_latent_frame=0, scale=(8, 32, 32), fps=24.0,
                        temporal_scale_factor=1, downscale_factor=1):
    """make_reference_positions (patchifier.rs:131-161, 267-332)."""
    ts, hs, ws = scale
    ref_fps = f32(f32(fps) / f32(temporal_scale_factor))
    shift_s = f32(f32(max(temporal_scale_factor - 1, 0)) / f32(fps))
    ds = f32(downscale_factor)
    T = F * H * W
    out = np.zeros((3, T, 2), np.float32)
    for t in range(T):
        f, rem = divmod(t, H * W)
        h, w = divmod(rem, W)
        a, b = _time_coords_s(f + first_latent_frame, ts, ref_fps)
        out[0, t] = (max(f32(a - shift_s), f32(0)), max(f32(b - shift_s), f32(0)))
        out[1, t] = (f32(h * hs) * ds, f32((h + 1) * hs) * ds)
        out[2, t] = (f32(w * ws) * ds, f32((w + 1) * ws) * ds)
    return np.broadcast_to(out, (batch, 3, T, 2)).copy()


class LatentState:
    """state.rs:19-32 (attention/keyframe masks unused on this path)."""

    def __init__(self, latent, denoise_mask, positions, clean_latent):
        self.latent = latent
        self.denoise_mask = denoise_mask
        self.positions = positions
        self.clean_latent = clean_latent


def apply_reference(state: LatentState, ref_latent5, strength=1.0, fps=24.0,
                    temporal_scale_factor=1, downscale_factor=1, first_latent_frame=0):
    """VideoReferenceCondition::apply_to (conditioning.rs:63-106)."""
    B, C, F, H, W = ref_latent5.shape
    ref_tok = patchify(ref_latent5)
    Tr = ref_tok.shape[1]
    pos = reference_positions(F, H, W, B, first_latent_frame, fps=fps,
                              temporal_scale_factor=temporal_scale_factor,
                              downscale_factor=downscale_factor)
    mask = np.full((B, Tr, 1), f32(1.0) - f32(strength), np.float32)
    return LatentState(np.concatenate([state.latent, np.zeros((B, Tr, C), np.float32)], 1),
                       np.concatenate([state.denoise_mask, mask], 1),
                       np.concatenate([state.positions, pos], 2),
                       np.concatenate([state.clean_latent, ref_tok], 1))


def apply_keyframe(state: LatentState, image_latent, latent_frame_index, tokens_per_frame, strength):
    """ImageKeyframeCondition::apply_to (conditioning.rs:127-205): image_latent [B, C, 1, H, W];
    clean[span] <- its tokens, mask[span] <- 1 - strength, every value as Burn computes it
    (clean*keep + img*frame, mask*keep + frame*(1-strength), f32 mul then add)."""
    s = f32(strength)
    if not (f32(0) <= s <= f32(1)):
        raise SamplerError("InvalidStrength", str(strength))
    B, C, F1, H, W = image_latent.shape
    if H * W != tokens_per_frame:
        raise SamplerError("Shape", "image_latent H*W does not match tokens_per_frame")
    img_tok = patchify(image_latent)
    T = state.latent.shape[1]
    start, end = latent_frame_index * tokens_per_frame, (latent_frame_index + 1) * tokens_per_frame
    if end > T:
        raise SamplerError("Shape", "image keyframe index exceeds latent frame count")
    img_clean = np.zeros(state.clean_latent.shape, np.float32)
    img_clean[:, start:end] = img_tok
    frame = np.zeros((B, T, 1), np.float32)
    frame[:, start:end] = 1.0
    keep = (np.float32(1.0) - frame).astype(np.float32)
    clean = (state.clean_latent * keep).astype(np.float32) + (img_clean * frame).astype(np.float32)
    mask = (state.denoise_mask * keep).astype(np.float32) + (frame * f32(f32(1.0) - s)).astype(np.float32)
    return LatentState(state.latent, mask.astype(np.float32), state.positions, clean.astype(np.float32))


def apply_noise(state: LatentState, noise, noise_scale):
    """noiser.rs:91-106."""
    ns = f32(noise_scale)
    noised = state.latent * (f32(1) - ns) + noise * ns
    m = state.denoise_mask
    out = state.clean_latent * (f32(1) - m) + noised * m
    return LatentState(out.astype(np.float32), m, state.positions, state.clean_latent)


def tensor_std(x):
    """tensor3_std (guidance.rs:178-195): sqrt(mean((x-mean)^2) + 1e-8), over all elements.
    Accumulated in f64 here; the reference's f32 reduction order is backend-defined."""
    x64 = x.astype(np.float64)
    m = x64.mean()
    return np.sqrt(((x64 - m) ** 2).mean() + 1e-8)


def cfg_combine(cond, uncond, cfg_scale, rescale_scale):
    """guidance.rs:149-165."""
    if abs(f32(cfg_scale) - f32(1.0)) <= 1e-5:
        return cond.copy()
    pred = cond + (cond - uncond) * f32(f32(cfg_scale) - f32(1.0))
    if abs(rescale_scale) < 1e-6:
        return pred.astype(np.float32)
    ratio = tensor_std(cond) / tensor_std(pred)
    adj = ratio * rescale_scale + (1.0 - rescale_scale)
    return (pred * f32(adj)).astype(np.float32)


def post_process(x0, mask, clean):
    """loop_.rs:37-44."""
    return x0 * mask + clean * (f32(1) - mask)


def euler_step(latent, x0_adj, sigma, sigma_next):
    """loop_.rs:56-65."""
    dt = f32(f32(sigma_next) - f32(sigma))
    v = (latent - x0_adj) / f32(sigma)
    return (latent + v * dt).astype(np.float32)


def velocity_to_x0(latent, timesteps, velocity):
    """x0 = latent - t * v per token: the adapter between a velocity-predicting
    DiT (model.rs:247-254 returns velocity) and the x0 protocol of
    VideoDenoiserModel (model.rs:40-51 of ltx-sampler).  The reference has no
    such adapter; this is the build's rule (upstream LTX-2's X0 wrapper)."""
    return (latent - timesteps[..., None] * velocity).astype(np.float32)


def check_sigmas(sigma, sigma_next, step):
    """loop_.rs:126-137."""
    if not np.isfinite(sigma) or sigma <= 0:
        raise SamplerError("InvalidSigma", f"step {step}: {sigma}")
    if not np.isfinite(sigma_next) or sigma_next < 0:
        raise SamplerError("InvalidSigma", f"step {step + 1}: {sigma_next}")


def euler_loop(sigmas, state: LatentState, target_tokens, model_x0, context, negative_context,
               cfg_scale=1.0, rescale_scale=0.7):
    """euler_denoising_loop (loop_.rs:93-149) with GuidedDenoiser::apply inlined.
    model_x0(latent, timesteps, positions, context) -> x0."""
    if len(sigmas) < 2:
        raise SamplerError("EmptySchedule", str(len(sigmas)))
    for i in range(len(sigmas) - 1):
        s, sn = f32(sigmas[i]), f32(sigmas[i + 1])
        check_sigmas(s, sn, i)
        ts = (state.denoise_mask[..., 0] * s).astype(np.float32)
        cond = model_x0(state.latent, ts, state.positions, context)
        if abs(f32(cfg_scale) - f32(1.0)) > 1e-5:
            if negative_context is None:
                raise SamplerError("MissingNegativeContext")
            unc = model_x0(state.latent, ts, state.positions, negative_context)
            x0 = cfg_combine(cond, unc, cfg_scale, rescale_scale)
        else:
            x0 = cond
        x0a = post_process(x0, state.denoise_mask, state.clean_latent)
        state = LatentState(euler_step(state.latent, x0a, s, sn), state.denoise_mask,
                            state.positions, state.clean_latent)
    return clear_conditioning(state, target_tokens)


def clear_conditioning(state: LatentState, target):
    """loop_.rs:162-185."""
    avail = state.latent.shape[1]
    if target > avail:
        raise SamplerError("TargetTokensTooLarge", f"{target} > {avail}")
    return LatentState(state.latent[:, :target], state.denoise_mask[:, :target],
                       state.positions[:, :, :target], state.clean_latent[:, :target])


def smoothstep(t):
    """ltx-chunk blend.rs:33-40: 3t^2 - 2t^3 with t clamped to [0, 1]."""
    t = np.clip(np.float32(t), 0.0, 1.0)
    return np.float32(t * t * (3.0 - 2.0 * t))
