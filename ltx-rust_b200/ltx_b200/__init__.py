"""ctypes binding of libltx_b200.so (the C ABI in include/ltx_b200.h).

This is the thin layer a Python caller (the tests, bench.py) uses; it mirrors
the names of the reference crates' entry points it wraps.  The compute path is
entirely in the shared library; when the library cannot be loaded every call
raises (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import weakref
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libltx_b200.so")

LTX_F32, LTX_F16, LTX_BF16, LTX_F8_E4M3, LTX_F8_E5M2 = 0, 1, 2, 3, 4
MAX_DELTAS = 8
COMM_ID_BYTES = 128

STATUS = {
    0: "OK", 1: "INVALID_ARG", 2: "SHAPE", 3: "DTYPE", 4: "MISSING_KEY", 5: "DUPLICATE_KEY",
    6: "LORA_RANK", 7: "NO_LORA_MATCHES", 8: "IO", 9: "FORMAT", 10: "CONFIG", 11: "SIGMA",
    12: "SCHEDULE", 13: "CUDA", 14: "NCCL", 15: "TIMEOUT", 16: "OOM", 17: "UNSUPPORTED",
    18: "MISSING_CONFIG", 19: "NEGATIVE_CONTEXT", 20: "CHUNK_PLAN",
    21: "TARGET_TOKENS", 22: "STRENGTH",
}


class LtxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ltx_b200 error {STATUS.get(code, code)}: {msg}")
        self.code = code
        self.kind = STATUS.get(code, str(code))


class LoraDelta(ctypes.Structure):
    _fields_ = [("a_dev", ctypes.c_void_p), ("b_dev", ctypes.c_void_p), ("rank", ctypes.c_int32),
                ("a_dtype", ctypes.c_int32), ("b_dtype", ctypes.c_int32), ("coeff", ctypes.c_float)]


class Chunk(ctypes.Structure):
    """ltx_chunk (plan::Chunk): frames [start, end) and the overlap with the previous chunk."""
    _fields_ = [("start", ctypes.c_uint32), ("end", ctypes.c_uint32), ("real_overlap", ctypes.c_uint32)]

    def as_tuple(self):
        return (self.start, self.end, self.real_overlap)


_lib = None


def lib() -> ctypes.CDLL:
    """Loads the library (raising if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run `python ltx-rust_b200/build.py` first")
    L = ctypes.CDLL(LIB_PATH)
    V, I, F, P, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int64
    sig = {
        "ltx_ctx_create": (I, [I, V, ctypes.POINTER(V)]),
        "ltx_ctx_destroy": (None, [V]),
        "ltx_last_error": (ctypes.c_char_p, [V]),
        "ltx_ctx_stream": (V, [V]),
        "ltx_ctx_synchronize": (I, [V]),
        "ltx_lora_coeff": (F, [F, F, ctypes.c_int32]),
        "ltx_dequant_merge": (I, [V, P, ctypes.c_int32, ctypes.c_int32, F, I64, I64,
                                  ctypes.POINTER(LoraDelta), ctypes.c_int32, P, ctypes.c_int32]),
        "ltx_gemm_bf16": (I, [V, P, I64, P, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                              P, P, I64, P, P, I64]),
        "ltx_gemm_e4m3": (I, [V, P, I64, P, P, I64, F, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                              ctypes.c_int32, P, P, I64, P, P, I64, P, I64, P, I64, ctypes.c_int32]),
        "ltx_quantize_rows_e4m3": (I, [V, P, I64, ctypes.c_int32, ctypes.c_int32, P, I64, P]),
        "ltx_attention_fwd": (I, [V, P, I64, P, I64, P, I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, F, P, I64]),
        "ltx_store_open": (I, [V, ctypes.POINTER(ctypes.c_char_p), ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(V)]),
        "ltx_store_destroy": (None, [V]),
        "ltx_store_merge_lora": (I, [V, ctypes.c_char_p, F, ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32)]),
        "ltx_store_contains": (I, [V, ctypes.c_char_p]),
        "ltx_store_num_keys": (ctypes.c_int32, [V]),
        "ltx_store_key": (ctypes.c_char_p, [V, ctypes.c_int32]),
        "ltx_store_shape": (I, [V, ctypes.c_char_p, ctypes.POINTER(I64), ctypes.c_int32,
                                ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
        "ltx_store_metadata": (I, [V, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t,
                                   ctypes.POINTER(ctypes.c_size_t)]),
        "ltx_store_read": (I, [V, ctypes.c_char_p, ctypes.c_int32, P, ctypes.c_size_t]),
        "ltx_model_load": (I, [V, V, ctypes.c_char_p, ctypes.POINTER(V)]),
        "ltx_model_init_random": (I, [V, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int32, F, ctypes.POINTER(V)]),
        "ltx_model_destroy": (None, [V]),
        "ltx_model_weight_bytes": (I64, [V]),
        "ltx_model_forward": (I, [V, V, P, P, P, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, P]),
        "ltx_block_forward": (I, [V, V, ctypes.c_int32, P, P, P, P, P, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.c_int32]),
        "ltx_cfg_euler_step": (I, [V, P, P, P, P, P, ctypes.c_int32, ctypes.c_int32, F, F, F, F]),
        "ltx_denoise_step": (I, [V, V, P, P, P, P, P, P, P, ctypes.c_int32, ctypes.c_int32, F, F, F, F]),
        "ltx_denoise_loop": (I, [V, V, P, P, P, P, P, P, P, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int32, F, F,
                                 ctypes.c_int32, P]),
        "ltx_apply_noise": (I, [V, P, P, P, P, ctypes.c_int32, ctypes.c_int32, F]),
        "ltx_apply_keyframe": (I, [V, P, P, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int32, ctypes.c_int32, F]),
        "ltx_seam_cond_plan": (I, [ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_float),
                                   ctypes.POINTER(ctypes.c_uint32)]),
        "ltx_scheduler_execute": (I, [ctypes.c_int32, ctypes.c_uint64, F, F, ctypes.c_int32, F, P]),
        "ltx_target_positions": (I, [ctypes.c_uint32] * 7 + [F, P]),
        "ltx_reference_positions": (I, [ctypes.c_uint32] * 8 + [F, ctypes.c_uint32, ctypes.c_uint32, P]),
        "ltx_patchify": (I, [V, P] + [ctypes.c_int32] * 5 + [P]),
        "ltx_unpatchify": (I, [V, P] + [ctypes.c_int32] * 5 + [P]),
        "ltx_host_last_error": (ctypes.c_char_p, []),
        "ltx_comm_unique_id": (I, [P, ctypes.c_size_t]),
        "ltx_ctx_init_comm": (I, [V, P, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32]),
        "ltx_ctx_comm_check": (I, [V]),
        "ltx_ctx_init_cfg_comm": (I, [V, P, ctypes.c_size_t, ctypes.c_int32]),
        "ltx_ctx_tp_exchange": (I, [V]),
        "ltx_ctx_abort_comm": (None, [V]),
        "ltx_wait_flag": (I, [V, P, ctypes.c_int32, ctypes.c_uint32]),
        "ltx_set_flag": (I, [V, P, ctypes.c_int32]),
        "ltx_chunk_plan": (I, [ctypes.c_uint32] * 3 + [ctypes.POINTER(Chunk), ctypes.c_int32,
                                                        ctypes.POINTER(ctypes.c_int32)]),
        "ltx_crossfade_weight": (F, [ctypes.c_uint32, ctypes.c_uint32]),
        "ltx_seam_blend": (I, [V, P, P, ctypes.c_uint32, I64, P]),
        "ltx_chunk_assemble": (I, [V, ctypes.POINTER(P), ctypes.POINTER(Chunk), ctypes.c_int32, I64, P]),
        "ltx_dequant_merge_noalloc": (I, [V, P, ctypes.c_int32, ctypes.c_int32, F, I64, I64,
                                          ctypes.POINTER(LoraDelta), ctypes.c_int32, P, ctypes.c_int32,
                                          ctypes.c_char_p, ctypes.c_size_t]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class Context:
    """An ltx_ctx bound to a CUDA device and stream (default: torch's current stream)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(device).cuda_stream
        self.h = ctypes.c_void_p()
        # stores and models made on this context: closed before it (their
        # destructors synchronise on the context's stream)
        self._owned = weakref.WeakSet()
        rc = lib().ltx_ctx_create(device, ctypes.c_void_p(stream), ctypes.byref(self.h))
        if rc != 0:
            raise LtxError(rc, f"ltx_ctx_create(device={device})")

    def check(self, rc: int, what: str):
        if rc != 0:
            msg = lib().ltx_last_error(self.h)
            raise LtxError(rc, f"{what}: {msg.decode() if msg else ''}")

    def init_comm(self, comm_id: bytes, nranks: int, rank: int):
        """Binds this context to rank `rank` of a tensor-parallel group (collective)."""
        buf = ctypes.create_string_buffer(bytes(comm_id), COMM_ID_BYTES)
        self.check(lib().ltx_ctx_init_comm(self.h, buf, COMM_ID_BYTES, nranks, rank), "ltx_ctx_init_comm")

    def tp_exchange(self) -> str:
        """How tensor-parallel sums run on this context (ltx_ctx_tp_exchange)."""
        return {0: "none", 1: "peer", 2: "nccl"}[lib().ltx_ctx_tp_exchange(self.h)]

    def init_cfg_comm(self, comm_id: bytes, cfg_rank: int):
        """Makes this context half of a CFG-parallel pair (ltx_ctx_init_cfg_comm)."""
        buf = ctypes.create_string_buffer(comm_id, len(comm_id))
        self.check(lib().ltx_ctx_init_cfg_comm(self.h, buf, len(comm_id), cfg_rank), "ltx_ctx_init_cfg_comm")

    def comm_check(self):
        self.check(lib().ltx_ctx_comm_check(self.h), "ltx_ctx_comm_check")

    def abort_comm(self):
        lib().ltx_ctx_abort_comm(self.h)

    def wait_flag(self, flag, expect: int, timeout_ms: int = 2000):
        """Enqueues a bounded device-side wait until flag (int32 device tensor/pointer) == expect."""
        self.check(lib().ltx_wait_flag(self.h, _ptr(flag), expect, timeout_ms), "ltx_wait_flag")

    def set_flag(self, flag, value: int):
        self.check(lib().ltx_set_flag(self.h, _ptr(flag), value), "ltx_set_flag")

    def synchronize(self):
        self.check(lib().ltx_ctx_synchronize(self.h), "synchronize")

    def close(self):
        if self.h:
            for obj in list(self._owned):
                obj.close()
            lib().ltx_ctx_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ── ltx-weights ──────────────────────────────────────────────────────────
    def dequant_merge(self, w_ptr: int, w_dtype: int, has_scale: bool, scale: float, out_features: int,
                      in_features: int, deltas, dst_ptr: int, dst_dtype: int):
        """WeightStore::read body on device pointers (ltx_dequant_merge)."""
        n = len(deltas)
        arr = (LoraDelta * max(n, 1))(*[LoraDelta(*d) for d in deltas])
        self.check(lib().ltx_dequant_merge(self.h, ctypes.c_void_p(w_ptr), w_dtype, int(has_scale), scale,
                                           out_features, in_features, arr, n, ctypes.c_void_p(dst_ptr),
                                           dst_dtype), "ltx_dequant_merge")


EPI_BF16, EPI_GELU_BF16, EPI_F32, EPI_RESID = 0, 1, 2, 3


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t if isinstance(t, int) else t.data_ptr())


def gemm(ctx: "Context", a, w, out, epilogue=EPI_BF16, bias=None, gate=None, gate_idx=None):
    """out = epilogue(a @ w.T) with torch CUDA tensors (a [M,K] bf16, w [N,K] bf16)."""
    M, K = a.shape
    N = w.shape[0]
    ctx.check(lib().ltx_gemm_bf16(ctx.h, _ptr(a), a.stride(0), _ptr(w), w.stride(0), M, N, K, epilogue,
                                  _ptr(bias), _ptr(out), out.stride(0), _ptr(gate), _ptr(gate_idx),
                                  gate.stride(0) if gate is not None else 0), "ltx_gemm_bf16")


def gemm_e4m3(ctx: "Context", a, a_scale, w, w_scale, out, epilogue=EPI_BF16, bias=None, gate=None, gate_idx=None,
              w_col_scale=None, a2=None, b2=None):
    """out = epilogue(((a @ w.T) + a2 @ b2.T) * a_scale[:, None] * w_scale) with e4m3 operands a [M,K],
    w [N,K] held as uint8 (or float8_e4m3fn) CUDA tensors; a_scale f32 [M] or None; w_col_scale f32 [N]
    overrides w_scale per column; a2 [M,k2] / b2 [N,k2] bf16 append a low-rank block (k2 % 64 == 0)."""
    M, K = a.shape
    N = w.shape[0]
    k2 = 0 if a2 is None else a2.shape[1]
    ctx.check(lib().ltx_gemm_e4m3(ctx.h, _ptr(a), a.stride(0), _ptr(a_scale), _ptr(w), w.stride(0), float(w_scale),
                                  _ptr(w_col_scale), M, N, K, epilogue, _ptr(bias), _ptr(out), out.stride(0), _ptr(gate),
                                  _ptr(gate_idx), gate.stride(0) if gate is not None else 0, _ptr(a2),
                                  a2.stride(0) if a2 is not None else 0, _ptr(b2),
                                  b2.stride(0) if b2 is not None else 0, k2), "ltx_gemm_e4m3")


def quantize_rows_e4m3(ctx: "Context", x, out, scale):
    """Per-row e4m3 of a bf16 [rows, cols] CUDA tensor into uint8 out [rows, cols] and f32 scale [rows]."""
    rows, cols = x.shape
    ctx.check(lib().ltx_quantize_rows_e4m3(ctx.h, _ptr(x), x.stride(0), rows, cols, _ptr(out), out.stride(0),
                                           _ptr(scale)), "ltx_quantize_rows_e4m3")


def attention(ctx: "Context", q, k, v, out, batch, heads, tq, tk, scale, head_dim=128):
    """out = softmax(q k^T * scale) v; q/k/out token-major bf16 CUDA tensors, v bf16 or f16 (row stride = stride(0))."""
    import torch
    vdt = LTX_F16 if v.dtype == torch.float16 else LTX_BF16
    ctx.check(lib().ltx_attention_fwd(ctx.h, _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0), vdt,
                                      batch, heads, tq, tk, head_dim, scale, _ptr(out), out.stride(0)),
              "ltx_attention_fwd")


KEYMAP_IDENTITY, KEYMAP_TRANSFORMER = 0, 1


class WeightStore:
    """ltx-weights WeightStore over the C ABI (ltx_store_*); reads land in device memory."""

    def __init__(self, ctx: Context, paths, keymap=KEYMAP_IDENTITY):
        self.ctx = ctx
        self.h = ctypes.c_void_p()
        arr = (ctypes.c_char_p * len(paths))(*[p.encode() for p in paths])
        ctx.check(lib().ltx_store_open(ctx.h, arr, len(paths), keymap, ctypes.byref(self.h)), "ltx_store_open")
        ctx._owned.add(self)

    def merge_lora(self, path: str, strength: float):
        m, u = ctypes.c_int32(), ctypes.c_int32()
        self.ctx.check(lib().ltx_store_merge_lora(self.h, path.encode(), strength, ctypes.byref(m), ctypes.byref(u)),
                       "ltx_store_merge_lora")
        return m.value, u.value

    def contains(self, key):
        return bool(lib().ltx_store_contains(self.h, key.encode()))

    def keys(self):
        return [lib().ltx_store_key(self.h, i).decode() for i in range(lib().ltx_store_num_keys(self.h))]

    def shape(self, key):
        dims = (ctypes.c_int64 * 8)()
        nd, dt = ctypes.c_int32(), ctypes.c_int32()
        self.ctx.check(lib().ltx_store_shape(self.h, key.encode(), dims, 8, ctypes.byref(nd), ctypes.byref(dt)),
                       "ltx_store_shape")
        return [dims[i] for i in range(nd.value)]

    def metadata(self, key):
        need = ctypes.c_size_t()
        rc = lib().ltx_store_metadata(self.h, key.encode(), None, 0, ctypes.byref(need))
        if rc != 0:
            raise LtxError(rc, f"metadata {key!r}")
        buf = ctypes.create_string_buffer(need.value)
        lib().ltx_store_metadata(self.h, key.encode(), buf, need.value, None)
        return buf.value.decode()

    def read(self, key, dtype=LTX_F32):
        """Returns a torch CUDA tensor (f32 or bf16) with the stored shape."""
        import torch
        shape = self.shape(key)
        t = torch.empty(shape, dtype=torch.float32 if dtype == LTX_F32 else torch.bfloat16, device="cuda")
        self.ctx.check(lib().ltx_store_read(self.h, key.encode(), dtype, _ptr(t), t.numel() * t.element_size()),
                       "ltx_store_read")
        return t

    def close(self):
        if self.h:
            lib().ltx_store_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VideoTransformer:
    """ltx-dit VideoTransformer over the C ABI (ltx_model_*)."""

    def __init__(self, ctx: Context, handle):
        self.ctx, self.h = ctx, handle
        ctx._owned.add(self)

    @staticmethod
    def load(ctx: Context, store: WeightStore, config_json: str | None = None):
        h = ctypes.c_void_p()
        ctx.check(lib().ltx_model_load(ctx.h, store.h, config_json.encode() if config_json else None, ctypes.byref(h)),
                  "ltx_model_load")
        return VideoTransformer(ctx, h)

    @staticmethod
    def init_random(ctx: Context, config_json: str, seed=0, lora_rank=64, lora_strength=1.0):
        h = ctypes.c_void_p()
        ctx.check(lib().ltx_model_init_random(ctx.h, config_json.encode(), seed, lora_rank, lora_strength,
                                              ctypes.byref(h)), "ltx_model_init_random")
        return VideoTransformer(ctx, h)

    def weight_bytes(self):
        return lib().ltx_model_weight_bytes(self.h)

    def forward(self, latent, timesteps, positions, context, out):
        """latent [B,T,in], timesteps [B,T], positions [B,3,T,2], context [B,S,Dc] -> out [B,T,out] (f32 CUDA)."""
        B, T, _ = latent.shape
        S = context.shape[1]
        self.ctx.check(lib().ltx_model_forward(self.h, self.ctx.h, _ptr(latent), _ptr(timesteps), _ptr(positions),
                                               _ptr(context), B, T, S, _ptr(out)), "ltx_model_forward")

    def block_forward(self, index, x, context, timestep, pe_cos, pe_sin):
        """TransformerBlock::forward of block `index` in place on x [B,T,D] (ltx_block_forward):
        context [B,S,Dc], timestep [B,T,K*D] (per-token modulation), pe_cos/pe_sin as
        precompute_freqs_cis returns them (split: [B,H,T,d/2]), all f32 CUDA."""
        B, T, _ = x.shape
        S = context.shape[1]
        self.ctx.check(lib().ltx_block_forward(self.h, self.ctx.h, index, _ptr(x), _ptr(context), _ptr(timestep),
                                               _ptr(pe_cos), _ptr(pe_sin), B, T, S), "ltx_block_forward")

    def denoise_step(self, latent, clean, mask, positions, ctx_cond, ctx_uncond, sigma, sigma_next, cfg_scale=1.0,
                     rescale_scale=0.7, mask_host=None):
        """One guided Euler step in place on latent [T, C] (ltx_denoise_step)."""
        T = latent.shape[0]
        S = ctx_cond.shape[0]
        mh = None
        if mask_host is not None:
            mh = mask_host.ctypes.data_as(ctypes.c_void_p)
        self.ctx.check(lib().ltx_denoise_step(self.h, self.ctx.h, _ptr(latent), _ptr(clean), mh, _ptr(mask),
                                              _ptr(positions), _ptr(ctx_cond), _ptr(ctx_uncond), T, S, sigma,
                                              sigma_next, cfg_scale, rescale_scale), "ltx_denoise_step")

    def denoise_loop(self, latent, clean, mask, positions, ctx_cond, ctx_uncond, sigmas, cfg_scale=1.0,
                     rescale_scale=0.7, target_tokens=None, out=None, mask_host=None):
        """euler_denoising_loop + clear_conditioning on the device (ltx_denoise_loop): every
        step in place on latent [T, C]; the first target_tokens tokens are copied to out."""
        import numpy as np
        T = latent.shape[0]
        S = ctx_cond.shape[0]
        sig = np.ascontiguousarray(np.asarray(sigmas, np.float32))
        mh = None if mask_host is None else mask_host.ctypes.data_as(ctypes.c_void_p)
        tt = T if target_tokens is None else target_tokens
        self.ctx.check(lib().ltx_denoise_loop(self.h, self.ctx.h, _ptr(latent), _ptr(clean), mh, _ptr(mask),
                                              _ptr(positions), _ptr(ctx_cond), _ptr(ctx_uncond), T, S,
                                              sig.ctypes.data_as(ctypes.c_void_p), len(sig), cfg_scale,
                                              rescale_scale, tt, _ptr(out)), "ltx_denoise_loop")

    def close(self):
        if self.h:
            lib().ltx_model_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def cfg_euler_step(ctx: "Context", cond_x0, uncond_x0, latent, clean, mask, sigma, sigma_next, cfg_scale=1.0,
                   rescale_scale=0.7):
    """CFG + rescale + post_process + Euler in place on latent [T, C] from x0 predictions
    (ltx_cfg_euler_step); uncond_x0 may be None when cfg_scale is 1."""
    T, C = latent.shape
    ctx.check(lib().ltx_cfg_euler_step(ctx.h, _ptr(cond_x0), _ptr(uncond_x0), _ptr(latent), _ptr(clean), _ptr(mask),
                                       T, C, sigma, sigma_next, cfg_scale, rescale_scale), "ltx_cfg_euler_step")


def apply_noise(ctx: "Context", latent, noise, clean, mask, noise_scale):
    """GaussianNoiser::apply_with_noise in place on latent [T, C] (ltx_apply_noise)."""
    T, C = latent.shape
    ctx.check(lib().ltx_apply_noise(ctx.h, _ptr(latent), _ptr(noise), _ptr(clean), _ptr(mask), T, C, noise_scale),
              "ltx_apply_noise")


def apply_keyframe(ctx: "Context", clean, mask, image, latent_frame_index, strength):
    """ImageKeyframeCondition::apply_to in place on clean [T, C] and mask [T] (ltx_apply_keyframe):
    image is the one-frame latent [C, 1, H, W] (or [C, H*W]); f32 CUDA tensors."""
    T, C = clean.shape
    tpf = image.numel() // C
    ctx.check(lib().ltx_apply_keyframe(ctx.h, _ptr(clean), _ptr(mask), T, C, _ptr(image), latent_frame_index, tpf,
                                       strength), "ltx_apply_keyframe")


def seam_cond_plan(overlap):
    """seam_cond_plan -> (chunk_local_idx, strength, blend_tail_len) (host, no GPU needed)."""
    idx, st, tail = ctypes.c_uint32(), ctypes.c_float(), ctypes.c_uint32()
    rc = lib().ltx_seam_cond_plan(overlap, ctypes.byref(idx), ctypes.byref(st), ctypes.byref(tail))
    if rc:
        raise LtxError(rc, lib().ltx_host_last_error().decode())
    return idx.value, st.value, tail.value


def scheduler_execute(steps, num_tokens, max_shift=2.05, base_shift=0.95, stretch=True, terminal=0.1):
    """LTX2Scheduler::execute -> list of steps+1 f32 sigmas (host, no GPU needed)."""
    import numpy as np
    out = np.empty(steps + 1, np.float32)
    rc = lib().ltx_scheduler_execute(steps, num_tokens, max_shift, base_shift, int(stretch), terminal,
                                     out.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise LtxError(rc, "ltx_scheduler_execute")
    return out


def target_positions(frames, height, width, batch=1, scale=(8, 32, 32), fps=24.0):
    """make_target_positions -> np.float32 [batch, 3, F*H*W, 2] (host, no GPU needed)."""
    import numpy as np
    out = np.empty((batch, 3, frames * height * width, 2), np.float32)
    rc = lib().ltx_target_positions(frames, height, width, batch, *scale, fps, out.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise LtxError(rc, "ltx_target_positions")
    return out


def reference_positions(frames, height, width, batch=1, first_latent_frame=0, scale=(8, 32, 32), fps=24.0,
                        temporal_scale_factor=1, downscale_factor=1):
    """make_reference_positions -> np.float32 [batch, 3, F*H*W, 2] (host, no GPU needed)."""
    import numpy as np
    out = np.empty((batch, 3, frames * height * width, 2), np.float32)
    rc = lib().ltx_reference_positions(frames, height, width, batch, first_latent_frame, *scale, fps,
                                       temporal_scale_factor, downscale_factor, out.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise LtxError(rc, "ltx_reference_positions")
    return out


def patchify(ctx: "Context", latent5, tokens):
    B, C, F, H, W = latent5.shape
    ctx.check(lib().ltx_patchify(ctx.h, _ptr(latent5), B, C, F, H, W, _ptr(tokens)), "ltx_patchify")


def unpatchify(ctx: "Context", tokens, latent5):
    B, C, F, H, W = latent5.shape
    ctx.check(lib().ltx_unpatchify(ctx.h, _ptr(tokens), B, C, F, H, W, _ptr(latent5)), "ltx_unpatchify")


NOALLOC_SCRATCH_BYTES = 16 << 20


def dequant_merge_noalloc(stream: int, w_ptr: int, w_dtype: int, has_scale: bool, scale: float, out_features: int,
                          in_features: int, deltas, dst_ptr: int, dst_dtype: int):
    """ltx_dequant_merge_noalloc: the same merge without allocating device memory
    (for callers that cannot call cudaMalloc); raises LtxError with the library's message."""
    n = len(deltas)
    arr = (LoraDelta * max(n, 1))(*[LoraDelta(*d) for d in deltas])
    err = ctypes.create_string_buffer(512)
    rc = lib().ltx_dequant_merge_noalloc(ctypes.c_void_p(stream), ctypes.c_void_p(w_ptr), w_dtype, int(has_scale),
                                         scale, out_features, in_features, arr, n, ctypes.c_void_p(dst_ptr),
                                         dst_dtype, err, len(err))
    if rc != 0:
        raise LtxError(rc, err.value.decode())


def lora_coeff(strength: float, alpha: float, rank: int) -> float:
    return lib().ltx_lora_coeff(strength, alpha, rank)


# ── temporal chunks (crates/ltx-chunk) ─────────────────────────────────────────

def chunk_plan(total: int, chunk_len: int, overlap: int):
    """plan::plan -> [(start, end, real_overlap), ...] (host, no GPU needed).
    Raises LtxError(kind "CHUNK_PLAN") naming the ChunkError variant."""
    n = ctypes.c_int32(0)
    cap = max(1, total // max(1, chunk_len - overlap) + 2)
    arr = (Chunk * cap)()
    rc = lib().ltx_chunk_plan(total, chunk_len, overlap, arr, cap, ctypes.byref(n))
    if rc:
        raise LtxError(rc, lib().ltx_host_last_error().decode())
    return [arr[i].as_tuple() for i in range(n.value)]


def crossfade_weight(offset: int, overlap_len: int) -> float:
    """blend::crossfade_weight (host)."""
    return lib().ltx_crossfade_weight(offset, overlap_len)


def seam_blend(ctx: "Context", outgoing, incoming, dst):
    """Blends overlap frames on the device: tensors [frames, ...] f32 (dst may be incoming)."""
    frames = outgoing.shape[0]
    fv = outgoing.numel() // max(frames, 1)
    ctx.check(lib().ltx_seam_blend(ctx.h, _ptr(outgoing), _ptr(incoming), frames, fv, _ptr(dst)), "ltx_seam_blend")


def chunk_assemble(ctx: "Context", chunk_tensors, chunks, dst):
    """The clip the reference's Blender emits, from per-chunk device tensors [len_n, ...] f32."""
    n = len(chunks)
    ptrs = (ctypes.c_void_p * n)(*[_ptr(t) for t in chunk_tensors])
    arr = (Chunk * n)(*[Chunk(*c) for c in chunks])
    fv = dst.numel() // max(dst.shape[0], 1)
    ctx.check(lib().ltx_chunk_assemble(ctx.h, ptrs, arr, n, fv, _ptr(dst)), "ltx_chunk_assemble")


# ── tensor parallelism ─────────────────────────────────────────────────────────

def comm_unique_id() -> bytes:
    """A fresh communicator id (host only; rank 0 makes it and shares it)."""
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    rc = lib().ltx_comm_unique_id(buf, COMM_ID_BYTES)
    if rc:
        raise LtxError(rc, lib().ltx_host_last_error().decode())
    return buf.raw


def share_comm_id(group=None) -> bytes:
    """Rank 0's fresh communicator id, broadcast to every rank of a torch.distributed group."""
    import torch.distributed as dist
    obj = [comm_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def init_tensor_parallel(ctx: "Context", group=None):
    """Binds ctx to this process's rank of a torch.distributed group (collective)."""
    import torch.distributed as dist
    rank, ws = dist.get_rank(group), dist.get_world_size(group)
    if ws > 1:
        ctx.init_comm(share_comm_id(group), ws, rank)


def cfg_tp_layout(world_size: int, rank: int):
    """CFG-parallel x tensor-parallel placement of `rank` among `world_size` (even)
    GPUs: ranks [0, n/2) run the conditional pass, [n/2, n) the unconditional one,
    each half one tensor-parallel group; rank r pairs with r + n/2.
    Returns (cfg_rank, tp_size, tp_rank, tp_group_ranks, pair_ranks)."""
    if world_size < 2 or world_size % 2:
        raise ValueError(f"CFG-parallel needs an even number of ranks, not {world_size}")
    half = world_size // 2
    cfg_rank, tp_rank = divmod(rank, half)
    return (cfg_rank, half, tp_rank, list(range(cfg_rank * half, cfg_rank * half + half)),
            [tp_rank, tp_rank + half])


def init_cfg_tensor_parallel(ctx: "Context"):
    """Binds ctx to its CFG pair and (for more than 2 ranks) its tensor-parallel group,
    over the default torch.distributed group; the ids travel over torch.distributed.
    Every rank creates every subgroup in the same order (new_group is collective)."""
    import torch.distributed as dist
    ws, rank = dist.get_world_size(), dist.get_rank()
    cfg_rank, half, tp_rank, tp_ranks, pair = cfg_tp_layout(ws, rank)
    tp_groups = [dist.new_group(list(range(g * half, g * half + half))) for g in range(2)]
    pair_groups = [dist.new_group([r, r + half]) for r in range(half)]
    if half > 1:
        g = tp_groups[cfg_rank]
        obj = [comm_unique_id() if rank == tp_ranks[0] else None]
        dist.broadcast_object_list(obj, src=tp_ranks[0], group=g)
        ctx.init_comm(obj[0], half, tp_rank)
    g = pair_groups[tp_rank]
    obj = [comm_unique_id() if rank == pair[0] else None]
    dist.broadcast_object_list(obj, src=pair[0], group=g)
    ctx.init_cfg_comm(obj[0], cfg_rank)
    return cfg_rank, half, tp_rank
