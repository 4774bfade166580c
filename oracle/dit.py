"""CPU (torch float32) restatement of the ltx-dit forward pass.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA DiT path, never imported by
the product library.  Pinned by the reference's golden fixtures
crates/ltx-dit/tests/fixtures/dit_parity{,_gated_adaln}.safetensors (copied to
tests/golden/ by tests/golden/make_golden.py) at the reference's own tolerance
(atol 1e-4 OR rtol 1e-3, crates/ltx-dit/tests/parity.rs:37-63).

Each function cites the reference code it restates:
  config/flags         crates/ltx-dit/src/config.rs:56-231
  rms_norm / LN        crates/ltx-dit/src/norm.rs:23-53
  adaLN-single         crates/ltx-dit/src/adaln.rs:43-142
  RoPE (split)         crates/ltx-dit/src/rope.rs:46-167, 231-257, 311-322
  RoPE (interleaved)   crates/ltx-dit/src/rope.rs:172-219, 269-293
  attention            crates/ltx-dit/src/attention.rs:137-195, 228-242
  feed-forward         crates/ltx-dit/src/feed_forward.rs:38-42
  block                crates/ltx-dit/src/block.rs:118-236
  model                crates/ltx-dit/src/model.rs:169-255
  loader key layout    crates/ltx-dit/src/load.rs:9-27
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class DiTConfig:
    """DiTConfig with the reference defaults (config.rs:98-151)."""
    num_attention_heads: int = 32
    attention_head_dim: int = 128
    in_channels: int = 128
    out_channels: int = 128
    num_layers: int = 28
    cross_attention_dim: int = 4096
    norm_eps: float = 1e-6
    positional_embedding_theta: float = 10000.0
    positional_embedding_max_pos: list = field(default_factory=lambda: [20, 2048, 2048])
    timestep_scale_multiplier: int = 1000
    use_middle_indices_grid: bool = True
    rope_type: str = "split"
    apply_gated_attention: bool = False
    cross_attention_adaln: bool = False
    use_prompt_adaln_single: bool = True
    ff_bias: bool = False
    use_keyframes_abs_pos_embedding: bool = False
    caption_proj_before_connector: bool = False

    @staticmethod
    def from_json(d: dict) -> "DiTConfig":
        d = d.get("transformer", d)
        c = DiTConfig()
        for k, v in d.items():
            if hasattr(c, k):
                setattr(c, k, v)
        c.validate()
        return c

    @property
    def inner_dim(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def adaln_coeff(self) -> int:
        return 9 if self.cross_attention_adaln else 6

    def validate(self):
        """config.rs:188-231."""
        if self.num_attention_heads == 0:
            raise ValueError("num_attention_heads must be > 0")
        if self.attention_head_dim % 2:
            raise ValueError("attention_head_dim must be even for RoPE")
        inner = self.inner_dim
        if inner < 2 * len(self.positional_embedding_max_pos):
            raise ValueError("inner_dim too small for RoPE")
        if (inner // 2) % self.num_attention_heads:
            raise ValueError("inner_dim/2 must be divisible by heads")
        if self.cross_attention_adaln and self.use_prompt_adaln_single:
            raise ValueError("use_prompt_adaln_single with cross_attention_adaln is not wired")
        if self.use_keyframes_abs_pos_embedding:
            raise ValueError("use_keyframes_abs_pos_embedding is not wired")


def rms_norm(x, eps):
    """norm.rs:23-35: x / sqrt(mean_f32(x^2) + eps)."""
    return x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def layer_norm_no_affine(x, eps):
    """norm.rs:46-53."""
    mean = x.mean(-1, keepdim=True)
    sh = x - mean
    var = sh.pow(2).mean(-1, keepdim=True)
    return sh / torch.sqrt(var + eps)


def rms_norm_gamma(x, gamma, eps):
    """Burn RmsNorm (q_norm/k_norm, attention.rs:109-114): x / sqrt(mean(x^2)+eps) * gamma."""
    return x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps) * gamma


def gelu_tanh(x):
    """tanh-approximate GELU (feed_forward.rs:31-32)."""
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x.pow(3))))


def linear(x, w, b=None):
    y = x @ w.t()
    return y + b if b is not None else y


def sinusoidal_emb(t):
    """adaln.rs:43-59: freqs exp(-ln(1e4) i/128) in f32, output [cos, sin]."""
    log10k = np.float32(math.log(10000.0))
    i = np.arange(128, dtype=np.float32)
    freqs = torch.from_numpy(np.exp(-log10k * i / np.float32(128.0)).astype(np.float32))
    ang = t.float().reshape(-1, 1) * freqs.reshape(1, -1)
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1)


def make_freq_grid(theta: float, n: int):
    """rope.rs:311-322: theta^(i/(n-1)) * pi/2 computed in f64, stored f32."""
    if n == 0:
        return np.zeros(0, np.float32)
    if n == 1:
        return np.array([theta * math.pi / 2.0], np.float32)
    return np.array([theta ** (i / (n - 1)) * math.pi / 2.0 for i in range(n)], dtype=np.float64).astype(np.float32)


def rope_angles(positions, cfg: DiTConfig):
    """rope.rs:46-116: angles (B, T, grid*n_pos) with (grid, axis) flattening."""
    B, n_pos, T, _ = positions.shape
    inner = cfg.inner_dim
    grid = inner // (2 * n_pos)
    freq = torch.from_numpy(make_freq_grid(cfg.positional_embedding_theta, grid))
    maxp = torch.tensor([float(m) for m in cfg.positional_embedding_max_pos], dtype=torch.float32).reshape(1, n_pos, 1)
    ps, pe = positions[..., 0], positions[..., 1]
    frac = ((ps + pe) / 2.0) / maxp if cfg.use_middle_indices_grid else ps / maxp
    fm = frac * 2.0 + (-1.0)
    f = fm.transpose(1, 2).reshape(B, T, n_pos, 1) * freq.reshape(1, 1, 1, grid)
    return f.transpose(2, 3).reshape(B, T, grid * n_pos)


def precompute_freqs_cis(positions, cfg: DiTConfig):
    """rope.rs:46-167: split -> (B,H,T,d/2) each; interleaved -> (B,1,T,inner)."""
    f = rope_angles(positions, cfg)
    B, T, cur = f.shape
    inner, H = cfg.inner_dim, cfg.num_attention_heads
    cos, sin = torch.cos(f), torch.sin(f)
    if cfg.rope_type == "split":
        pad = inner // 2 - cur
        if pad > 0:
            cos = torch.cat([torch.ones(B, T, pad), cos], 2)
            sin = torch.cat([torch.zeros(B, T, pad), sin], 2)
        dh = inner // 2 // H
        return (cos.reshape(B, T, H, dh).transpose(1, 2), sin.reshape(B, T, H, dh).transpose(1, 2))
    cos = torch.stack([cos, cos], -1).reshape(B, T, 2 * cur)
    sin = torch.stack([sin, sin], -1).reshape(B, T, 2 * cur)
    pad = inner - 2 * cur
    if pad > 0:
        cos = torch.cat([torch.ones(B, T, pad), cos], 2)
        sin = torch.cat([torch.zeros(B, T, pad), sin], 2)
    return cos.reshape(B, 1, T, inner), sin.reshape(B, 1, T, inner)


def apply_split_rope(x, cos, sin, heads):
    """rope.rs:231-257."""
    B, T, inner = x.shape
    d = inner // heads
    half = d // 2
    x4 = x.reshape(B, T, heads, d).transpose(1, 2)
    x1, x2 = x4[..., :half], x4[..., half:]
    o1 = cos * x1 - sin * x2
    o2 = sin * x1 + cos * x2
    return torch.cat([o1, o2], 3).transpose(1, 2).reshape(B, T, inner)


def apply_interleaved_rope(x, cos, sin):
    """rope.rs:269-293."""
    B, T, inner = x.shape
    c, s = cos.reshape(B, T, inner), sin.reshape(B, T, inner)
    xp = x.reshape(B, T, inner // 2, 2)
    rot = torch.stack([-xp[..., 1], xp[..., 0]], -1).reshape(B, T, inner)
    return x * c + rot * s


def attention(p, pre, cfg: DiTConfig, x, context=None, pe=None, mask=None):
    """attention.rs:137-195 with sdp_attention :228-242 (materialised softmax)."""
    kv = x if context is None else context
    B, Tq, _ = x.shape
    Tk = kv.shape[1]
    H, d = cfg.num_attention_heads, cfg.attention_head_dim
    q = linear(x, p[pre + "to_q.weight"], p.get(pre + "to_q.bias"))
    k = linear(kv, p[pre + "to_k.weight"], p.get(pre + "to_k.bias"))
    v = linear(kv, p[pre + "to_v.weight"], p.get(pre + "to_v.bias"))
    q = rms_norm_gamma(q, p[pre + "q_norm.weight"], cfg.norm_eps)
    k = rms_norm_gamma(k, p[pre + "k_norm.weight"], cfg.norm_eps)
    if pe is not None:
        cos, sin = pe
        if cfg.rope_type == "split":
            q, k = apply_split_rope(q, cos, sin, H), apply_split_rope(k, cos, sin, H)
        else:
            q, k = apply_interleaved_rope(q, cos, sin), apply_interleaved_rope(k, cos, sin)
    q4 = q.reshape(B, Tq, H, d).transpose(1, 2)
    k4 = k.reshape(B, Tk, H, d).transpose(1, 2)
    v4 = v.reshape(B, Tk, H, d).transpose(1, 2)
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    out = sdpa(q4, k4, v4, float(scale), mask)
    out = out.transpose(1, 2).reshape(B, Tq, H * d)
    if cfg.apply_gated_attention:
        g = torch.sigmoid(linear(x, p[pre + "to_gate_logits.weight"], p.get(pre + "to_gate_logits.bias"))) * 2.0
        out = (out.reshape(B, Tq, H, d) * g.reshape(B, Tq, H, 1)).reshape(B, Tq, H * d)
    return linear(out, p[pre + "to_out.0.weight"], p.get(pre + "to_out.0.bias"))


SDPA_Q_CHUNK = 2048   # rows of scores materialised at once (memory bound for full-size runs)


def sdpa(q, k, v, scale, mask=None, q_chunk=None):
    """softmax(q k^T * scale + mask) v; rows are processed in query chunks,
    which is the reference's own chunked_sdp_attention (attention.rs:252-285):
    identical per-row results, bounded memory."""
    q_chunk = q_chunk or SDPA_Q_CHUNK
    outs = []
    for s in range(0, q.shape[2], q_chunk):
        sc = (q[:, :, s:s + q_chunk] @ k.transpose(2, 3)) * scale
        if mask is not None:
            sc = sc + mask[:, :, s:s + q_chunk]
        outs.append(torch.softmax(sc, dim=3) @ v)
    return torch.cat(outs, 2)


def ada_values(sst, timestep, start):
    """block.rs:164-198: (shift, scale, gate) = sst[start+i] + timestep[..., start+i, :]."""
    B, T, cd = timestep.shape
    coeff, inner = sst.shape
    ts = timestep.reshape(B, T, coeff, inner)
    comb = sst[start:start + 3].reshape(1, 1, 3, inner) + ts[:, :, start:start + 3]
    return comb[:, :, 0], comb[:, :, 1], comb[:, :, 2]


def block_forward(p, i, cfg: DiTConfig, x, context, timestep, pe):
    """block.rs:118-153 (and cross_attn_adaln :209-236)."""
    pre = f"transformer_blocks.{i}."
    sst = p[pre + "scale_shift_table"]
    sh, sc, g = ada_values(sst, timestep, 0)
    nx = rms_norm(x, cfg.norm_eps) * (sc + 1.0) + sh
    x = x + attention(p, pre + "attn1.", cfg, nx, None, pe) * g
    nx2 = rms_norm(x, cfg.norm_eps)
    if cfg.cross_attention_adaln:
        shq, scq, gq = ada_values(sst, timestep, 6)
        xm = nx2 * (scq + 1.0) + shq
        ctx = context
        pst = p.get(pre + "prompt_scale_shift_table")
        if pst is not None:
            ctx = context * (pst[1].reshape(1, 1, -1) + 1.0) + pst[0].reshape(1, 1, -1)
        ca = attention(p, pre + "attn2.", cfg, xm, ctx, None) * gq
    else:
        ca = attention(p, pre + "attn2.", cfg, nx2, context, None)
    x = x + ca
    sh2, sc2, g2 = ada_values(sst, timestep, 3)
    ffin = rms_norm(x, cfg.norm_eps) * (sc2 + 1.0) + sh2
    h = gelu_tanh(linear(ffin, p[pre + "ff.net.0.proj.weight"], p.get(pre + "ff.net.0.proj.bias")))
    return x + linear(h, p[pre + "ff.net.2.weight"], p.get(pre + "ff.net.2.bias")) * g2


def adaln_single(p, cfg: DiTConfig, ts_flat):
    """adaln.rs:130-142: returns (modulation (N, coeff*inner), embedded_timestep (N, inner))."""
    e = sinusoidal_emb(ts_flat)
    pre = "adaln_single.emb.timestep_embedder."
    h = torch.nn.functional.silu(linear(e, p[pre + "linear_1.weight"], p[pre + "linear_1.bias"]))
    emb = linear(h, p[pre + "linear_2.weight"], p[pre + "linear_2.bias"])
    mod = linear(torch.nn.functional.silu(emb), p["adaln_single.linear.weight"], p["adaln_single.linear.bias"])
    return mod, emb


def model_forward(p, cfg: DiTConfig, latent, timesteps, positions, context, n_blocks=None):
    """model.rs:169-255.  p: dict name -> f32 tensor in the checkpoint layout ([out, in])."""
    B, T, _ = latent.shape
    x = linear(latent, p["patchify_proj.weight"], p["patchify_proj.bias"])
    ts = (timesteps * float(cfg.timestep_scale_multiplier)).reshape(B * T)
    mod, emb = adaln_single(p, cfg, ts)
    mod = mod.reshape(B, T, -1)
    emb = emb.reshape(B, T, -1)
    pe = precompute_freqs_cis(positions, cfg)
    for i in range(cfg.num_layers if n_blocks is None else n_blocks):
        x = block_forward(p, i, cfg, x, context, mod, pe)
    sst = p["scale_shift_table"]
    shift = sst[0].reshape(1, 1, -1) + emb
    scale = sst[1].reshape(1, 1, -1) + emb
    xo = layer_norm_no_affine(x, cfg.norm_eps) * (scale + 1.0) + shift
    return linear(xo, p["proj_out.weight"], p["proj_out.bias"])


def load_params(tensors: dict) -> dict:
    """name -> torch f32 tensor from {name: np.ndarray}."""
    return {k: torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)) for k, v in tensors.items()}
