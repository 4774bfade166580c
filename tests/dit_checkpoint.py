"""Writes small LTX-style DiT checkpoints for tests: FP8 e4m3 linear weights
with per-tensor `_scale` siblings under `model.diffusion_model.` (the real
checkpoint layout, read with KeyMap::transformer), f32 norms and tables, plus
a bf16 IC-LoRA file with `.lora_A/.lora_B/.alpha` keys.  Seeded numpy RNG."""
import json

import numpy as np
import torch

from oracle.weight_store import f32_to_bf16_bits, write_safetensors

PREFIX = "model.diffusion_model."


def small_config(heads=2, head_dim=128, layers=2, in_ch=128, cross_dim=None, **flags):
    d = heads * head_dim
    cfg = {"num_attention_heads": heads, "attention_head_dim": head_dim, "in_channels": in_ch, "out_channels": in_ch,
           "num_layers": layers, "cross_attention_dim": cross_dim or d, "norm_eps": 1e-6,
           "positional_embedding_theta": 10000.0, "positional_embedding_max_pos": [20, 2048, 2048],
           "timestep_scale_multiplier": 1000, "use_middle_indices_grid": True, "rope_type": "split",
           "apply_gated_attention": False, "cross_attention_adaln": False, "use_prompt_adaln_single": True,
           "ff_bias": False, "use_keyframes_abs_pos_embedding": False, "caption_proj_before_connector": True}
    cfg.update(flags)
    return cfg


def _fp8(w: np.ndarray):
    scale = np.float32(np.abs(w).max() / 448.0)
    q = torch.from_numpy((w / scale).astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return q.tobytes(), np.array(scale, np.float32).tobytes()


def linear_shapes(cfg):
    D = cfg["num_attention_heads"] * cfg["attention_head_dim"]
    Dc, K = cfg["cross_attention_dim"], (9 if cfg["cross_attention_adaln"] else 6)
    shapes = {"patchify_proj": (D, cfg["in_channels"]), "proj_out": (cfg["out_channels"], D),
              "adaln_single.emb.timestep_embedder.linear_1": (D, 256),
              "adaln_single.emb.timestep_embedder.linear_2": (D, D), "adaln_single.linear": (K * D, D)}
    for i in range(cfg["num_layers"]):
        p = f"transformer_blocks.{i}."
        for a, kv in (("attn1.", D), ("attn2.", Dc)):
            shapes[p + a + "to_q"] = (D, D)
            shapes[p + a + "to_k"] = (D, kv)
            shapes[p + a + "to_v"] = (D, kv)
            shapes[p + a + "to_out.0"] = (D, D)
        shapes[p + "ff.net.0.proj"] = (4 * D, D)
        shapes[p + "ff.net.2"] = (D, 4 * D)
    return shapes


def write_checkpoint(path, cfg, seed=0, std=0.02):
    rng = np.random.default_rng(seed)
    D = cfg["num_attention_heads"] * cfg["attention_head_dim"]
    K = 9 if cfg["cross_attention_adaln"] else 6
    t = {}
    f32 = lambda a: ("F32", list(a.shape), a.astype(np.float32).tobytes())
    for name, (o, i) in linear_shapes(cfg).items():
        w = (rng.standard_normal((o, i)) * std).astype(np.float32)
        q, s = _fp8(w)
        t[PREFIX + name + ".weight"] = ("F8_E4M3", [o, i], q)
        t[PREFIX + name + ".weight_scale"] = ("F32", [], s)
        if not (name.startswith("transformer_blocks") and ".ff." in name and not cfg["ff_bias"]):
            t[PREFIX + name + ".bias"] = f32((rng.standard_normal(o) * 0.02).astype(np.float32))
    t[PREFIX + "scale_shift_table"] = f32((rng.standard_normal((2, D)) * 0.1).astype(np.float32))
    for i in range(cfg["num_layers"]):
        p = PREFIX + f"transformer_blocks.{i}."
        for a in ("attn1.", "attn2."):
            t[p + a + "q_norm.weight"] = f32((1 + rng.standard_normal(D) * 0.05).astype(np.float32))
            t[p + a + "k_norm.weight"] = f32((1 + rng.standard_normal(D) * 0.05).astype(np.float32))
        t[p + "scale_shift_table"] = f32((rng.standard_normal((K, D)) * 0.1).astype(np.float32))
    write_safetensors(path, t, {"config": json.dumps({"transformer": cfg})})


def write_lora(path, cfg, rank=16, alpha=8.0, seed=1):
    rng = np.random.default_rng(seed)
    t = {}
    for name, (o, i) in linear_shapes(cfg).items():
        if not name.startswith("transformer_blocks"):
            continue
        a = (rng.standard_normal((rank, i)) * 0.01).astype(np.float32)
        b = (rng.standard_normal((o, rank)) * 0.01).astype(np.float32)
        # merge_lora pairs LoRA keys with the store's renamed keys (store.rs:549-560)
        t[name + ".lora_A.weight"] = ("BF16", [rank, i], f32_to_bf16_bits(a).tobytes())
        t[name + ".lora_B.weight"] = ("BF16", [o, rank], f32_to_bf16_bits(b).tobytes())
        t[name + ".alpha"] = ("F32", [], np.array(alpha, np.float32).tobytes())
    write_safetensors(path, t, {"reference_downscale_factor": "1", "reference_temporal_scale_factor": "1"})
