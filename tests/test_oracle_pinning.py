"""Pins the CPU oracle against the reference's own golden vectors and known answers.

Nothing here needs a GPU.  Sources of every expected value:
  fp8 known answers        crates/ltx-weights/src/fp8.rs:161-205
  FP8 / LoRA integration   crates/ltx-weights/tests/integration.rs:400-666
  FP8 / LoRA / keymap fixtures   crates/ltx-weights/tests/parity.rs:23-105
  DiT fixtures             crates/ltx-dit/tests/parity.rs:65-168 (atol 1e-4 OR rtol 1e-3)
  scheduler known values   crates/ltx-sampler/src/scheduler.rs:205-216
  CFG / Euler toy models   crates/ltx-sampler/src/guidance.rs:222-281, loop_.rs:203-357
"""
import math
import os

import numpy as np
import pytest
import torch

from oracle import dit, sampler
from oracle.weight_store import (KeyMap, LoraFile, WeightError, WeightStore, bf16_bits_to_f32,
                                 f32_to_bf16_bits, lib, read_safetensors, write_safetensors)

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def gold(name):
    return os.path.join(GOLD, name)


# ── FP8 decode known answers (fp8.rs:161-205) ────────────────────────────────

def test_e4m3fn_known_values():
    L = lib()
    assert np.float32(L.oracle_decode_e4m3fn(0x00)).tobytes() == np.float32(0.0).tobytes()
    assert np.float32(L.oracle_decode_e4m3fn(0x80)).tobytes() == np.float32(-0.0).tobytes()
    assert math.isnan(L.oracle_decode_e4m3fn(0x7F)) and math.isnan(L.oracle_decode_e4m3fn(0xFF))
    assert L.oracle_decode_e4m3fn(0x38) == 1.0
    # The reference test says "0x77 ... should be 448" but only checks > 100.
    # 0x77 = 0_1110_111 = 2^7 * 1.875 = 240; the max normal 448 is 0x7E.
    assert L.oracle_decode_e4m3fn(0x77) == 240.0
    assert L.oracle_decode_e4m3fn(0x7E) == 448.0
    assert L.oracle_decode_e4m3fn(0x01) == 2.0 ** -9          # min subnormal
    assert L.oracle_decode_e4m3fn(0x07) == 7 * 2.0 ** -9      # max subnormal


def test_e4m3fn_matches_torch_for_all_bytes():
    """torch.float8_e4m3fn is the upstream dtype the fixtures were made with."""
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).float().numpy()
    got = np.array([lib().oracle_decode_e4m3fn(i) for i in range(256)], np.float32)
    nan = np.isnan(ref)
    assert (np.isnan(got) == nan).all()
    assert (got[~nan].view(np.uint32) == ref[~nan].view(np.uint32)).all()


def test_e5m2_matches_torch_for_all_bytes():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e5m2).float().numpy()
    got = np.array([lib().oracle_decode_e5m2(i) for i in range(256)], np.float32)
    nan = np.isnan(ref)
    assert (np.isnan(got) == nan).all()
    assert (got[~nan].view(np.uint32) == ref[~nan].view(np.uint32)).all()
    assert np.isinf(lib().oracle_decode_e5m2(0x7C)) and lib().oracle_decode_e5m2(0xFC) < 0


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e38, -3e38, 1.00390625, 1.01171875], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert (f32_to_bf16_bits(x) == ref).all()
    assert all(lib().oracle_f32_to_bf16(float(v)) == r for v, r in zip(x[:2000], ref[:2000]))


# ── weights fixtures (ltx-weights/tests/parity.rs) ────────────────────────────

def test_fp8_fixture_parity():
    st = WeightStore([gold("fp8_e4m3fn_parity.safetensors")], KeyMap.identity())
    assert not st.contains("w_scale")
    got = st.read("w")
    exp = WeightStore([gold("fp8_e4m3fn_expected.safetensors")], KeyMap.identity()).read("w")
    nan = np.isnan(exp)
    assert (np.isnan(got) == nan).all()
    np.testing.assert_allclose(got[~nan], exp[~nan], atol=1e-5, rtol=0)
    # The fixture's expected values were made with `fp8.float() * scale`; the
    # reference reads with fma(scale, v, 0): both round once, so they are equal.
    assert (got[~nan].view(np.uint32) == exp[~nan].view(np.uint32)).all()


def test_lora_fixture_parity():
    st = WeightStore([gold("lora_parity_base.safetensors")], KeyMap.identity())
    rep = st.merge_lora(LoraFile(gold("lora_parity_lora.safetensors")), 0.75)
    assert "layer.weight" in rep.matched_keys
    got = st.read("layer.weight")
    exp = WeightStore([gold("lora_parity_expected.safetensors")], KeyMap.identity()).read("layer.weight")
    np.testing.assert_allclose(got, exp, atol=5e-2, rtol=0)
    # Stronger than the reference test: the bf16 rounding of our f32 chain equals
    # upstream's bf16 result for every element of the fixture.
    got16 = st.read("layer.weight", want="bf16")
    assert (bf16_bits_to_f32(got16).reshape(exp.shape) == exp).mean() >= 0.9


def test_transformer_keymap_parity():
    st = WeightStore([gold("transformer_keymap_fixture.safetensors")], KeyMap.transformer())
    ex = WeightStore([gold("transformer_keymap_expected.safetensors")], KeyMap.identity())
    key = "transformer_blocks.0.attn1.to_q.weight"
    assert st.contains(key)
    np.testing.assert_array_equal(st.read(key), ex.read(key))
    assert sorted(st.keys()) == sorted(ex.keys())


def test_iclora_layout_fixture():
    assert LoraFile(gold("iclora_layout.safetensors")).ic_layout() == (2, 4)


# ── integration known answers (integration.rs) ───────────────────────────────

def _st(tmp_path, name, tensors, meta=None):
    p = str(tmp_path / name)
    write_safetensors(p, tensors, meta)
    return p


def f32b(v):
    return np.asarray(v, np.float32).tobytes()


def test_fp8_scale_known_answers(tmp_path):
    p = _st(tmp_path, "a.st", {"w": ("F8_E4M3", [1], bytes([0x38]))})
    assert WeightStore([p], KeyMap.identity()).read("w")[0] == 1.0
    p = _st(tmp_path, "b.st", {"w": ("F8_E4M3", [1], bytes([0x38])), "w_scale": ("F32", [1], f32b([3.0]))})
    st = WeightStore([p], KeyMap.identity())
    assert not st.contains("w_scale") and st.read("w")[0] == 3.0
    p = _st(tmp_path, "c.st", {"w": ("F32", [1], f32b([2.0])), "w_scale": ("F32", [1], f32b([100.0]))})
    st = WeightStore([p], KeyMap.identity())
    assert st.contains("w_scale") and st.read("w")[0] == 2.0


def test_fp8_negative_zero_becomes_positive_zero(tmp_path):
    """fma(scale, -0.0, +0.0) = +0.0 (store.rs:506)."""
    p = _st(tmp_path, "z.st", {"w": ("F8_E4M3", [2], bytes([0x80, 0x00])), "w_scale": ("F32", [], f32b([2.0]))})
    got = WeightStore([p], KeyMap.identity()).read("w")
    assert got.view(np.uint32).tolist() == [0, 0]


def test_lora_basic_alpha_stack(tmp_path):
    base = _st(tmp_path, "base.st", {"layer.weight": ("F32", [2, 2], f32b([1, 0, 0, 1]))})
    lora = _st(tmp_path, "l.st", {"layer.lora_A.weight": ("F32", [1, 2], f32b([1, 2])),
                                  "layer.lora_B.weight": ("F32", [2, 1], f32b([3, 4]))})
    st = WeightStore([base], KeyMap.identity())
    rep = st.merge_lora(LoraFile(lora), 1.0)
    assert rep.matched_keys == ["layer.weight"] and rep.unmatched_lora_keys == []
    np.testing.assert_array_equal(st.read("layer.weight").ravel(), [4, 6, 4, 9])
    # alpha = 2, rank 1 -> coeff 2
    base0 = _st(tmp_path, "b0.st", {"w.weight": ("F32", [2, 2], f32b([0, 0, 0, 0]))})
    la = _st(tmp_path, "la.st", {"w.lora_A.weight": ("F32", [1, 2], f32b([1, 2])),
                                 "w.lora_B.weight": ("F32", [2, 1], f32b([3, 4])),
                                 "w.alpha": ("F32", [1], f32b([2.0]))})
    st = WeightStore([base0], KeyMap.identity())
    st.merge_lora(LoraFile(la), 1.0)
    np.testing.assert_array_equal(st.read("w.weight").ravel(), [6, 12, 8, 16])
    # two stacked LoRAs: W + 1.0*B1A1 + 0.5*B2A2
    b1 = _st(tmp_path, "s0.st", {"w.weight": ("F32", [2, 2], f32b([1, 0, 0, 1]))})
    l1 = _st(tmp_path, "s1.st", {"w.lora_A.weight": ("F32", [1, 2], f32b([1, 2])),
                                 "w.lora_B.weight": ("F32", [2, 1], f32b([3, 4]))})
    l2 = _st(tmp_path, "s2.st", {"w.lora_A.weight": ("F32", [2, 2], f32b([1, 0, 0, 1])),
                                 "w.lora_B.weight": ("F32", [2, 2], f32b([2, 0, 0, -2]))})
    st = WeightStore([b1], KeyMap.identity())
    st.merge_lora(LoraFile(l1), 1.0)
    st.merge_lora(LoraFile(l2), 0.5)
    np.testing.assert_array_equal(st.read("w.weight").ravel(), [5, 6, 4, 8])


def test_lora_error_paths(tmp_path):
    base = _st(tmp_path, "b.st", {"present.weight": ("F32", [1], f32b([1.0]))})
    l = _st(tmp_path, "l.st", {"present.lora_A.weight": ("F32", [1, 1], f32b([1])),
                               "present.lora_B.weight": ("F32", [1, 1], f32b([1])),
                               "absent.lora_A.weight": ("F32", [1, 1], f32b([1])),
                               "absent.lora_B.weight": ("F32", [1, 1], f32b([1]))})
    rep = WeightStore([base], KeyMap.identity()).merge_lora(LoraFile(l), 1.0)
    assert "present.weight" in rep.matched_keys and any("absent" in k for k in rep.unmatched_lora_keys)
    l2 = _st(tmp_path, "l2.st", {"absent.lora_A.weight": ("F32", [1, 1], f32b([1])),
                                 "absent.lora_B.weight": ("F32", [1, 1], f32b([1]))})
    with pytest.raises(WeightError) as e:
        WeightStore([base], KeyMap.identity()).merge_lora(LoraFile(l2), 1.0)
    assert e.value.kind == "NoLoraMatches"
    b23 = _st(tmp_path, "b23.st", {"layer.weight": ("F32", [2, 3], f32b([0] * 6))})
    lbad = _st(tmp_path, "lbad.st", {"layer.lora_A.weight": ("F32", [1, 3], f32b([1, 2, 3])),
                                     "layer.lora_B.weight": ("F32", [4, 1], f32b([0] * 4))})
    with pytest.raises(WeightError) as e:
        WeightStore([b23], KeyMap.identity()).merge_lora(LoraFile(lbad), 1.0)
    assert e.value.kind == "LoraShapeMismatch"
    bi = _st(tmp_path, "bi.st", {"layer.weight": ("F32", [1, 1], f32b([0]))})
    li = _st(tmp_path, "li.st", {"layer.lora_A.weight": ("I32", [1, 1], np.int32(7).tobytes()),
                                 "layer.lora_B.weight": ("F32", [1, 1], f32b([1]))})
    with pytest.raises(WeightError) as e:
        WeightStore([bi], KeyMap.identity()).merge_lora(LoraFile(li), 1.0)
    assert e.value.kind == "UnsupportedDtype"


def test_store_error_paths(tmp_path):
    p = _st(tmp_path, "x.st", {"x": ("F32", [1], f32b([0]))})
    with pytest.raises(WeightError) as e:
        WeightStore([p], KeyMap.identity()).read("nope")
    assert e.value.kind == "MissingKey"
    p2 = _st(tmp_path, "y.st", {"x": ("F32", [1], f32b([0]))})
    with pytest.raises(WeightError) as e:
        WeightStore([p, p2], KeyMap.identity())
    assert e.value.kind == "DuplicateKey"
    pi = _st(tmp_path, "i.st", {"w": ("I32", [2], np.array([42, -1], np.int32).tobytes())})
    with pytest.raises(WeightError) as e:
        WeightStore([pi], KeyMap.identity()).read("w")
    assert e.value.kind == "UnsupportedDtype"


def test_merge_chain_is_sequential_fma():
    """A hand-computed chain: the order and rounding of add_to (store.rs:781-791)."""
    from oracle.weight_store import LowRankDelta, read_raw
    rng = np.random.default_rng(3)
    out, inn, R = 5, 7, 3
    base = rng.standard_normal(out * inn).astype(np.float32)
    a = rng.standard_normal((R, inn)).astype(np.float32)
    b = rng.standard_normal((out, R)).astype(np.float32)
    coeff = np.float32(0.37)
    got = read_raw(base.tobytes(), "F32", False, 1.0, out, inn, [LowRankDelta(b, a, out, R, inn, float(coeff))])
    exp = base.reshape(out, inn).copy()
    for o in range(out):
        for r in range(R):
            c = np.float32(coeff * b[o, r])
            for i in range(inn):
                exp[o, i] = lib().oracle_fmaf(float(c), float(a[r, i]), float(exp[o, i]))
    assert (got.view(np.uint32) == exp.ravel().view(np.uint32)).all()


# ── DiT fixtures (ltx-dit/tests/parity.rs) ────────────────────────────────────

def _dit_fixture(name):
    st = WeightStore([gold(name)], KeyMap.identity())
    cfg = dit.DiTConfig.from_json(st.config())
    params = dit.load_params({k: st.read(k) for k in st.keys() if not k.startswith("input.") and k != "output"})
    inp = {k: torch.from_numpy(st.read("input." + k)) for k in ("latent", "timesteps", "positions", "context")}
    return cfg, params, inp, st.read("output")


@pytest.mark.parametrize("name", ["dit_parity.safetensors", "dit_parity_gated_adaln.safetensors"])
def test_dit_fixture_parity(name):
    cfg, params, inp, expected = _dit_fixture(name)
    if "gated" in name:
        assert cfg.apply_gated_attention and cfg.cross_attention_adaln and cfg.ff_bias
    with torch.no_grad():
        out = dit.model_forward(params, cfg, inp["latent"], inp["timesteps"], inp["positions"], inp["context"]).numpy()
    absd = np.abs(out - expected)
    rel = absd / (np.abs(expected) + 1e-8)
    assert ((absd <= 1e-4) | (rel <= 1e-3)).all(), (absd.max(), rel.max())


def test_dit_config_validation():
    c = dit.DiTConfig()
    c.validate()
    with pytest.raises(ValueError):
        dit.DiTConfig(cross_attention_adaln=True, use_prompt_adaln_single=True).validate()
    with pytest.raises(ValueError):
        dit.DiTConfig(use_keyframes_abs_pos_embedding=True).validate()
    with pytest.raises(ValueError):
        dit.DiTConfig(num_attention_heads=0).validate()
    with pytest.raises(ValueError):
        dit.DiTConfig(attention_head_dim=127).validate()
    with pytest.raises(ValueError):
        dit.DiTConfig(num_attention_heads=1, attention_head_dim=4).validate()


def test_rope_grid_shape_for_22b():
    """682-entry grid, 2 pad entries, 32 heads x 64 (rope.rs:46-167)."""
    pos = torch.from_numpy(sampler.target_positions(2, 2, 2))
    cos, sin = dit.precompute_freqs_cis(pos, dit.DiTConfig())
    assert cos.shape == (1, 32, 8, 64)
    c = cos.transpose(1, 2).reshape(1, 8, 2048)
    assert (c[..., :2] == 1).all() and (sin.transpose(1, 2).reshape(1, 8, 2048)[..., :2] == 0).all()


def test_interleaved_rope_pairs():
    """rope.rs:332-350: [a, b] angles -> [a, a, b, b], no pad when inner == 2*len."""
    f = torch.tensor([[[0.0, 1.0]]])
    cos = torch.stack([torch.cos(f), torch.cos(f)], -1).reshape(1, 1, 4)
    exp = np.array([1.0, 1.0, math.cos(1.0), math.cos(1.0)], np.float32)
    np.testing.assert_allclose(cos.numpy().ravel(), exp, atol=1e-6)


# ── sampler (ltx-sampler unit tests) ─────────────────────────────────────────

def test_scheduler_known_values():
    got = sampler.scheduler_execute(5, 1024)
    np.testing.assert_allclose(got, [1.0, 0.8694, 0.6963, 0.4560, 0.1000, 0.0], atol=1e-3)
    assert len(sampler.scheduler_execute(10, 4096)) == 11
    s = sampler.scheduler_execute(10, 4096)
    assert (np.diff(s) <= 0).all() and abs(s[-1]) < 1e-6
    s = sampler.scheduler_execute(3, 4096, stretch=False)
    assert len(s) == 4 and abs(s[-1]) < 1e-6


def test_patchify_roundtrip_and_positions():
    x = np.random.default_rng(0).random((1, 4, 3, 2, 2), dtype=np.float32)
    t = sampler.patchify(x)
    assert t.shape == (1, 12, 4)
    np.testing.assert_array_equal(sampler.unpatchify(t, 3, 2, 2), x)
    pos = sampler.target_positions(3, 1, 1)
    assert pos.shape == (1, 3, 3, 2) and abs(pos[0, 0, 0, 0]) < 1e-6
    assert abs(pos[0, 0, 0, 1] - pos[0, 0, 1, 0]) < 1e-6
    r2 = sampler.reference_positions(1, 1, 1, downscale_factor=2)
    r1 = sampler.reference_positions(1, 1, 1, downscale_factor=1)
    assert abs(r2[0, 1, 0, 0] - 2 * r1[0, 1, 0, 0]) < 1e-4 and abs(r2[0, 1, 0, 1] - 2 * r1[0, 1, 0, 1]) < 1e-4


def test_cfg_and_euler_toy_models():
    ctx = np.ones((1, 4, 16), np.float32)
    st = sampler.LatentState(np.zeros((1, 8, 4), np.float32), np.ones((1, 8, 1), np.float32),
                             np.zeros((1, 3, 8, 2), np.float32), np.zeros((1, 8, 4), np.float32))

    def toy(latent, ts, pos, c):
        return latent + np.float32(c.mean() * 0.1)

    x0 = toy(st.latent, None, None, ctx)
    np.testing.assert_allclose(x0, 0.1, atol=1e-5)

    def zero(latent, ts, pos, c):
        return np.zeros_like(latent)

    s4 = sampler.LatentState(np.full((1, 4, 2), 0.5, np.float32), np.ones((1, 4, 1), np.float32),
                             np.zeros((1, 3, 4, 2), np.float32), np.zeros((1, 4, 2), np.float32))
    res = sampler.euler_loop([0.9, 0.5, 0.1, 0.0], s4, 4, zero, ctx[:, :1, :4], None)
    assert np.abs(res.latent).max() < 1e-5
    with pytest.raises(sampler.SamplerError) as e:
        sampler.euler_loop([0.5], s4, 4, zero, ctx, None)
    assert e.value.kind == "EmptySchedule"
    with pytest.raises(sampler.SamplerError) as e:
        sampler.euler_loop([0.5, 0.0, 0.0], s4, 4, zero, ctx, None)
    assert e.value.kind == "InvalidSigma"
    with pytest.raises(sampler.SamplerError) as e:
        sampler.clear_conditioning(s4, 5)
    assert e.value.kind == "TargetTokensTooLarge"
    s6 = sampler.LatentState(np.zeros((1, 6, 2), np.float32), np.ones((1, 6, 1), np.float32),
                             np.zeros((1, 3, 6, 2), np.float32), np.zeros((1, 6, 2), np.float32))
    assert sampler.clear_conditioning(s6, 4).positions.shape == (1, 3, 4, 2)
    neg = np.zeros((1, 2, 8), np.float32)
    res = sampler.euler_loop([0.8, 0.3, 0.0], s4, 4, toy, np.ones((1, 2, 8), np.float32), neg, cfg_scale=3.0)
    assert res.latent.shape == (1, 4, 2)
