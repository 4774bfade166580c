"""The block and sampler seams of the C ABI against the oracle.

ltx_block_forward runs one TransformerBlock::forward (crates/ltx-dit/src/
block.rs:118-153) on the block's own inputs: the residual stream, the context,
the per-token modulation (`timestep`) and the RoPE tables in the layout
precompute_freqs_cis returns (rope.rs:118-167).  Bar: rel-L2 <= 1e-2 against
oracle/dit.block_forward (the north star's bf16 bar).

ltx_cfg_euler_step runs GuidedDenoiser::apply's combine and rescale
(guidance.rs:149-195) and post_process + euler_step (loop_.rs:37-65) on x0
predictions from any denoiser.  Its arithmetic is f32 with the std in f64 on
both sides, so the bar is a tight relative tolerance (1e-5), not bits: the
two sums are taken in different orders.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import dit, sampler
from oracle.weight_store import KeyMap, LoraFile, WeightStore as OracleStore

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import ltx_b200
    c = ltx_b200.Context(0)
    yield c
    c.close()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _block_case(tmp_path, heads, layers, seed):
    from dit_checkpoint import small_config, write_checkpoint, write_lora
    cfg = small_config(heads=heads, head_dim=128, layers=layers)
    ck, lo = str(tmp_path / f"b{heads}.safetensors"), str(tmp_path / f"l{heads}.safetensors")
    write_checkpoint(ck, cfg, seed=seed)
    write_lora(lo, cfg, rank=16, alpha=8.0, seed=seed + 1)
    o = OracleStore([ck], KeyMap.transformer())
    o.merge_lora(LoraFile(lo), 0.8)
    params = dit.load_params({k: o.read(k, n_threads=os.cpu_count() or 1) for k in o.keys()})
    return cfg, ck, lo, params


@pytest.mark.parametrize("heads,B", [(2, 2), (32, 1)])
def test_block_forward_matches_oracle(ctx, tmp_path, heads, B):
    """Every block of a 2-layer FP8 + LoRA checkpoint, batch rows with different contexts,
    per-token modulation that differs across tokens (as a conditioned latent's does)."""
    import ltx_b200
    cfg, ck, lo, params = _block_case(tmp_path, heads, 2, seed=40 + heads)
    c = dit.DiTConfig.from_json(cfg)
    D, K = heads * 128, 6
    F, Hh, W, S = 2, 8, 8, 48
    T = 2 * F * Hh * W
    rng = np.random.default_rng(heads)
    pos = np.concatenate([sampler.target_positions(F, Hh, W, B), sampler.reference_positions(F, Hh, W, B)], axis=2)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    ctxt = rng.standard_normal((B, S, cfg["cross_attention_dim"])).astype(np.float32)
    mod = (rng.standard_normal((B, T, K * D)) * 0.1).astype(np.float32)
    with torch.no_grad():
        cos, sin = dit.precompute_freqs_cis(torch.from_numpy(pos), c)
    st = ltx_b200.WeightStore(ctx, [ck], ltx_b200.KEYMAP_TRANSFORMER)
    st.merge_lora(lo, 0.8)
    model = ltx_b200.VideoTransformer.load(ctx, st)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    for i in range(cfg["num_layers"]):
        xd = dev(x)
        model.block_forward(i, xd, dev(ctxt), dev(mod), dev(cos.numpy()), dev(sin.numpy()))
        ctx.synchronize()
        with torch.no_grad():
            exp = dit.block_forward(params, i, c, torch.from_numpy(x), torch.from_numpy(ctxt),
                                    torch.from_numpy(mod), (cos, sin)).numpy()
        got = xd.cpu().numpy()
        err, upd = rel_l2(got, exp), rel_l2(got - x, exp - x)
        print(f"\nblock {i} ({heads} heads, batch {B}): rel-L2 {err:.2e}, update rel-L2 {upd:.2e}")
        assert np.isfinite(got).all() and err < 1e-2 and upd < 1e-2
    model.close()
    st.close()


def test_block_forward_rejects_bad_arguments(ctx):
    import ltx_b200
    from dit_checkpoint import small_config
    model = ltx_b200.VideoTransformer.init_random(ctx, json.dumps(small_config(heads=2, layers=1)), seed=1, lora_rank=8)
    z = torch.zeros(1, 4, 256, device="cuda")
    for idx in (-1, 1):
        with pytest.raises(ltx_b200.LtxError) as e:
            model.block_forward(idx, z, z, z, z, z)
        assert e.value.kind == "INVALID_ARG"
    model.close()


def _cfg_case(T=3000, C=128, seed=0):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    mask = rng.choice(np.array([0.0, 0.5, 1.0], np.float32), size=T)
    return f(T, C), f(T, C), f(T, C), f(T, C), mask


@pytest.mark.parametrize("cfg_scale,rescale", [(3.0, 0.7), (3.0, 0.0), (1.0, 0.7), (4.5, 1.0)])
def test_cfg_euler_step_matches_oracle(ctx, cfg_scale, rescale):
    import ltx_b200
    cond, unc, lat, clean, mask = _cfg_case(seed=int(cfg_scale * 10 + rescale * 10))
    s0, s1 = 0.8125, 0.6
    x0 = sampler.cfg_combine(cond[None], unc[None], cfg_scale, rescale)
    x0a = sampler.post_process(x0, mask[None, :, None], clean[None])
    exp = sampler.euler_step(lat[None], x0a, s0, s1)[0]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    ld = dev(lat)
    ltx_b200.cfg_euler_step(ctx, dev(cond), dev(unc) if cfg_scale != 1.0 else None, ld, dev(clean), dev(mask), s0, s1,
                            cfg_scale, rescale)
    ctx.synchronize()
    got = ld.cpu().numpy()
    np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-5)
    assert rel_l2(got - lat, exp - lat) < 1e-5
    # tokens with mask 0 keep x0' = clean exactly
    m0 = mask == 0
    np.testing.assert_allclose(got[m0], lat[m0] + (lat[m0] - clean[m0]) / np.float32(s0) * np.float32(s1 - s0),
                               rtol=1e-6, atol=1e-6)


def test_cfg_euler_step_errors(ctx):
    import ltx_b200
    z = torch.zeros(8, 4, device="cuda")
    m = torch.ones(8, device="cuda")
    for (s0, s1, g, unc, kind) in ((0.0, 0.0, 1.0, z, "SIGMA"), (0.5, -1.0, 1.0, z, "SIGMA"),
                                   (float("nan"), 0.2, 1.0, z, "SIGMA"), (0.5, 0.2, 3.0, None, "NEGATIVE_CONTEXT")):
        with pytest.raises(ltx_b200.LtxError) as e:
            ltx_b200.cfg_euler_step(ctx, z, unc, z, z, m, s0, s1, g)
        assert e.value.kind == kind
    assert float(z.abs().sum()) == 0.0   # nothing ran
