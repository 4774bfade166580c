"""Configs 3 and 4 at their full width: one 22B-class block (D 4096, 32 x 128
heads, FFN 16384) on T = 12288 tokens (16x24x16 target + the same-size IC
reference) with 1024 context tokens, loaded from an FP8 + LoRA checkpoint,
against the oracle (torch f32, the checkpoint read by the C restatement of the
weight store) on the same inputs:

  * the block forward (config 3);
  * one guided Euler step (config 4 with L = 1 so that the oracle fits in a
    test): CFG batch 2 (cond / uncond contexts), guidance 3.0, rescale 0.7,
    the global-std rescale over all 12288 x 128 values (guidance.rs:149-195),
    post_process and the Euler update (loop_.rs:37-65).

Bar: rel-L2 <= 1e-2 (the north star's bf16 bar), on the step's new latent and
on its update.  The oracle runs on the host cores (about 10-40 s each)."""
import os

import numpy as np
import pytest
import torch

from oracle import dit, sampler
from oracle.weight_store import KeyMap, LoraFile, WeightStore as OracleStore

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def full_ckpt(tmp_path_factory):
    """A one-block checkpoint at the 22B width (FP8 e4m3 + scales) and a rank-64 bf16 LoRA."""
    from dit_checkpoint import small_config, write_checkpoint, write_lora
    d = tmp_path_factory.mktemp("full")
    cfg = small_config(heads=32, head_dim=128, layers=1)
    ck, lo = str(d / "block.safetensors"), str(d / "lora.safetensors")
    write_checkpoint(ck, cfg, seed=21)
    write_lora(lo, cfg, rank=64, alpha=64.0, seed=22)
    return cfg, ck, lo


def _oracle_params(ck, lo):
    o = OracleStore([ck], KeyMap.transformer())
    o.merge_lora(LoraFile(lo), 1.0)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return dit.load_params({k: o.read(k, n_threads=threads) for k in o.keys()})


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_config3_block_full_size_matches_oracle(full_ckpt):
    import ltx_b200
    cfg, ck, lo = full_ckpt
    F, Hh, W, S = 16, 24, 16, 1024
    Tt = F * Hh * W
    rng = np.random.default_rng(23)
    lat = rng.standard_normal((1, 2 * Tt, 128)).astype(np.float32)
    ts = np.concatenate([np.full(Tt, 0.7, np.float32), np.zeros(Tt, np.float32)])[None]
    pos = np.concatenate([sampler.target_positions(F, Hh, W), sampler.reference_positions(F, Hh, W)], axis=2)
    ctxt = rng.standard_normal((1, S, cfg["cross_attention_dim"])).astype(np.float32)

    ctx = ltx_b200.Context(0)
    st = ltx_b200.WeightStore(ctx, [ck], ltx_b200.KEYMAP_TRANSFORMER)
    st.merge_lora(lo, 1.0)
    model = ltx_b200.VideoTransformer.load(ctx, st)
    out = torch.empty(lat.shape, dtype=torch.float32, device="cuda")
    model.forward(*(torch.from_numpy(a).cuda() for a in (lat, ts, pos, ctxt)), out)
    ctx.synchronize()
    got = out.cpu().numpy()
    model.close()
    st.close()
    ctx.close()

    params = _oracle_params(ck, lo)
    old_chunk = dit.SDPA_Q_CHUNK
    dit.SDPA_Q_CHUNK = 256
    try:
        with torch.no_grad():
            exp = dit.model_forward(params, dit.DiTConfig.from_json(cfg),
                                    *(torch.from_numpy(a) for a in (lat, ts, pos, ctxt))).numpy()
    finally:
        dit.SDPA_Q_CHUNK = old_chunk
    err = float(np.linalg.norm(got - exp) / np.linalg.norm(exp))
    print(f"\nconfig 3 full size (T={2 * Tt}, S={S}): rel-L2 {err:.2e}")
    assert np.isfinite(got).all() and err < 1e-2


def test_config4_step_full_width_matches_oracle(full_ckpt):
    """ltx_denoise_step at the config-4 width and token count (L = 1) against
    oracle/sampler.euler_loop over oracle/dit.model_forward: same checkpoint,
    same latent / IC reference / contexts / sigmas."""
    import ltx_b200
    cfg, ck, lo = full_ckpt
    F, Hh, W, S = 16, 24, 16, 1024
    C, Tt = cfg["in_channels"], F * Hh * W
    rng = np.random.default_rng(31)
    init = sampler.LatentState(rng.standard_normal((1, Tt, C)).astype(np.float32), np.ones((1, Tt, 1), np.float32),
                               sampler.target_positions(F, Hh, W), np.zeros((1, Tt, C), np.float32))
    ref = rng.standard_normal((1, C, F, Hh, W)).astype(np.float32)
    state = sampler.apply_reference(init, ref, strength=1.0)          # T = 12288, mask 0 on the reference
    cc = rng.standard_normal((1, S, cfg["cross_attention_dim"])).astype(np.float32)
    cu = rng.standard_normal((1, S, cfg["cross_attention_dim"])).astype(np.float32)
    sig = sampler.scheduler_execute(8, Tt)
    s0, s1 = float(sig[1]), float(sig[2])

    ctx = ltx_b200.Context(0)
    st = ltx_b200.WeightStore(ctx, [ck], ltx_b200.KEYMAP_TRANSFORMER)
    st.merge_lora(lo, 1.0)
    model = ltx_b200.VideoTransformer.load(ctx, st)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    lat = dev(state.latent[0])
    model.denoise_step(lat, dev(state.clean_latent[0]), dev(state.denoise_mask[0, :, 0]), dev(state.positions),
                       dev(cc[0]), dev(cu[0]), s0, s1, 3.0, 0.7)
    ctx.synchronize()
    got = lat.cpu().numpy()
    model.close()
    st.close()
    ctx.close()

    params = _oracle_params(ck, lo)
    c = dit.DiTConfig.from_json(cfg)
    old_chunk = dit.SDPA_Q_CHUNK
    dit.SDPA_Q_CHUNK = 256

    def model_x0(latent, ts, pos, ctx_):
        with torch.no_grad():
            v = dit.model_forward(params, c, torch.from_numpy(latent), torch.from_numpy(ts), torch.from_numpy(pos),
                                  torch.from_numpy(ctx_)).numpy()
        return sampler.velocity_to_x0(latent, ts, v)

    try:
        exp = sampler.euler_loop([s0, s1], state, state.latent.shape[1], model_x0, cc, cu, cfg_scale=3.0,
                                 rescale_scale=0.7).latent[0]
    finally:
        dit.SDPA_Q_CHUNK = old_chunk
    err = rel_l2(got, exp)
    d_err = rel_l2(got - state.latent[0], exp - state.latent[0])
    print(f"\nconfig 4 step, full width (T={2 * Tt}, S={S}, L=1): latent rel-L2 {err:.2e}, update rel-L2 {d_err:.2e}")
    assert np.isfinite(got).all() and err < 1e-2 and d_err < 1e-2
    # the IC-reference tokens (mask 0) keep x0' = clean exactly
    x, cl = state.latent[0, Tt:], state.clean_latent[0, Tt:]
    np.testing.assert_allclose(got[Tt:], x + (x - cl) / np.float32(s0) * np.float32(s1 - s0), rtol=1e-5, atol=1e-5)
