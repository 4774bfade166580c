"""Config 3 at its full size: one 22B-class block (D 4096, 32 x 128 heads, FFN
16384) on T = 12288 tokens (16x24x16 target + the same-size IC reference) with
1024 context tokens, loaded from an FP8 + LoRA checkpoint, against the oracle
(torch f32, the checkpoint read by the C restatement of the weight store) on
the same inputs.  Bar: rel-L2 <= 1e-2 (the north star's bf16 bar).  The oracle
runs on the host cores (about 10-20 s)."""
import os

import numpy as np
import pytest
import torch

from oracle import dit, sampler
from oracle.weight_store import KeyMap, LoraFile, WeightStore as OracleStore

pytestmark = pytest.mark.gpu


def test_config3_block_full_size_matches_oracle(tmp_path):
    import ltx_b200
    from dit_checkpoint import small_config, write_checkpoint, write_lora
    cfg = small_config(heads=32, head_dim=128, layers=1)
    ck, lo = str(tmp_path / "block.safetensors"), str(tmp_path / "lora.safetensors")
    write_checkpoint(ck, cfg, seed=21)
    write_lora(lo, cfg, rank=64, alpha=64.0, seed=22)
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

    o = OracleStore([ck], KeyMap.transformer())
    o.merge_lora(LoraFile(lo), 1.0)
    threads = os.cpu_count() or 1
    params = dit.load_params({k: o.read(k, n_threads=threads) for k in o.keys()})
    torch.set_num_threads(threads)
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
