"""Device patchify / unpatchify (ltx_patchify, ltx_unpatchify) against the
oracle's restatement of patchifier.rs:50-89 (patch size 1):

    [B, C, F, H, W]  <->  [B, F*H*W, C],   token t = f*H*W + h*W + w

Bit-exact (a permutation moves f32 values unchanged), at the config-4 latent
shape [1, 128, 16, 24, 16], a ragged shape, batch 2 and an empty latent; the
round trip returns the input unchanged.
"""
import numpy as np
import pytest
import torch

from oracle import sampler

pytestmark = pytest.mark.gpu

SHAPES = [(1, 128, 16, 24, 16),   # config 4 target latent
          (1, 7, 3, 5, 9),        # ragged: nothing a multiple of anything
          (2, 128, 4, 6, 10),     # batch 2
          (2, 3, 1, 1, 1),
          (1, 16, 0, 4, 4)]       # no frames: nothing to move


@pytest.fixture(scope="module")
def ctx():
    import ltx_b200
    c = ltx_b200.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("shape", SHAPES)
def test_patchify_bit_exact_and_round_trip(ctx, shape):
    import ltx_b200
    B, C, F, H, W = shape
    rng = np.random.default_rng(sum(shape))
    lat = rng.standard_normal(shape).astype(np.float32)
    # a few special values travel bit for bit too
    flat = lat.reshape(-1)
    flat[: min(4, flat.size)] = np.array([-0.0, np.inf, -np.inf, 1e-40], np.float32)[: min(4, flat.size)]
    exp = sampler.patchify(lat)
    lat_d = torch.from_numpy(lat).cuda()
    tok_d = torch.full((B, F * H * W, C), float("nan"), device="cuda")
    ltx_b200.patchify(ctx, lat_d, tok_d)
    back = torch.full(shape, float("nan"), device="cuda")
    ltx_b200.unpatchify(ctx, tok_d, back)
    ctx.synchronize()
    got = tok_d.cpu().numpy()
    assert got.shape == exp.shape
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    assert np.array_equal(back.cpu().numpy().view(np.uint32), lat.view(np.uint32))
    # unpatchify is the oracle's inverse as well
    assert np.array_equal(sampler.unpatchify(exp, F, H, W).view(np.uint32), lat.view(np.uint32))


def test_patchify_token_order(ctx):
    """Token t = f*H*W + h*W + w holds channel c at column c (patchifier.rs:50-60)."""
    import ltx_b200
    B, C, F, H, W = 1, 4, 2, 3, 5
    idx = np.arange(B * C * F * H * W, dtype=np.float32).reshape(B, C, F, H, W)
    tok = torch.empty(B, F * H * W, C, device="cuda")
    ltx_b200.patchify(ctx, torch.from_numpy(idx).cuda(), tok)
    ctx.synchronize()
    got = tok.cpu().numpy()
    for f in range(F):
        for h in range(H):
            for w in range(W):
                t = f * H * W + h * W + w
                for c in range(C):
                    assert got[0, t, c] == idx[0, c, f, h, w]


def test_patchify_rejects_bad_arguments(ctx):
    import ltx_b200
    z = torch.zeros(8, device="cuda")
    for args in ((1, 2, -1, 2, 2, z.data_ptr()), (1, 2, 1, 2, 2, None)):   # negative extent; null output
        with pytest.raises(ltx_b200.LtxError) as e:
            ctx.check(ltx_b200.lib().ltx_patchify(ctx.h, z.data_ptr(), *args), "ltx_patchify")
        assert e.value.kind == "INVALID_ARG"
