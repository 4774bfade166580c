"""K1 parity on the GPU: ltx_dequant_merge against the bit-exact CPU oracle.

Bar: bit-exact (NaN compared as NaN) for every element, F32 and BF16 outputs.
Cases: the reference's FP8 and LoRA golden fixtures, the integration-test
known answers, ragged shapes, every base dtype, NaN / -0 bytes, stacked
deltas of mixed ranks and dtypes, and the full config-1 shape
(FP8 4096x4096 + rank-64 bf16 LoRA).
"""
import os

import numpy as np
import pytest
import torch

from oracle.weight_store import (DTYPE_CODE, KeyMap, LoraFile, LowRankDelta, WeightStore, decode_to_f32,
                                 f32_to_bf16_bits, read_raw)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ctx():
    import ltx_b200
    return ltx_b200.Context(0)


def to_dev(raw: bytes) -> torch.Tensor:
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda() if raw else torch.empty(1, dtype=torch.uint8, device="cuda")


def gpu_read(ctx, raw, dt, has_scale, scale, out, inn, deltas_np, want):
    """deltas_np: list of (a_raw, a_dt, b_raw, b_dt, rank, coeff)."""
    import ltx_b200
    w = to_dev(raw)
    keep = []
    ds = []
    for a_raw, a_dt, b_raw, b_dt, rank, coeff in deltas_np:
        a, b = to_dev(a_raw), to_dev(b_raw)
        keep += [a, b]
        ds.append((a.data_ptr(), b.data_ptr(), rank, DTYPE_CODE[a_dt], DTYPE_CODE[b_dt], coeff))
    if want == "f32":
        dst = torch.empty(out * inn, dtype=torch.float32, device="cuda")
        ctx.dequant_merge(w.data_ptr(), DTYPE_CODE[dt], has_scale, scale, out, inn, ds, dst.data_ptr(), ltx_b200.LTX_F32)
    else:
        dst = torch.empty(out * inn, dtype=torch.bfloat16, device="cuda")
        ctx.dequant_merge(w.data_ptr(), DTYPE_CODE[dt], has_scale, scale, out, inn, ds, dst.data_ptr(), ltx_b200.LTX_BF16)
    ctx.synchronize()
    if want == "f32":
        return dst.cpu().numpy()
    return dst.cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_read(raw, dt, has_scale, scale, out, inn, deltas_np, want):
    deltas = [LowRankDelta(np.ascontiguousarray(decode_to_f32(b_dt, b_raw).reshape(out, rank)),
                           np.ascontiguousarray(decode_to_f32(a_dt, a_raw).reshape(rank, inn)),
                           out, rank, inn, coeff) for a_raw, a_dt, b_raw, b_dt, rank, coeff in deltas_np]
    return read_raw(raw, dt, has_scale, scale, out, inn, deltas, want, n_threads=os.cpu_count() or 1)


def assert_bits_equal(got, exp, want):
    if want == "f32":
        gn, en = np.isnan(got), np.isnan(exp)
        assert (gn == en).all(), f"NaN mismatch at {np.argwhere(gn != en)[:5]}"
        g, e = got[~gn].view(np.uint32), exp[~en].view(np.uint32)
    else:
        gf = (got.astype(np.uint32) << 16).view(np.float32)
        ef = (exp.astype(np.uint32) << 16).view(np.float32)
        gn, en = np.isnan(gf), np.isnan(ef)
        assert (gn == en).all()
        g, e = got[~gn], exp[~en]
    bad = np.flatnonzero(g != e)
    assert bad.size == 0, f"{bad.size} mismatching elements, first {bad[:5]}: got {g[bad[:5]]} exp {e[bad[:5]]}"


def rand_raw(rng, dt, n, special=False):
    if dt in ("F8_E4M3", "F8_E5M2"):
        b = rng.integers(0, 256, n, dtype=np.uint8)
        if dt == "F8_E4M3" and not special:
            b[(b & 0x7F) == 0x7F] = 0x38
        if dt == "F8_E5M2" and not special:
            b[(b & 0x7C) == 0x7C] = 0x3C
        return b.tobytes()
    x = (rng.standard_normal(n) * 0.05).astype(np.float32)
    if dt == "F32":
        return x.tobytes()
    if dt == "BF16":
        return f32_to_bf16_bits(x).tobytes()
    return x.astype(np.float16).tobytes()


def test_fp8_fixture(ctx):
    st = WeightStore([os.path.join(GOLD, "fp8_e4m3fn_parity.safetensors")], KeyMap.identity())
    dt, shape, raw = st.entries["w"]
    hs, sc = st.scale_of("w")
    for want in ("f32", "bf16"):
        got = gpu_read(ctx, raw, dt, hs, sc, 4, 4, [], want)
        assert_bits_equal(got, oracle_read(raw, dt, hs, sc, 4, 4, [], want), want)
    exp = WeightStore([os.path.join(GOLD, "fp8_e4m3fn_expected.safetensors")], KeyMap.identity()).read("w").ravel()
    got = gpu_read(ctx, raw, dt, hs, sc, 4, 4, [], "f32")
    ok = ~np.isnan(exp)
    np.testing.assert_allclose(got[ok], exp[ok], atol=1e-5, rtol=0)   # the reference test's bar


def test_lora_fixture(ctx):
    st = WeightStore([os.path.join(GOLD, "lora_parity_base.safetensors")], KeyMap.identity())
    lora = LoraFile(os.path.join(GOLD, "lora_parity_lora.safetensors"))
    st.merge_lora(lora, 0.75)
    d = st.lora_deltas["layer.weight"][0]
    dt, shape, raw = st.entries["layer.weight"]
    _, _, a_raw = lora.tensors["layer.lora_A.weight"]
    _, _, b_raw = lora.tensors["layer.lora_B.weight"]
    dn = [(a_raw, "F32", b_raw, "F32", d.rank, d.scale)]
    for want in ("f32", "bf16"):
        got = gpu_read(ctx, raw, dt, False, 1.0, 8, 4, dn, want)
        assert_bits_equal(got, oracle_read(raw, dt, False, 1.0, 8, 4, dn, want), want)
    exp = WeightStore([os.path.join(GOLD, "lora_parity_expected.safetensors")], KeyMap.identity()).read("layer.weight")
    got = gpu_read(ctx, raw, dt, False, 1.0, 8, 4, dn, "f32")
    np.testing.assert_allclose(got, exp.ravel(), atol=5e-2)   # the reference test's bar


def test_integration_known_answers(ctx):
    f32b = lambda v: np.asarray(v, np.float32).tobytes()
    got = gpu_read(ctx, f32b([1, 0, 0, 1]), "F32", False, 1.0, 2, 2,
                   [(f32b([1, 2]), "F32", f32b([3, 4]), "F32", 1, 1.0)], "f32")
    np.testing.assert_array_equal(got, [4, 6, 4, 9])
    got = gpu_read(ctx, f32b([1, 0, 0, 1]), "F32", False, 1.0, 2, 2,
                   [(f32b([1, 2]), "F32", f32b([3, 4]), "F32", 1, 1.0),
                    (f32b([1, 0, 0, 1]), "F32", f32b([2, 0, 0, -2]), "F32", 2, 0.5)], "f32")
    np.testing.assert_array_equal(got, [5, 6, 4, 8])
    got = gpu_read(ctx, bytes([0x38]), "F8_E4M3", True, 3.0, 1, 1, [], "f32")
    assert got[0] == 3.0
    got = gpu_read(ctx, bytes([0x80, 0x00]), "F8_E4M3", True, 2.0, 1, 2, [], "f32")
    assert got.view(np.uint32).tolist() == [0, 0]   # fma(scale, -0, +0) = +0


CASES = [
    # (rows, cols, base dtype, has_scale, deltas [(rank, a_dt, b_dt)], special bytes)
    (1, 1, "F8_E4M3", True, [], True),
    (3, 5, "F8_E4M3", True, [(2, "BF16", "BF16")], True),
    (17, 33, "F8_E5M2", True, [(1, "F32", "F32")], True),
    (129, 257, "F8_E4M3", True, [(33, "BF16", "BF16")], True),
    (130, 520, "F8_E4M3", False, [(64, "BF16", "F16"), (3, "F32", "BF16")], False),
    (64, 4096, "BF16", False, [(64, "BF16", "BF16")], False),
    (300, 1000, "F16", False, [(100, "F32", "F32")], False),
    (257, 300, "F32", False, [(7, "F8_E4M3", "F8_E5M2")], False),
    (1000, 4096, "F8_E4M3", True, [], True),
    (4096, 17, "F8_E4M3", True, [], False),
]


@pytest.mark.parametrize("rows,cols,dt,has_scale,dspec,special", CASES)
def test_random_cases(ctx, rows, cols, dt, has_scale, dspec, special):
    rng = np.random.default_rng(rows * 131 + cols)
    raw = rand_raw(rng, dt, rows * cols, special)
    scale = float(np.float32(rng.random() * 0.01 + 1e-4))
    dn = []
    for rank, a_dt, b_dt in dspec:
        coeff = float(np.float32(rng.random() * 2))
        dn.append((rand_raw(rng, a_dt, rank * cols), a_dt, rand_raw(rng, b_dt, rows * rank), b_dt, rank, coeff))
    for want in ("f32", "bf16"):
        got = gpu_read(ctx, raw, dt, has_scale, scale, rows, cols, dn, want)
        assert_bits_equal(got, oracle_read(raw, dt, has_scale, scale, rows, cols, dn, want), want)


def make_config1(seed=0):
    """W ~ N(0,0.02) [4096,4096] quantised to e4m3 with scale
    amax/448; A [64,4096], B [4096,64] bf16 ~ N(0,0.01); alpha 64, strength 1."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(4096, 4096, generator=g) * 0.02
    scale = (w.abs().max() / 448.0).float()
    q = (w / scale).to(torch.float8_e4m3fn)
    a = (torch.randn(64, 4096, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(4096, 64, generator=g) * 0.01).to(torch.bfloat16)
    return q.view(torch.uint8).numpy().tobytes(), float(scale), a.view(torch.int16).numpy().tobytes(), \
        b.view(torch.int16).numpy().tobytes()


def test_config1_full_size_bit_exact(ctx):
    import ltx_b200
    raw, scale, a_raw, b_raw = make_config1()
    coeff = ltx_b200.lora_coeff(1.0, 64.0, 64)
    dn = [(a_raw, "BF16", b_raw, "BF16", 64, coeff)]
    got = gpu_read(ctx, raw, "F8_E4M3", True, scale, 4096, 4096, dn, "bf16")
    assert_bits_equal(got, oracle_read(raw, "F8_E4M3", True, scale, 4096, 4096, dn, "bf16"), "bf16")


def test_bad_arguments_are_errors(ctx):
    import ltx_b200
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")
    dst = torch.zeros(16, dtype=torch.float32, device="cuda")
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.dequant_merge(w.data_ptr(), 99, False, 1.0, 4, 4, [], dst.data_ptr(), ltx_b200.LTX_F32)
    assert e.value.kind == "DTYPE"
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.dequant_merge(w.data_ptr(), ltx_b200.LTX_F8_E4M3, False, 1.0, 4, 4, [], dst.data_ptr(), ltx_b200.LTX_F16)
    assert e.value.kind == "DTYPE"
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.dequant_merge(w.data_ptr(), ltx_b200.LTX_F8_E4M3, False, 1.0, 4, 4,
                          [(w.data_ptr(), w.data_ptr(), 0, 0, 0, 1.0)], dst.data_ptr(), ltx_b200.LTX_F32)
    assert e.value.kind == "SHAPE"
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.dequant_merge(0, ltx_b200.LTX_F8_E4M3, False, 1.0, 4, 4, [], dst.data_ptr(), ltx_b200.LTX_F32)
    assert e.value.kind == "INVALID_ARG"
