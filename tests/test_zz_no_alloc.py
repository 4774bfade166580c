"""The allocation-free merge entry point, for callers that cannot call cudaMalloc.

Some hosts own every device allocation (a memory pool, a framework's caching
allocator, a process that must not allocate after start-up); they can still
run the FP8 dequant + LoRA merge through ltx_dequant_merge_noalloc, which
keeps its chain scratch in a fixed file-scope device array instead of
allocating.  These tests call it through the C ABI and check that it gives
exactly what ltx_dequant_merge gives (bit-exact: both run the same kernels),
on calls in a row so that the shared scratch is reused: a config-1 merge, a
ragged f32 merge with two stacked deltas, a merge with no LoRA at all, and
the largest 22B DiT weight (the 24576 x 4096 adaLN projection with a rank-64
LoRA, 7.3 MB of its 16 MiB scratch).  They also check that the device's free
memory does not change across a call once the library is loaded, and that a
merge too large for the array is refused with a clear error.

Named test_zz_* so it is collected after every other test file; it creates
its own context and inputs, so it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, rows, cols, specs, w_dtype):
    """Random weight + deltas on the device.  specs: [(rank, dtype), ...]."""
    import ltx_b200
    g = torch.Generator().manual_seed(seed)
    if w_dtype == ltx_b200.LTX_F8_E4M3:
        w = (torch.randn(rows, cols, generator=g) * 0.02 / (0.02 * 4.5 / 448)).clamp(-440, 440)
        w = w.to(torch.float8_e4m3fn).view(torch.uint8).cuda()
    else:
        w = (torch.randn(rows, cols, generator=g) * 0.02).cuda()
    keep, deltas = [], []
    for rank, dt in specs:
        tdt = torch.bfloat16 if dt == ltx_b200.LTX_BF16 else torch.float32
        a = (torch.randn(rank, cols, generator=g) * 0.01).to(tdt).cuda()
        b = (torch.randn(rows, rank, generator=g) * 0.01).to(tdt).cuda()
        keep += [a, b]
        deltas.append((a.data_ptr(), b.data_ptr(), rank, dt, dt, ltx_b200.lora_coeff(0.8, float(rank) / 2, rank)))
    return w, keep, deltas


def _bits(t):
    return t.view(torch.int16 if t.dtype == torch.bfloat16 else torch.int32).cpu().numpy()


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    import ltx_b200
    ctx = ltx_b200.Context(0)
    stream = torch.cuda.current_stream().cuda_stream
    cases = [
        # config 1: FP8 4096x4096 with a rank-64 bf16 LoRA, bf16 out
        (0, 4096, 4096, [(64, ltx_b200.LTX_BF16)], ltx_b200.LTX_F8_E4M3, ltx_b200.LTX_BF16),
        # a second, different call: ragged f32 weight, two stacked deltas, f32 out
        (1, 1000, 777, [(33, ltx_b200.LTX_F32), (7, ltx_b200.LTX_BF16)], ltx_b200.LTX_F32, ltx_b200.LTX_F32),
        # no LoRA: the dequant-only kernel, no scratch
        (2, 512, 4096, [], ltx_b200.LTX_F8_E4M3, ltx_b200.LTX_BF16),
        # the largest 22B DiT weight with a rank-64 LoRA: close to the scratch limit
        (3, 24576, 4096, [(64, ltx_b200.LTX_BF16)], ltx_b200.LTX_F8_E4M3, ltx_b200.LTX_BF16),
    ]
    free_after = []
    for seed, rows, cols, specs, wdt, odt in cases:
        w, keep, deltas = _case(seed, rows, cols, specs, wdt)
        tdt = torch.bfloat16 if odt == ltx_b200.LTX_BF16 else torch.float32
        ref = torch.empty(rows * cols, dtype=tdt, device="cuda")
        got = torch.full((rows * cols,), float("nan"), dtype=tdt, device="cuda")
        ctx.dequant_merge(w.data_ptr(), wdt, True, 0.02 * 4.5 / 448, rows, cols, deltas, ref.data_ptr(), odt)
        ctx.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        ltx_b200.dequant_merge_noalloc(stream, w.data_ptr(), wdt, True, 0.02 * 4.5 / 448, rows, cols, deltas,
                                       got.data_ptr(), odt)
        ctx.synchronize()
        free_after.append((free_before, torch.cuda.mem_get_info()[0]))
        assert np.array_equal(_bits(got), _bits(ref)), f"case {seed}: outputs differ"
        del w, keep, ref, got
    ctx.close()
    # The first call on a device may load the library's device code (and its
    # scratch array) lazily; every call after it leaves free memory unchanged.
    for i, (before, after) in enumerate(free_after[1:], 1):
        assert before == after, f"call {i}: device free memory changed by {before - after} bytes"


def test_noalloc_rejects_merges_beyond_its_scratch():
    import ltx_b200
    # 4 * 64 * (16384 + 65536) bytes of chain scratch > 16 MiB: refused before anything is enqueued,
    # so small placeholder buffers are enough.
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    d = [(buf.data_ptr(), buf.data_ptr(), 64, ltx_b200.LTX_BF16, ltx_b200.LTX_BF16, 1.0)]
    with pytest.raises(ltx_b200.LtxError) as e:
        ltx_b200.dequant_merge_noalloc(torch.cuda.current_stream().cuda_stream, buf.data_ptr(), ltx_b200.LTX_F8_E4M3,
                                       True, 1.0, 65536, 16384, d, buf.data_ptr(), ltx_b200.LTX_BF16)
    assert e.value.kind == "UNSUPPORTED" and "scratch" in str(e.value)
