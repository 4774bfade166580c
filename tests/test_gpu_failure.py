"""Failure detection on the GPU without faulting it: a bounded device-side
wait on a flag that nothing sets gives up after its limit, the context
reports LTX_ERR_TIMEOUT, and the same context keeps working afterwards."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_on_unset_flag_times_out_and_context_survives():
    import ltx_b200
    ctx = ltx_b200.Context(0)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    ctx.wait_flag(flag, 1, timeout_ms=300)
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.synchronize()
    waited = time.time() - t0
    assert e.value.kind == "TIMEOUT"
    assert 0.25 < waited < 10, waited
    # the flag is cleared by the report, and the context still computes correctly
    ctx.synchronize()
    a = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    w = torch.randn(384, 512, device="cuda").to(torch.bfloat16)
    o = torch.empty(256, 384, device="cuda", dtype=torch.bfloat16)
    ltx_b200.gemm(ctx, a, w, o)
    ctx.synchronize()
    ref = a.float() @ w.float().t()
    assert float((o.float() - ref).norm() / ref.norm()) < 1e-2
    ctx.close()


def test_flag_set_earlier_on_the_stream_releases_the_wait():
    import ltx_b200
    ctx = ltx_b200.Context(0)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.set_flag(flag, 7)
    ctx.wait_flag(flag, 7, timeout_ms=2000)
    t0 = time.time()
    ctx.synchronize()
    assert time.time() - t0 < 1.0
    assert int(flag.item()) == 7
    ctx.close()


def test_wait_flag_rejects_bad_pointers():
    import ltx_b200
    ctx = ltx_b200.Context(0)
    buf = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(ltx_b200.LtxError) as e:
        ctx.wait_flag(buf.data_ptr() + 2, 0)
    assert e.value.kind == "INVALID_ARG"
    ctx.close()
