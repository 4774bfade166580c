"""K3 flash attention against a torch fp32 reference of softmax(q k^T * s) v.

Tolerance rel-L2 <= 1e-2 (the north star's bf16 bar); the kernel's only
departures from fp32 are bf16 P and bf16 output.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import ltx_b200
    return ltx_b200.Context(0)


def ref_attention(q, k, v, B, H, Tq, Tk, scale, rows=None):
    """fp32 reference; q/k/v token-major [B*T, H*128]."""
    qf = q.float().view(B, Tq, H, 128).transpose(1, 2)
    kf = k.float().view(B, Tk, H, 128).transpose(1, 2)
    vf = v.float().view(B, Tk, H, 128).transpose(1, 2)
    if rows is not None:
        qf = qf[:, :, rows]
    s = (qf @ kf.transpose(2, 3)) * scale
    o = torch.softmax(s, -1) @ vf
    return o.transpose(1, 2).reshape(B, -1, H * 128)


def rel_l2(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


@pytest.mark.parametrize("vdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,Tq,Tk", [(1, 1, 128, 128), (2, 2, 256, 384), (2, 3, 200, 300), (1, 2, 1, 5),
                                       (2, 4, 1024, 77), (1, 2, 384, 1024), (2, 1, 130, 129)])
def test_attention_small(ctx, B, H, Tq, Tk, vdt):
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + H * 100 + Tq + Tk)
    q = torch.randn(B * Tq, H * 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B * Tk, H * 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B * Tk, H * 128, device="cuda", generator=g).to(vdt)
    out = torch.zeros(B * Tq, H * 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    ltx_b200.attention(ctx, q, k, v, out, B, H, Tq, Tk, scale)
    ctx.synchronize()
    ref = ref_attention(q, k, v, B, H, Tq, Tk, scale).reshape(B * Tq, H * 128)
    assert rel_l2(out.float(), ref) < 1e-2


def test_attention_strided_qkv(ctx):
    """q/k/v as column slices of one fused [T, 3*H*128] projection (the QKV GEMM output)."""
    import ltx_b200
    B, H, T = 2, 2, 320
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(B * T, 3 * H * 128, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = qkv[:, :H * 128], qkv[:, H * 128:2 * H * 128], qkv[:, 2 * H * 128:]
    out = torch.zeros(B * T, H * 128, device="cuda", dtype=torch.bfloat16)
    ltx_b200.attention(ctx, q, k, v, out, B, H, T, T, 0.0884)
    ctx.synchronize()
    ref = ref_attention(q.contiguous(), k.contiguous(), v.contiguous(), B, H, T, T, 0.0884).reshape(B * T, H * 128)
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("Tq,Tk", [(512, 1024), (300, 777)])
def test_attention_row_max_grows_unevenly(ctx, Tq, Tk):
    """Logits whose row maxima grow along the keys at different rates per query
    row: the lazy O rescale then triggers for some rows of a warp and not for
    others, which a warp-collective TMEM access must handle (deep DiT layers
    produce such logits; N(0,1) inputs almost never do)."""
    import ltx_b200
    B, H = 1, 2
    g = torch.Generator(device="cuda").manual_seed(Tq + Tk)
    row_gain = 1.0 + 10.0 * (torch.rand(B * Tq, 1, device="cuda", generator=g) > 0.5).float()
    key_gain = 0.2 + 3.0 * torch.arange(B * Tk, device="cuda").float().view(-1, 1) / (B * Tk)
    q = (torch.randn(B * Tq, H * 128, device="cuda", generator=g) * row_gain).to(torch.bfloat16)
    k = (torch.randn(B * Tk, H * 128, device="cuda", generator=g) * key_gain).to(torch.bfloat16)
    v = torch.randn(B * Tk, H * 128, device="cuda", generator=g).to(torch.float16)
    out = torch.zeros(B * Tq, H * 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    ltx_b200.attention(ctx, q, k, v, out, B, H, Tq, Tk, scale)
    ctx.synchronize()
    ref = ref_attention(q, k, v, B, H, Tq, Tk, scale).reshape(B * Tq, H * 128)
    assert rel_l2(out.float(), ref) < 1e-2


def test_attention_full_size(ctx):
    """The config-3/4 self-attention shape: B=2 (CFG), H=32, T=12288; checked on sampled rows."""
    import ltx_b200
    B, H, T = 2, 32, 12288
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(B * T, H * 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B * T, H * 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B * T, H * 128, device="cuda", generator=g).to(torch.float16)
    out = torch.zeros(B * T, H * 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    ltx_b200.attention(ctx, q, k, v, out, B, H, T, T, scale)
    ctx.synchronize()
    rows = torch.cat([torch.arange(0, 256), torch.arange(6000, 6128), torch.arange(T - 128, T)]).cuda()
    ref = ref_attention(q, k, v, B, H, T, T, scale, rows=rows)
    got = out.view(B, T, H * 128)[:, rows]
    assert rel_l2(got.float(), ref) < 1e-2
    # timing (informational, not a bench value)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(3):
        ltx_b200.attention(ctx, q, k, v, out, B, H, T, T, scale)
    e.record()
    ctx.synchronize()
    ms = s.elapsed_time(e) / 3
    flops = 4.0 * B * H * T * T * 128
    qt, kt, vt = (x.view(B, T, H, 128).transpose(1, 2) for x in (q, k, v.to(torch.bfloat16)))
    torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
    s.record()
    for _ in range(3):
        torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
    e.record()
    torch.cuda.synchronize()
    ref_ms = s.elapsed_time(e) / 3
    print(f"\nattention B={B} H={H} T={T}: {ms:.2f} ms = {flops / ms / 1e9:.0f} TFLOP/s; "
          f"torch SDPA {ref_ms:.2f} ms = {flops / ref_ms / 1e9:.0f} TFLOP/s")
