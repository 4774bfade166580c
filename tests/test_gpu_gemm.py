"""K2 tcgen05 GEMM against a torch fp32 reference of the same op (bf16 inputs).

Tolerance: the kernel accumulates in f32 like the reference; the only
rounding the reference does not do is the bf16 output (2^-9 relative), so
rel-L2 <= 1e-2 (the bf16 bar the north star states) is loose by ~10x.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import ltx_b200
    return ltx_b200.Context(0)


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


SHAPES = [(128, 256, 64), (256, 512, 4096), (200, 300, 136), (1, 8, 8), (12, 32, 8), (12, 192, 32),
          (1000, 128, 256), (4096, 4096, 4096), (384, 16384, 4096), (2048, 4096, 16384), (24576, 128, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bias_bf16(ctx, M, N, K):
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ltx_b200.gemm(ctx, a, w, out, ltx_b200.EPI_BF16, bias)
    ctx.synchronize()
    ref = a.float() @ w.float().t() + bias
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 4096), (300, 1000, 264), (2048, 16384, 4096)])
def test_gemm_gelu(ctx, M, N, K):
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ltx_b200.gemm(ctx, a, w, out, ltx_b200.EPI_GELU_BF16, None)
    ctx.synchronize()
    ref = torch.nn.functional.gelu(a.float() @ w.float().t(), approximate="tanh")
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (24576, 128, 4096), (77, 8, 32)])
def test_gemm_f32(ctx, M, N, K):
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    ltx_b200.gemm(ctx, a, w, out, ltx_b200.EPI_F32, bias)
    ctx.synchronize()
    ref = a.float() @ w.float().t() + bias
    assert rel_l2(out, ref) < 1e-4


@pytest.mark.parametrize("M,N,K,gated", [(512, 4096, 4096, True), (300, 520, 128, True), (512, 4096, 16384, False)])
def test_gemm_resid_gate(ctx, M, N, K, gated):
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g)
    x = torch.randn(M, N, device="cuda", generator=g)
    gate = torch.randn(2, N, device="cuda", generator=g) if gated else None
    gidx = (torch.arange(M, device="cuda") % 2).to(torch.int32) if gated else None
    ref = x + (a.float() @ w.float().t() + bias) * (gate[gidx.long()] if gated else 1.0)
    ltx_b200.gemm(ctx, a, w, x, ltx_b200.EPI_RESID, bias, gate, gidx)
    ctx.synchronize()
    assert rel_l2(x, ref) < 1e-4


def test_gemm_throughput_report(ctx):
    """Prints the achieved TFLOP/s at the FFN-in shape of one CFG pass (not a bench value)."""
    import ltx_b200
    M, N, K = 24576, 16384, 4096
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") / 64).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ltx_b200.gemm(ctx, a, w, out, ltx_b200.EPI_GELU_BF16)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(10):
        ltx_b200.gemm(ctx, a, w, out, ltx_b200.EPI_GELU_BF16)
    e.record()
    ctx.synchronize()
    ms = s.elapsed_time(e) / 10
    ref_ms = None
    b = w.t()
    torch.matmul(a, b)
    s.record()
    for _ in range(10):
        torch.matmul(a, b)
    e.record()
    torch.cuda.synchronize()
    ref_ms = s.elapsed_time(e) / 10
    print(f"\nGEMM {M}x{N}x{K}: {ms:.3f} ms = {2 * M * N * K / ms / 1e9:.1f} TFLOP/s; "
          f"torch/cuBLAS {ref_ms:.3f} ms = {2 * M * N * K / ref_ms / 1e9:.1f} TFLOP/s")
