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


def _e4m3(x, per_row):
    """Quantise to e4m3 with scale amax/448 (per row or per tensor): (uint8 bits, scale, dequantised f32)."""
    amax = x.abs().amax(dim=1, keepdim=True) if per_row else x.abs().max()
    s = (amax / 448.0).clamp_min(1e-30)
    q = (x / s).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), s.reshape(-1).float(), q.float() * s


@pytest.mark.parametrize("M,N,K,epi", [(128, 256, 128, 0), (300, 1000, 272, 0), (256, 512, 4096, 1),
                                       (1000, 128, 4096, 2), (2048, 4096, 16384, 3), (77, 8, 48, 2)])
def test_gemm_e4m3_against_dequantised_fp32(ctx, M, N, K, epi):
    """Native FP8: e4m3 A (per-row scale) and W (per-tensor scale).  The reference is the
    fp32 product of the dequantised operands, so the only differences are the f32
    accumulation order and the output rounding."""
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    a32 = torch.randn(M, K, device="cuda", generator=g) * (1 + torch.rand(M, 1, device="cuda", generator=g) * 4)
    w32 = torch.randn(N, K, device="cuda", generator=g) * 0.02
    aq, a_s, a_deq = _e4m3(a32, True)
    wq, w_s, w_deq = _e4m3(w32, False)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    ref = a_deq @ w_deq.t() + bias
    if epi == ltx_b200.EPI_GELU_BF16:
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    if epi in (ltx_b200.EPI_BF16, ltx_b200.EPI_GELU_BF16):
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    else:
        out = torch.zeros(M, N, device="cuda")
    gate = torch.rand(2, N, device="cuda", generator=g) if epi == ltx_b200.EPI_RESID else None
    gidx = (torch.arange(M, device="cuda", dtype=torch.int32) % 2) if gate is not None else None
    ltx_b200.gemm_e4m3(ctx, aq, a_s, wq, float(w_s), out, epi, bias, gate, gidx)
    ctx.synchronize()
    if gate is not None:
        ref = ref * gate[gidx.long()]
    assert rel_l2(out.float(), ref) < 1e-2


def test_gemm_e4m3_throughput(ctx):
    """FFN-in shape of the step (informational): e4m3 vs bf16 on the same shape."""
    import ltx_b200
    M, N, K = 24576, 16384, 4096
    a = torch.randint(0, 120, (M, K), device="cuda", dtype=torch.uint8)
    w = torch.randint(0, 120, (N, K), device="cuda", dtype=torch.uint8)
    sa = torch.full((M,), 0.01, device="cuda")
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        ltx_b200.gemm_e4m3(ctx, a, sa, w, 0.01, out, ltx_b200.EPI_GELU_BF16)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(5):
        ltx_b200.gemm_e4m3(ctx, a, sa, w, 0.01, out, ltx_b200.EPI_GELU_BF16)
    e.record()
    ctx.synchronize()
    ms = s.elapsed_time(e) / 5
    print(f"\ne4m3 GEMM {M}x{N}x{K} + GELU: {ms:.3f} ms = {2 * M * N * K / ms / 1e9:.0f} TFLOP/s")


@pytest.mark.parametrize("M,N,K,k2,epi", [(256, 512, 4096, 64, 0), (300, 384, 512, 128, 2), (1000, 4096, 4096, 64, 3)])
def test_gemm_e4m3_lowrank_and_column_scales(ctx, M, N, K, k2, epi):
    """Exact FP8 base + unmerged LoRA in one accumulator: out = x.(W*s_col + coeff B A)^T with
    x = xq * sx[row]; the low-rank block gets A2 = (x A^T)/sx and B2 = coeff B / s_col."""
    import ltx_b200
    g = torch.Generator(device="cuda").manual_seed(M + K + k2)
    x32 = torch.randn(M, K, device="cuda", generator=g)
    xq, sx, x_deq = _e4m3(x32, True)
    w32 = torch.randn(N, K, device="cuda", generator=g) * 0.02
    wq8 = w32.to(torch.float8_e4m3fn)
    s_col = (torch.rand(N, device="cuda", generator=g) + 0.5) * 0.01      # per-column (e.g. Q|K|V) scales
    w_deq = wq8.float() * s_col[:, None]
    A = (torch.randn(k2, K, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    B = (torch.randn(N, k2, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    coeff = 0.8
    a2 = ((x_deq @ A.float().t()) / sx[:, None]).to(torch.bfloat16)
    b2 = (coeff * B.float() / s_col[:, None]).to(torch.bfloat16)
    out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16 if epi == 0 else torch.float32)
    ltx_b200.gemm_e4m3(ctx, xq, sx, wq8.view(torch.uint8), 1.0, out, epi, None, None, None,
                       w_col_scale=s_col, a2=a2, b2=b2)
    ctx.synchronize()
    ref = x_deq @ (w_deq + coeff * B.float() @ A.float()).t()
    assert rel_l2(out.float(), ref) < 1e-2
    if epi == ltx_b200.EPI_BF16:
        return   # bf16 output rounding is larger than the low-rank term's share; f32 cases check it below
    # without the appended block the low-rank term is missing: the check above is not vacuous
    out0 = torch.zeros_like(out)
    ltx_b200.gemm_e4m3(ctx, xq, sx, wq8.view(torch.uint8), 1.0, out0, epi, None, None, None, w_col_scale=s_col)
    ctx.synchronize()
    lr = x_deq @ (coeff * B.float() @ A.float()).t()
    assert rel_l2(out.float() - out0.float(), lr) < 2e-2
