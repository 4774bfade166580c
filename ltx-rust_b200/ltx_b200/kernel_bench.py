"""Times one library kernel at a chosen shape (CUDA events, after warm-up).

    python ltx-rust_b200/ltx_b200/kernel_bench.py attention --B 1 --H 8 --T 4096 [--Tk N] [--iters 3]
    python ltx-rust_b200/ltx_b200/kernel_bench.py gemm --M 4096 --N 4096 --K 4096 [--epi 0..3] [--fp8]
    python ltx-rust_b200/ltx_b200/kernel_bench.py merge --rows 4096 --cols 4096 --rank 64 [--sets 8]

Used for small, self-contained profiler captures of a single kernel and for
quick shape sweeps; prints one line per run.
"""
import argparse
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _time(fn, iters):
    import torch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main():
    import torch
    import ltx_b200
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["attention", "gemm", "merge"])
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--H", type=int, default=8)
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--Tk", type=int, default=0)
    ap.add_argument("--M", type=int, default=4096)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--epi", type=int, default=0)
    ap.add_argument("--fp8", action="store_true", help="gemm: e4m3 operands (native FP8)")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--rank", type=int, default=64)
    ap.add_argument("--sets", type=int, default=1, help="merge: distinct weight sets used in turn")
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    ctx = ltx_b200.Context(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.kernel == "attention":
        Tk = a.Tk or a.T
        q = torch.randn(a.B * a.T, a.H * 128, device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn(a.B * Tk, a.H * 128, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(a.B * Tk, a.H * 128, device="cuda", generator=g).to(torch.float16)
        o = torch.empty_like(q)
        fn = lambda: ltx_b200.attention(ctx, q, k, v, o, a.B, a.H, a.T, Tk, 1 / math.sqrt(128))
        flops = 4.0 * a.B * a.H * a.T * Tk * 128
        unit = "TFLOP/s"
    elif a.kernel == "gemm":
        if a.epi in (2, 3):
            o = torch.zeros(a.M, a.N, device="cuda")
        else:
            o = torch.empty(a.M, a.N, device="cuda", dtype=torch.bfloat16)
        if a.fp8:
            x = torch.randn(a.M, a.K, device="cuda", generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
            w = torch.randn(a.N, a.K, device="cuda", generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
            sa = torch.full((a.M,), 0.05, device="cuda")
            fn = lambda: ltx_b200.gemm_e4m3(ctx, x, sa, w, 0.02, o, a.epi)
        else:
            x = torch.randn(a.M, a.K, device="cuda", generator=g).to(torch.bfloat16)
            w = (torch.randn(a.N, a.K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
            fn = lambda: ltx_b200.gemm(ctx, x, w, o, a.epi)
        flops = 2.0 * a.M * a.N * a.K
        unit = "TFLOP/s"
    else:
        # --sets distinct weight/output pairs merged in turn (more than L2 together: no reuse between
        # launches); --rank 0 = no LoRA (the dequant-only kernel)
        wqs = [torch.randint(0, 126, (a.rows * a.cols,), dtype=torch.uint8, device="cuda") for _ in range(a.sets)]
        A = (torch.randn(max(a.rank, 1), a.cols, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        B = (torch.randn(a.rows, max(a.rank, 1), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        os_ = [torch.empty(a.rows * a.cols, device="cuda", dtype=torch.bfloat16) for _ in range(a.sets)]
        d = [(A.data_ptr(), B.data_ptr(), a.rank, ltx_b200.LTX_BF16, ltx_b200.LTX_BF16, 1.0)] if a.rank else []
        turn = [0]

        def fn():
            i = turn[0] % a.sets
            turn[0] += 1
            ctx.dequant_merge(wqs[i].data_ptr(), ltx_b200.LTX_F8_E4M3, True, 0.01, a.rows, a.cols, d,
                              os_[i].data_ptr(), ltx_b200.LTX_BF16)
        flops = a.rows * a.cols * (1 + 2) + 2 * a.rank * (a.rows + a.cols)   # algorithmic bytes
        unit = "GB/s"
    for _ in range(a.warmup):
        fn()
    ctx.synchronize()
    ms = _time(fn, a.iters)
    ctx.synchronize()
    rate = flops / ms / (1e6 if unit == "GB/s" else 1e9)
    print(f"{a.kernel}: {ms:.4f} ms  {rate:.1f} {unit}")


if __name__ == "__main__":
    main()
