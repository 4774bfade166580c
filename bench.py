"""Benchmark driver for the B200 hot path of ltx-rust.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Prints ONE JSON line (rank 0).  For N > 1 it is launched under torchrun, one
rank per GPU; the step time is the max over ranks.

Workloads:
  denoise_step   config 4 (default): one Euler/CFG denoising step of the
                 48-block 22B-class DiT (D 4096, 32x128 heads, FFN 16384) on
                 T = 12288 tokens (16x24x16 target latent + same-size IC
                 reference), 1024 context tokens, guidance 3.0 (CFG batch 2:
                 cond / uncond contexts), rescale 0.7.  Random-init FP8 e4m3
                 weights merged with a rank-64 LoRA on the device at load.
                 metric tokens/s = 12288 / step time.  At N > 1 the N ranks
                 run ONE sequence (strong scaling, value = 12288/t): at even
                 N the CFG batch's conditional and unconditional passes run
                 on two halves of the GPUs and each half is tensor-parallel
                 as config 4 states (heads and FFN units per rank, NCCL
                 allreduce after each row-split projection), with one
                 all-gather of the two velocities per step (`--parallel
                 cfg_tp`, the default); `--parallel tp` splits the model over
                 all N for both passes.  The N > 1 line also carries the
                 other of those two layouts (`tp` or `cfg_tp`; `tp` only up
                 to 4 GPUs), `tp_nccl` (plain TP with the NCCL exchange), `replicas`
                 (one independent sequence per GPU, no collective: weak
                 scaling) and `chunk_pipeline` (config 5 on the N GPUs).  --parallel chunk
                 makes the replica figure the headline instead.  The N = 1
                 line carries `step_fp8` (the same step with FP8 FFN GEMMs).
  dequant_merge  config 1: FP8 e4m3 [4096,4096] (+scale) + rank-64 bf16 LoRA
                 -> bf16 [4096,4096], metric GB/s of algorithmic bytes; also
                 reported as the `dequant_merge` object of the step line, with
                 the dequant-only (no LoRA) rate beside it.
  chunk_pipeline config 5: 8 overlapping temporal chunks x 8 Euler steps,
                 chunks spread over the ranks, seams exchanged and blended on
                 the device, clip gathered on rank 0 (strong scaling).

`--impl reference` times the reference algorithm's CPU restatement (the
reference is a Rust workspace that cannot be built here) on the host cores,
rank 0 only, on the same config and metric.
"""
from __future__ import annotations

import argparse
import json
import math
import numpy as np
import os
import platform
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "ltx-rust_b200"))

L2_BYTES = 126 * 1024 * 1024
# Config 1 algorithmic bytes: fp8 W + scale + bf16 A and B + bf16 output.
CFG1_BYTES = 4096 * 4096 + 4 + 2 * (64 * 4096 * 2) + 4096 * 4096 * 2
CFG1_FMAS = 4096 * 4096 * 64
# Config 1 without the LoRA (dequant only): fp8 W + scale + bf16 output.
CFG1_DQ_BYTES = 4096 * 4096 + 4 + 4096 * 4096 * 2
# DRAM bytes (read + write) per launch, from one ncu capture of each kernel
# at the bench's shape (kernel_bench.py merge 4096x4096 rank 64; gemm
# 24576x16384x4096 GELU).  The merge's 33.5 MB bf16 output is still dirty in
# L2 when a lone captured launch ends (ncu read 20.02 MB, wrote 0.25 MB), so
# its write-back, which happens after the launch, is added as output bytes.
CFG1_NCU_TRAFFIC = 20.02e6 + 4096 * 4096 * 2
FFN_IN_NCU_TRAFFIC = 1.812415e9 + 0.78335488e9
# self-attention at B=2, H=32, T=12288: DRAM read+write of a B=1, T=8192 launch
# (201.56 MB + 46.14 MB) scaled by the Q/K/V/O bytes (805.3 MB / 268.4 MB)
ATTN_NCU_TRAFFIC = (201.555968e6 + 46.135808e6) * 3.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.out = open(os.devnull, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        if not getattr(self, "lines", None):
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


_T0 = time.time()


def _log(msg):
    """Progress on stderr (the JSON result line is the only stdout)."""
    print(f"[bench {time.time() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ── workload: dequant_merge (config 1) ───────────────────────────────────────

def make_config1(seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(4096, 4096, generator=g) * 0.02
    scale = float((w.abs().max() / 448.0).float())
    q = (w / scale).to(torch.float8_e4m3fn).view(torch.uint8)
    a = (torch.randn(64, 4096, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(4096, 64, generator=g) * 0.01).to(torch.bfloat16)
    return q, scale, a, b


def run_dequant_merge(args, rank, ws, device):
    import torch
    import ltx_b200
    torch.cuda.set_device(device)
    # SETS independent weight sets, larger than L2 together (8 x (16.8 MB fp8 +
    # 33.5 MB bf16 out) = 403 MB), merged back to back in each timed step: no
    # L2 reuse between launches and the host's per-call cost overlaps the GPU.
    SETS = 8
    q, scale, a, b = make_config1(1234 + rank)
    qs = [q.cuda()] + [torch.roll(q, 4096 * (i + 1)).cuda() for i in range(SETS - 1)]
    qd, ad, bd = qs[0], a.cuda(), b.cuda()
    outs = [torch.empty(4096, 4096, dtype=torch.bfloat16, device="cuda") for _ in range(SETS)]
    out = outs[0]
    ctx = ltx_b200.Context(device)
    coeff = ltx_b200.lora_coeff(1.0, 64.0, 64)
    deltas = [(ad.data_ptr(), bd.data_ptr(), 64, ltx_b200.LTX_BF16, ltx_b200.LTX_BF16, coeff)]
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def merge(i):
        ctx.dequant_merge(qs[i].data_ptr(), ltx_b200.LTX_F8_E4M3, True, scale, 4096, 4096, deltas, outs[i].data_ptr(),
                          ltx_b200.LTX_BF16)

    def step():
        merge(0)

    for _ in range(args.warmup):
        for i in range(SETS):
            merge(i)
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    barrier(ws)
    torch.cuda.synchronize()
    # each timed step merges the SETS weights ROUNDS times, so the timed region
    # lasts ~0.3 s and the clock sampler sees it
    ROUNDS = max(1, int(0.3 / (SETS * 80e-6)) // max(args.steps, 1))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record(stream)
        for _ in range(args.steps * ROUNDS):
            for i in range(SETS):
                merge(i)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(ws)
    ctx.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / (args.steps * ROUNDS * SETS), ws)
    times = [ms]
    # the same weights without a LoRA: the HBM-bound dequant-only kernel.  A
    # launch from Python costs more than the ~8 us kernel, so the calls (the
    # same C-ABI calls) are captured once into a CUDA graph on a context of
    # their own and the graph is replayed: the device time of back-to-back
    # dequants.  The eager figure (Python launch per call) is reported beside it.
    def dq(c, i):
        c.dequant_merge(qs[i].data_ptr(), ltx_b200.LTX_F8_E4M3, True, scale, 4096, 4096, [], outs[i].data_ptr(),
                        ltx_b200.LTX_BF16)

    DQ_ROUNDS = 4 * ROUNDS
    for _ in range(args.warmup):
        for i in range(SETS):
            dq(ctx, i)
    barrier(ws)
    torch.cuda.synchronize()
    ds, de = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ds.record(stream)
    for _ in range(args.steps * DQ_ROUNDS):
        for i in range(SETS):
            dq(ctx, i)
    de.record(stream)
    torch.cuda.synchronize()
    ctx.synchronize()
    dq_eager_ms = max_over_ranks(ds.elapsed_time(de) / (args.steps * DQ_ROUNDS * SETS), ws)
    gstream = torch.cuda.Stream()
    gctx = ltx_b200.Context(device, stream=gstream.cuda_stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gstream, capture_error_mode="thread_local"):
        for _ in range(4):
            for i in range(SETS):
                dq(gctx, i)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    gs_, ge_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    G_REPLAYS = max(1, DQ_ROUNDS * args.steps // 4)
    with torch.cuda.stream(gstream):
        gs_.record(gstream)
        for _ in range(G_REPLAYS):
            graph.replay()
        ge_.record(gstream)
    torch.cuda.synchronize()
    dq_ms = max_over_ranks(gs_.elapsed_time(ge_) / (G_REPLAYS * 4 * SETS), ws)
    del graph
    gctx.close()
    # e2e through the C ABI with host buffers: pinned H2D of the step's inputs,
    # the kernel, D2H of the result; all inside the timed region.
    qh, ah, bh = q.pin_memory(), a.pin_memory(), b.pin_memory()
    oh = torch.empty(4096, 4096, dtype=torch.bfloat16).pin_memory()
    e2e_times = []
    for i in range(args.warmup + args.steps):
        flush.fill_(float(i))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        qd.copy_(qh, non_blocking=True)
        ad.copy_(ah, non_blocking=True)
        bd.copy_(bh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)
        e.record(stream)
        e.synchronize()
        if i >= args.warmup:
            e2e_times.append(s.elapsed_time(e))
    ctx.synchronize()
    e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), ws)
    peaks, src = measured_peaks()
    per_launch_ms = sum(times) / len(times)
    achieved = CFG1_BYTES / (per_launch_ms * 1e-3) / 1e9
    res = {
        "metric": "dequant+merge HBM GB/s (config 1: FP8 4096x4096 + rank-64 LoRA -> bf16)",
        "value": ws * CFG1_BYTES / (ms * 1e-3) / 1e9,
        "unit": "GB/s",
        "ms_per_step": ms,   # one config-1 merge
        "higher_is_better": True,
        "scaling": "weak",
        "dtype": "f32 (fp8 in, bf16 out)",
        "config": {"workload": "dequant_merge_config1", "rows": 4096, "cols": 4096, "rank": 64,
                   "weight": "fp8_e4m3 per-tensor scale", "lora": "bf16", "out": "bf16",
                   "l2": "8 distinct weight sets (403 MB > L2) merged back to back; no reuse between launches",
                   "units_per_rank_per_step": 1},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": CFG1_NCU_TRAFFIC, "peak_source": src,
                     "algorithmic_bytes_per_launch": CFG1_BYTES,
                     "fp32_fma_per_launch": CFG1_FMAS,
                     "note": "the bit-exact rank-64 FMA chain makes this kernel FP32-pipe bound, not HBM bound",
                     "traffic_note": "ncu DRAM reads of one launch + the bf16 output's write-back (the output "
                                     "was still in L2 when the captured launch ended)"},
        "e2e": {"value": ws * CFG1_BYTES / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": q.numel() + 2 * a.numel() + 2 * b.numel(),
                "d2h_bytes_per_step": out.numel() * 2},
        "dequant_only": {"value": ws * CFG1_DQ_BYTES / (dq_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": dq_ms,
                         "frac": CFG1_DQ_BYTES / (dq_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"],
                         "peak_source": src, "algorithmic_bytes_per_launch": CFG1_DQ_BYTES,
                         "eager_ms_per_step": dq_eager_ms,
                         "note": "config 1 without the LoRA (fp8 in, bf16 out): 8 distinct weight sets back to back "
                                 "(403 MB > L2), the C-ABI calls replayed from a CUDA graph; eager_ms_per_step is "
                                 "the same with one Python launch per call"},
        "gpu_launches": 2 * SETS * ROUNDS * args.steps,   # pre-pass + merge kernel per merge
        "merges_timed": SETS * ROUNDS * args.steps,
        "clocks": clk.summary(),
    }
    ctx.close()
    return res


# ── workload: denoise_step (config 4) ────────────────────────────────────────

CFG4 = {"transformer": {"num_attention_heads": 32, "attention_head_dim": 128, "in_channels": 128,
                        "out_channels": 128, "num_layers": 48, "cross_attention_dim": 4096, "norm_eps": 1e-6,
                        "positional_embedding_theta": 10000.0, "positional_embedding_max_pos": [20, 2048, 2048],
                        "timestep_scale_multiplier": 1000, "use_middle_indices_grid": True, "rope_type": "split",
                        "apply_gated_attention": False, "cross_attention_adaln": False,
                        "use_prompt_adaln_single": True, "ff_bias": False, "use_keyframes_abs_pos_embedding": False,
                        "caption_proj_before_connector": True}}
LAT_F, LAT_H, LAT_W = 16, 24, 16            # latent [1,128,16,24,16]
T_TARGET = LAT_F * LAT_H * LAT_W             # 6144
T_TOTAL = 2 * T_TARGET                       # + IC reference tokens
S_CTX, D, FF = 1024, 4096, 16384


def step_flops(layers=48, T=T_TOTAL, S=S_CTX, B=2):
    """Matmul FLOPs of one CFG step, per pass of the batch: per block the seven
    projections 2*T*D*(3D + D + D + D + 2F) (self QKV, self out, cross q, cross
    out, FFN in + out) plus cross k/v 2*S*D*2D, and the two attentions
    4*T*T*D + 4*T*S*D (Q.K^T and P.V); at T 12288, S 1024, D 4096, F 16384 that
    is 8.521 TFLOP per block per pass.  The head adds patchify_proj and
    proj_out, 2*T*128*D each."""
    gemm = 2 * T * D * (3 * D + D + D + D + 2 * FF) + 2 * S * D * 2 * D
    attn = 4 * T * T * D + 4 * T * S * D
    head = 2 * T * 128 * D + 2 * T * D * 128
    return B * (layers * (gemm + attn) + head), B * layers * gemm, B * layers * attn


def make_step_inputs(F, H, W, S, Dc, seed):
    """Config-4 sampler state through the product API: target latent N(0,1) with
    the IC reference appended (VideoReferenceCondition::apply_to,
    conditioning.rs:63-106: zeros in the noisy latent, clean reference tokens,
    mask 1 - strength = 0), positions from make_target/reference_positions,
    cond/uncond contexts N(0,1), sigmas from LTX2Scheduler::execute(8, 6144)."""
    import ltx_b200
    rng = np.random.default_rng(seed)
    Tt, C = F * H * W, 128
    ref_tokens = rng.standard_normal((Tt, C), dtype=np.float32)
    latent = np.concatenate([rng.standard_normal((Tt, C), dtype=np.float32), np.zeros((Tt, C), np.float32)])
    clean = np.concatenate([np.zeros((Tt, C), np.float32), ref_tokens])
    mask = np.concatenate([np.ones(Tt, np.float32), np.zeros(Tt, np.float32)])
    pos = np.concatenate([ltx_b200.target_positions(F, H, W), ltx_b200.reference_positions(F, H, W)], axis=2)
    return {"latent": latent, "clean": clean, "mask": mask, "positions": pos,
            "ctx_cond": rng.standard_normal((S, Dc), dtype=np.float32),
            "ctx_uncond": rng.standard_normal((S, Dc), dtype=np.float32),
            "sigmas": ltx_b200.scheduler_execute(8, Tt)}


def step_mode(ws, parallel):
    """How config 4 uses `ws` GPUs: "single" (one GPU), "cfg_tp" (even N: the CFG
    batch's two passes on two halves, each half tensor-parallel), "tp" (every GPU
    one shard of the model, both passes) or "replicas" (one sequence per GPU)."""
    if ws == 1:
        return "single"
    if parallel == "chunk":
        return "replicas"
    return "cfg_tp" if parallel == "cfg_tp" and ws % 2 == 0 else "tp"


def step_config(ws, mode):
    """The config-4 workload as both arms' lines name it (identical dicts)."""
    half = ws // 2
    par = {"single": "one GPU, one sequence",
           "tp": f"tp{ws}: one sequence, heads and FFN units split over {ws} GPUs, NCCL allreduce",
           "cfg_tp": (f"cfg2 x tp{half}: one sequence; the conditional and unconditional passes of the CFG batch "
                      f"on two halves of {half} GPU(s)" + (", heads and FFN units split inside a half (NCCL "
                                                            "allreduce)" if half > 1 else "") +
                      "; one NCCL all-gather of the two velocities per step"),
           "replicas": f"replicas x{ws}: one independent sequence per GPU"}[mode]
    return {"workload": "denoise_step_config4", "layers": 48, "hidden": D, "heads": 32, "head_dim": 128,
            "ffn": FF, "tokens": T_TOTAL, "latent": [1, 128, LAT_F, LAT_H, LAT_W], "ic_reference": True,
            "context_tokens": S_CTX, "cfg_batch": 2, "guidance": 3.0, "rescale": 0.7,
            "weights": "random-init fp8 e4m3 per-tensor scale + rank-64 LoRA merged on device",
            "parallelism": par,
            "l2": "inputs and weights exceed L2 (25.8 GB bf16 weights streamed per step)",
            "step_tflop": step_flops()[0] / 1e12}


def init_step_mode(ctx, mode):
    """Binds the context for `mode`; returns (seed offset of this rank's model and
    inputs, whether the model is split over ranks)."""
    import ltx_b200
    if mode == "tp":
        ltx_b200.init_tensor_parallel(ctx)   # this rank's shard of one model
        return 0, True
    if mode == "cfg_tp":
        _, half, _ = ltx_b200.init_cfg_tensor_parallel(ctx)   # one pass, this rank's shard of it
        return 0, half > 1
    return (dist_env()[1] if mode == "replicas" else 0), False


class StepRunner:
    """One config-4 model and sampler state on this rank's GPU, stepped through
    the C ABI (ltx_denoise_step) on the context's stream."""

    def __init__(self, ctx, seed_model, seed_inputs, precision="bf16", offload_blocks=0):
        import torch
        import ltx_b200
        cfg = json.loads(json.dumps(CFG4))
        if precision != "bf16":
            cfg["gemm_precision"] = precision
        if offload_blocks:
            cfg["offload_blocks"] = offload_blocks
        t0 = time.time()
        self.model = ltx_b200.VideoTransformer.init_random(ctx, json.dumps(cfg), seed=seed_model, lora_rank=64,
                                                           lora_strength=1.0)
        ctx.synchronize()
        self.load_s = time.time() - t0
        self.ctx = ctx
        inp = make_step_inputs(LAT_F, LAT_H, LAT_W, S_CTX, D, seed=seed_inputs)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        self.lat0 = inp["latent"]
        self.lat, self.clean, self.mask = dev(self.lat0), dev(inp["clean"]), dev(inp["mask"])
        self.pos, self.cc, self.cu = dev(inp["positions"]), dev(inp["ctx_cond"]), dev(inp["ctx_uncond"])
        self.mask_h = np.ascontiguousarray(inp["mask"], np.float32)
        self.sig = inp["sigmas"]

    def step(self, i):
        n = len(self.sig) - 1
        s0, s1 = float(self.sig[i % n]), float(self.sig[i % n + 1])
        self.model.denoise_step(self.lat, self.clean, self.mask, self.pos, self.cc, self.cu, s0, max(s1, 0.0), 3.0,
                                0.7, mask_host=self.mask_h)

    def reference_step(self):
        """One step (sigma pair 1 -> 2) from the initial latent: the new latent, on the host."""
        import torch
        self.lat.copy_(torch.from_numpy(np.ascontiguousarray(self.lat0, np.float32)))
        self.step(1)
        self.ctx.synchronize()
        return self.lat.double().cpu()

    def timed(self, steps, warmup, ws, device, clocks=True, label="denoise_timed"):
        """ms per step over `steps` steps after `warmup` (CUDA events on the stream, max over ranks).
        The timed launches sit in an NVTX range named `label` (a profiler can capture just them)."""
        import torch
        for i in range(warmup):
            self.step(i)
        self.ctx.synchronize()
        stream = torch.cuda.current_stream()
        barrier(ws)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(device) if clocks else None
        if clk:
            clk.__enter__()
        torch.cuda.nvtx.range_push(label)
        start.record(stream)
        for i in range(steps):
            self.step(i)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if clk:
            clk.__exit__(None, None, None)
        self.ctx.synchronize()
        barrier(ws)
        return max_over_ranks(start.elapsed_time(end) / steps, ws), (clk.summary() if clk else None)

    def e2e(self, n, ws):
        """ms per step through the C ABI from host buffers: pinned latent in, new latent out, each step."""
        import torch
        lat_h = torch.from_numpy(np.ascontiguousarray(self.lat0, np.float32)).pin_memory()
        out_h = torch.empty_like(lat_h).pin_memory()
        stream = torch.cuda.current_stream()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(ws)
        torch.cuda.synchronize()
        s2.record(stream)
        for i in range(n):
            self.lat.copy_(lat_h, non_blocking=True)
            self.step(i)
            out_h.copy_(self.lat, non_blocking=True)
        e2.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(s2.elapsed_time(e2) / n, ws)
        return ms, lat_h.numel() * 4, out_h.numel() * 4, bool(torch.isfinite(out_h).all())

    def close(self):
        self.model.close()


def run_denoise_step(args, rank, ws, device):
    import torch
    import ltx_b200
    torch.cuda.set_device(device)
    ctx = ltx_b200.Context(device)
    mode = step_mode(ws, args.parallel)
    one_seq = mode != "replicas"   # every rank holds the same weights and inputs
    off, split = init_step_mode(ctx, mode)
    run = StepRunner(ctx, 7 + off, 100 + off, offload_blocks=args.offload_blocks)
    _log(f"model initialised in {run.load_s:.1f}s")
    ms, clocks = run.timed(args.steps, args.warmup, ws, device)
    _log(f"{args.steps} timed steps: {ms:.1f} ms/step")
    e2e_ms, h2d, d2h, ok = run.e2e(max(1, min(args.steps, 3)), ws)
    _log(f"e2e: {e2e_ms:.1f} ms/step")
    bf16_ref = run.reference_step() if ws == 1 else None
    weight_bytes = run.model.weight_bytes()
    # how the split model's sums ran (for the launch count): fused or NCCL, and
    # whether the norms were sequence-parallel (the library's rule: from 4
    # ranks per tensor-parallel group, unless LTX_TP_SEQ_NORMS says otherwise)
    exchange = ctx.tp_exchange()
    tp_group = ws if mode == "tp" else (ws // 2 if mode == "cfg_tp" else 1)
    sp_env = os.environ.get("LTX_TP_SEQ_NORMS", "")
    seq_norms = exchange == "peer" and (sp_env == "1" if sp_env else tp_group >= 4)
    load_s = run.load_s
    run.close()
    # dominant kernels timed alone at the step's shapes
    gemm_ms = attn_ms = None
    M, N, K = 2 * T_TOTAL, FF, D
    H, TA = D // 128, T_TOTAL
    attn_flop = 4.0 * 2 * H * TA * TA * 128
    stream = torch.cuda.current_stream()
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ltx_b200.gemm(ctx, a, w, o, ltx_b200.EPI_GELU_BF16)
    gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gs.record(stream)
    for _ in range(10):
        ltx_b200.gemm(ctx, a, w, o, ltx_b200.EPI_GELU_BF16)
    ge.record(stream)
    torch.cuda.synchronize()
    gemm_ms = gs.elapsed_time(ge) / 10
    _log(f"FFN-in GEMM alone: {gemm_ms:.3f} ms")
    del a, w, o
    # the step's largest kernel by time share, timed alone: self-attention
    # (bf16 Q/K, f16 V as the model feeds it) at B=2, H=32, T=12288
    q = torch.randn(2 * TA, D, device="cuda").to(torch.bfloat16)
    kk = torch.randn(2 * TA, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(2 * TA, D, device="cuda").to(torch.float16)
    ao = torch.empty(2 * TA, D, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ltx_b200.attention(ctx, q, kk, v, ao, 2, H, TA, TA, 1.0 / math.sqrt(128))
    as_, ae = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    as_.record(stream)
    for _ in range(10):
        ltx_b200.attention(ctx, q, kk, v, ao, 2, H, TA, TA, 1.0 / math.sqrt(128))
    ae.record(stream)
    torch.cuda.synchronize()
    attn_ms = as_.elapsed_time(ae) / 10
    _log(f"self-attention alone: {attn_ms:.3f} ms")
    del q, kk, v, ao
    peaks, src = measured_peaks()
    total, gemm_f, attn_f = step_flops()
    gemm_tf = 2.0 * M * N * K / (gemm_ms * 1e-3) / 1e12
    res = {
        "metric": "DiT denoise-step tokens/s (config 4: 48 blocks, T=12288, CFG batch 2 + Euler)",
        "value": (1 if one_seq else ws) * T_TOTAL / (ms * 1e-3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if one_seq and ws > 1 else "weak",
        "dtype": "bf16 (tensor-core GEMM/attention inputs; f32 accumulate, residual and sampler)",
        "config": step_config(ws, mode),
        "model_load_s": load_s,
        **({"offload_blocks": args.offload_blocks, "device_weight_bytes": weight_bytes}
           if args.offload_blocks else {}),
        "roofline": {"bound": "tensor", "kernel": "attn_fwd_kernel, self-attention (B=2, H=32, T=12288, d=128)",
                     "achieved": attn_flop / (attn_ms * 1e-3) / 1e12, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": attn_flop / (attn_ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
                     "traffic": ATTN_NCU_TRAFFIC, "peak_source": src, "algorithmic_flops_per_launch": attn_flop,
                     "traffic_note": "ncu DRAM bytes of a B=1, T=8192 launch scaled by Q/K/V/O bytes",
                     "step_tflops_per_gpu": (total / ws if one_seq else total) / (ms * 1e-3) / 1e12,
                     "step_frac_of_sustained": (total / ws if one_seq else total) / (ms * 1e-3) / 1e12 /
                     peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])},
        "roofline_gemm": {"bound": "tensor", "kernel": "tcgen05 GEMM, FFN-in + GELU (M=24576, N=16384, K=4096)",
                          "achieved": gemm_tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                          "frac": gemm_tf / peaks["bf16_tflops"], "traffic": FFN_IN_NCU_TRAFFIC, "peak_source": src,
                          "algorithmic_flops_per_launch": 2.0 * M * N * K},
        "e2e": {"value": (1 if one_seq else ws) * T_TOTAL / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * launches_per_step(48, split, fused=split and exchange == "peer",
                                                       seq_norms=seq_norms),
        "clocks": clocks,
        "finite_output": ok,
    }
    if ws > 1:
        res["tp_exchange"] = ctx.tp_exchange()
    if ws == 1:
        res["step_fp8"] = run_fp8_step(args, ctx, device, bf16_ref, ms)
    ctx.close()
    return res


def run_fp8_step(args, ctx, device, bf16_ref, bf16_ms):
    """Config 4 with the two FFN projections of every block as native FP8 GEMMs
    (gemm_precision e4m3_ffn: exact e4m3 base weights, per-row e4m3 activations,
    the LoRA factored in the same accumulator), on the same synthetic weights
    as the bf16 step: tokens/s, the FP8 FFN-in GEMM alone, and the rel-L2 of
    one step's new latent and of its update against the bf16 step."""
    import torch
    import ltx_b200
    run = StepRunner(ctx, 7, 100, precision="e4m3_ffn")
    steps = max(3, min(args.steps, 10))
    ms, clocks = run.timed(steps, 3, 1, device, label="denoise_timed_fp8")
    got = run.reference_step()
    lat0 = torch.from_numpy(np.ascontiguousarray(run.lat0, np.float64))
    run.close()
    err = float((got - bf16_ref).norm() / bf16_ref.norm())
    upd_err = float(((got - lat0) - (bf16_ref - lat0)).norm() / (bf16_ref - lat0).norm())
    _log(f"FP8-FFN step: {ms:.1f} ms, latent rel-L2 vs bf16 {err:.2e}, update rel-L2 {upd_err:.2e}")
    # the FP8 FFN-in GEMM alone (e4m3 A and W, per-row / per-tensor scales, GELU)
    M, N, K = 2 * T_TOTAL, FF, D
    # e4m3 operands as the model quantises them: N(0,1) rows scaled to amax 448, N(0,0.02) weights / (amax/448)
    x = torch.randn(M, K, device="cuda")
    sa = x.abs().amax(dim=1) / 448.0
    a = (x / sa[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    del x
    w32 = torch.randn(N, K, device="cuda") * 0.02
    w = (w32 / (w32.abs().max() / 448.0)).to(torch.float8_e4m3fn).view(torch.uint8)
    del w32
    o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ltx_b200.gemm_e4m3(ctx, a, sa, w, 1.0, o, ltx_b200.EPI_GELU_BF16)
    stream = torch.cuda.current_stream()
    gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gs.record(stream)
    for _ in range(10):
        ltx_b200.gemm_e4m3(ctx, a, sa, w, 1.0, o, ltx_b200.EPI_GELU_BF16)
    ge.record(stream)
    torch.cuda.synchronize()
    g_ms = gs.elapsed_time(ge) / 10
    del a, w, o
    g_tf = 2.0 * M * N * K / (g_ms * 1e-3) / 1e12
    return {"gemm_precision": "e4m3_ffn", "value": T_TOTAL / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "steps": steps, "speedup_vs_bf16_step": bf16_ms / ms,
            "rel_l2_latent_vs_bf16_step": err, "rel_l2_update_vs_bf16_step": upd_err, "bar": 3e-2,
            "fp8_ffn_in_gemm": {"achieved": g_tf, "unit": "TFLOP/s", "peak": 4500.0,
                                "frac": g_tf / 4500.0, "peak_source": "nominal dense FP8 (no measured FP8 peak)"},
            "clocks": clocks,
            "note": "same seeded weights as the bf16 step (exact FP8 base, LoRA factored); one step from the same "
                    "latent over all 48 blocks compared against the bf16 model's step"}


def run_replicas(args, rank, ws, device):
    """N independent sequences, one per GPU, no collective on the data path
    (weak scaling): value = N * 12288 / max-over-ranks step time."""
    import torch
    import ltx_b200
    torch.cuda.set_device(device)
    ctx = ltx_b200.Context(device)
    run = StepRunner(ctx, 7 + rank, 100 + rank)
    steps = max(3, min(args.steps, 5))
    ms, clocks = run.timed(steps, 3, ws, device, clocks=False, label="denoise_timed_replicas")
    run.close()
    ctx.close()
    return {"value": ws * T_TOTAL / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "scaling": "weak", "parallelism": f"replicas x{ws}: one independent sequence per GPU"}


def run_parallel_step(args, rank, ws, device, mode, exchange="peer"):
    """Config 4's one sequence on the N GPUs in another layout than the line's
    headline ("tp" or "cfg_tp"), timed like it (max over ranks, a few steps).
    exchange "nccl" sums the tensor-parallel projections with NCCL instead of
    inside the GEMM over peer memory."""
    import torch
    import ltx_b200
    torch.cuda.set_device(device)
    old = os.environ.get("LTX_TP_EXCHANGE")
    os.environ["LTX_TP_EXCHANGE"] = exchange
    try:
        ctx = ltx_b200.Context(device)
        init_step_mode(ctx, mode)
        run = StepRunner(ctx, 7, 100)
        steps = max(3, min(args.steps, 5))
        ms, _ = run.timed(steps, 3, ws, device, clocks=False, label=f"denoise_timed_{mode}_{exchange}")
        used = ctx.tp_exchange()
        run.close()
        ctx.close()
    finally:
        if old is None:
            os.environ.pop("LTX_TP_EXCHANGE", None)
        else:
            os.environ["LTX_TP_EXCHANGE"] = old
    return {"value": T_TOTAL / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "scaling": "strong", "parallelism": step_config(ws, mode)["parallelism"], "tp_exchange": used}


def run_chunk_pipeline(args, rank, ws, device):
    """Config 5: 8 overlapping temporal chunks (pixel chunk_len 121 -> 16 latent
    frames, overlap 16 pixel frames -> 2 latent frames), each a config-4 state
    denoised through the full 8-step schedule with ltx_denoise_loop, chunks
    spread over the ranks (one per GPU at 8 GPUs), then the seam frames are
    exchanged point to point, smoothstep-blended on the device
    (ltx_seam_blend) and the clip gathered on rank 0.  Total work is fixed
    (strong scaling); value = chunks x steps x 12288 tokens / time."""
    import numpy as np
    import torch
    import ltx_b200
    from ltx_b200 import chunks as cp
    torch.cuda.set_device(device)
    ctx = ltx_b200.Context(device)
    n_chunks, lat_len, lat_ov = 8, LAT_F, 2
    pix_plan = ltx_b200.chunk_plan(105 * (n_chunks - 1) + 121, 121, 16)
    assert len(pix_plan) == n_chunks and all(c[2] in (0, 16) for c in pix_plan)
    plan = [(n * (lat_len - lat_ov), n * (lat_len - lat_ov) + lat_len, lat_ov if n else 0) for n in range(n_chunks)]
    total_lat = plan[-1][1]
    asg = cp.assign(n_chunks, ws)
    model = ltx_b200.VideoTransformer.init_random(ctx, json.dumps(CFG4), seed=7, lora_rank=64, lora_strength=1.0)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    states = {}
    for n in asg[rank]:
        inp = make_step_inputs(LAT_F, LAT_H, LAT_W, S_CTX, D, seed=1000 + n)   # seed = base + chunk index
        states[n] = {k: dev(inp[k]) for k in ("latent", "clean", "mask", "positions", "ctx_cond", "ctx_uncond")}
        states[n]["mask_h"] = np.ascontiguousarray(inp["mask"], np.float32)
        states[n]["sigmas"] = inp["sigmas"]
    outs = {n: torch.empty(T_TARGET, 128, device="cuda") for n in asg[rank]}

    chunk_events = []   # per chunk on this rank: device time of its denoise loop

    def pipeline(steps_limit=None):
        chunk_events.clear()
        for n in asg[rank]:
            st = states[n]
            lat = st["latent"].clone()
            sig = st["sigmas"] if steps_limit is None else st["sigmas"][:steps_limit + 1]
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
            model.denoise_loop(lat, st["clean"], st["mask"], st["positions"], st["ctx_cond"], st["ctx_uncond"],
                               sig, 3.0, 0.7, target_tokens=T_TARGET, out=outs[n], mask_host=st["mask_h"])
            ev[1].record()
            chunk_events.append(ev)
        data = {n: outs[n].view(lat_len, -1) for n in asg[rank]}
        recv = cp.exchange_seams(plan, asg, rank, data)
        cp.blend_seams(ctx, plan, recv, data)
        return cp.gather_clip(plan, asg, rank, data, (total_lat, LAT_H * LAT_W * 128))

    for _ in range(args.warmup):   # warm-up: one Euler step per chunk, the exchange and the gather
        pipeline(steps_limit=1)
    ctx.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk:
        start.record(stream)
        clip = pipeline()
        end.record(stream)
        torch.cuda.synchronize()
    ctx.synchronize()
    barrier(ws)
    ms = max_over_ranks(start.elapsed_time(end), ws)
    # the chunks' denoise loops back to back on one GPU: the sum of every
    # chunk's loop time over all ranks (each chunk's loop runs alone on its GPU)
    serial_ms = sum_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in chunk_events), ws)
    steps = len(states[asg[rank][0]]["sigmas"]) - 1 if asg[rank] else 8
    res = {
        "metric": "chunk-parallel pipeline tokens/s (config 5: 8 chunks x 8 Euler steps of config 4, latent seam blend)",
        "value": n_chunks * 8 * T_TOTAL / (ms * 1e-3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "dtype": "bf16 (tensor-core GEMM/attention inputs; f32 accumulate, residual and sampler)",
        "config": {"workload": "chunk_pipeline_config5", "chunks": n_chunks, "euler_steps": steps,
                   "pixel_plan": pix_plan, "latent_plan": plan, "clip_latent_frames": total_lat,
                   "parallelism": f"{len(asg[0])} chunk(s) per GPU over {ws} GPU(s)",
                   "seam": "2 latent frames per seam, sent point to point (NCCL), blended with ltx_seam_blend"},
        "serial_chunks_ms": serial_ms,
        "speedup_vs_serial_chunks": serial_ms / ms,
        "clip_finite": bool(torch.isfinite(clip).all()) if clip is not None else None,
        # per chunk: 8 Euler steps (each as ltx_denoise_step) + 1 seam blend per received seam
        "gpu_launches": len(asg[rank]) * steps * launches_per_step(48) + sum(1 for n in asg[rank] if n > 0),
        "clocks": clk.summary(),
    }
    model.close()
    ctx.close()
    return res


def run_ffn_config2(device, iters=5):
    """Config 2: x bf16 [12288, 4096] N(0,1) -> linear 4096->4096 -> FFN
    4096->16384 (tanh-GELU) -> 4096, weights FP8 e4m3 (per-tensor scale) with
    a rank-64 LoRA.  bf16: the merged weights (ltx_dequant_merge) on the bf16
    tcgen05 GEMM.  e4m3: per-row e4m3 activations (ltx_quantize_rows_e4m3)
    against the exact FP8 base weights on the FP8 GEMM, the LoRA factored in
    the same accumulator.  Both against an f32 reference on the merged f32
    weights; bias zeros (no bias)."""
    import torch
    import ltx_b200
    ctx = ltx_b200.Context(device)
    g = torch.Generator(device="cuda").manual_seed(42)
    M, R = 12288, 64
    x = torch.randn(M, D, device="cuda", generator=g).to(torch.bfloat16)
    layers = []
    for (n_out, n_in) in ((D, D), (FF, D), (D, FF)):
        w32 = torch.randn(n_out, n_in, device="cuda", generator=g) * 0.02
        sw = float(w32.abs().max() / 448.0)
        wq = (w32 / sw).to(torch.float8_e4m3fn).view(torch.uint8)
        A = (torch.randn(R, n_in, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        B = (torch.randn(n_out, R, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        coeff = ltx_b200.lora_coeff(1.0, float(R), R)
        d = [(A.data_ptr(), B.data_ptr(), R, ltx_b200.LTX_BF16, ltx_b200.LTX_BF16, coeff)]
        w_bf16 = torch.empty(n_out, n_in, device="cuda", dtype=torch.bfloat16)
        w_f32 = torch.empty(n_out, n_in, device="cuda")
        ctx.dequant_merge(wq.data_ptr(), ltx_b200.LTX_F8_E4M3, True, sw, n_out, n_in, d, w_bf16.data_ptr(),
                          ltx_b200.LTX_BF16)
        ctx.dequant_merge(wq.data_ptr(), ltx_b200.LTX_F8_E4M3, True, sw, n_out, n_in, d, w_f32.data_ptr(),
                          ltx_b200.LTX_F32)
        sa = float(A.float().abs().max() / 448.0)
        aq = (A.float() / sa).to(torch.float8_e4m3fn).view(torch.uint8)
        b2 = (coeff * B.float() / sw).to(torch.bfloat16)
        layers.append(dict(n_out=n_out, n_in=n_in, wq=wq, sw=sw, w_bf16=w_bf16, w_f32=w_f32, aq=aq, sa=sa, b2=b2))
    ctx.synchronize()
    y = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(M, FF, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    xq = torch.empty(M, FF, device="cuda", dtype=torch.uint8)
    sx = torch.empty(M, device="cuda")
    xa = torch.empty(M, R, device="cuda", dtype=torch.bfloat16)
    epis = (ltx_b200.EPI_BF16, ltx_b200.EPI_GELU_BF16, ltx_b200.EPI_BF16)

    def bf16_chain():
        ltx_b200.gemm(ctx, x, layers[0]["w_bf16"], y, epis[0])
        ltx_b200.gemm(ctx, y, layers[1]["w_bf16"], h, epis[1])
        ltx_b200.gemm(ctx, h, layers[2]["w_bf16"], out, epis[2])

    def e4m3_chain():
        for L, inp, dst, epi in zip(layers, (x, y, h), (y, h, out), epis):
            q = xq[:, :L["n_in"]]
            ltx_b200.quantize_rows_e4m3(ctx, inp, q, sx)
            ltx_b200.gemm_e4m3(ctx, q, None, L["aq"], L["sa"], xa)                     # (x A^T) / sx
            ltx_b200.gemm_e4m3(ctx, q, sx, L["wq"], L["sw"], dst, epi, a2=xa, b2=L["b2"])

    res = {}
    with torch.no_grad():
        ref = x.float() @ layers[0]["w_f32"].t()
        ref = torch.nn.functional.gelu(ref @ layers[1]["w_f32"].t(), approximate="tanh")
        ref = ref @ layers[2]["w_f32"].t()
    tflop = 2.0 * M * D * D + 2 * 2.0 * M * D * FF
    for name, chain in (("bf16", bf16_chain), ("e4m3", e4m3_chain)):
        for _ in range(2):
            chain()
        ctx.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            chain()
        e.record()
        ctx.synchronize()
        ms = s.elapsed_time(e) / iters
        err = float((out.float() - ref).norm() / ref.norm())
        res[name] = {"ms": ms, "tflops": tflop / (ms * 1e-3) / 1e12, "rel_l2_vs_f32": err}
    res["note"] = (f"{tflop / 1e12:.3f} TFLOP per chain (linear + FFN at 12288 tokens); e4m3 includes the row "
                   "quantisation passes and the skinny x.A^T GEMMs of the factored LoRA")
    ctx.close()
    return res


def run_block_forward(device, iters=5):
    """Config 3: one 22B-class block forward (model with num_layers = 1, B = 1,
    T = 12288 tokens with the IC reference, S = 1024), in both GEMM precisions
    (bf16 on merged weights; e4m3 on the exact FP8 base with the LoRA
    factored), with the rel-L2 between them (the FP8 path's bar is 3e-2)."""
    import numpy as np
    import torch
    import ltx_b200
    ctx = ltx_b200.Context(device)
    inp = make_step_inputs(LAT_F, LAT_H, LAT_W, S_CTX, D, seed=300)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    lat = dev(inp["latent"][None])
    ts = dev((inp["mask"] * np.float32(inp["sigmas"][1]))[None])
    pos, cc = dev(inp["positions"]), dev(inp["ctx_cond"][None])
    res, outs = {}, {}
    block_tflop = 2 * T_TOTAL * D * (6 * D + 2 * FF) + 2 * S_CTX * D * 2 * D + 4 * T_TOTAL * T_TOTAL * D + \
        4 * T_TOTAL * S_CTX * D
    for prec in ("bf16", "e4m3_ffn", "e4m3"):
        cfg = json.loads(json.dumps(CFG4))
        cfg["transformer"]["num_layers"] = 1
        cfg["gemm_precision"] = prec
        model = ltx_b200.VideoTransformer.init_random(ctx, json.dumps(cfg), seed=11, lora_rank=64, lora_strength=1.0)
        out = torch.empty(1, T_TOTAL, 128, device="cuda")
        for _ in range(2):
            model.forward(lat, ts, pos, cc, out)
        ctx.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            model.forward(lat, ts, pos, cc, out)
        e.record()
        ctx.synchronize()
        ms = s.elapsed_time(e) / iters
        outs[prec] = out.double().cpu()
        res[prec] = {"ms": ms, "tflops": block_tflop / (ms * 1e-3) / 1e12}
        model.close()
    for prec in ("e4m3_ffn", "e4m3"):
        res[prec]["rel_l2_vs_bf16"] = float((outs[prec] - outs["bf16"]).norm() / outs["bf16"].norm())
    res["note"] = ("one block + patchify/adaLN/output head per forward; "
                   f"{block_tflop / 1e12:.3f} TFLOP of block matmul; e4m3 = FP8 GEMMs for all 7 projections, "
                   "e4m3_ffn = for the 2 FFN projections (north-star FP8 bar: rel-L2 <= 3e-2)")
    ctx.close()
    return res


def launches_per_step(L, tp=False, fused=False, seq_norms=False):
    """Kernels one ltx_denoise_step enqueues, counted from model.cpp's forward.
    Head 9: latent convert, patchify GEMM, sinusoid, 3 small linears, adaLN
    tables, RoPE table, context convert.  Per block 15: 3 norm+modulate, QKV /
    out / cross-q / cross-kv / out / FFN-in / FFN-out GEMMs, fused Q/K
    norm+RoPE, cross q and k norms, 2 attentions.  Split over ranks (tp), the
    Q/K norms become 3 sum-of-squares and 4 apply launches, and each of the 3
    row-split projections runs either (NCCL exchange) as 4 token slabs of a
    GEMM plus a residual add, 40 per block, or (fused exchange) as one GEMM
    plus its wait kernel, 22 per block; sequence-parallel norms add one rank
    barrier after the head.  NCCL's own kernels are not counted.  Output head
    2, sampler 2."""
    per_block = (22 if fused else 40) if tp else 15
    return 9 + L * per_block + 2 + 2 + (1 if tp and fused and seq_norms else 0)


def cpu_model():
    """The host CPU's model string (from /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def cpu_baseline_step(blocks=1, threads=None):
    """The torch-f32 oracle (oracle/dit.py, oracle/sampler.py) on the host
    cores, on the config-4 shapes: `blocks` full-size block forward(s) for the
    CFG batch 2 (T=12288, S=1024, D=4096), the model's per-token head
    (patchify_proj, the adaLN-single MLP on every token as model.rs:196-206
    runs it, the RoPE tables, the output LN + proj_out) for the batch, and the
    CFG combine + global-std rescale + post_process + Euler update.  The step
    is extrapolated as 48 x block + head + sampler."""
    import torch
    from oracle import dit
    from oracle import sampler as osam
    dit.SDPA_Q_CHUNK = 256
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    cfg = dit.DiTConfig(num_layers=1)
    p = {}
    pre = "transformer_blocks.0."
    shapes = {"attn1.to_q": (D, D), "attn1.to_k": (D, D), "attn1.to_v": (D, D), "attn1.to_out.0": (D, D),
              "attn2.to_q": (D, D), "attn2.to_k": (D, D), "attn2.to_v": (D, D), "attn2.to_out.0": (D, D),
              "ff.net.0.proj": (FF, D), "ff.net.2": (D, FF),
              "patchify_proj": (D, 128), "proj_out": (128, D),
              "adaln_single.emb.timestep_embedder.linear_1": (D, 256),
              "adaln_single.emb.timestep_embedder.linear_2": (D, D), "adaln_single.linear": (6 * D, D)}
    for k, (o, i) in shapes.items():
        name = k if not k.startswith(("attn", "ff.")) else pre + k
        p[name + ".weight"] = torch.randn(o, i, generator=g) * 0.02
        if "ff." not in k:
            p[name + ".bias"] = torch.zeros(o)
    for a in ("attn1.", "attn2."):
        p[pre + a + "q_norm.weight"] = torch.ones(D)
        p[pre + a + "k_norm.weight"] = torch.ones(D)
    p[pre + "scale_shift_table"] = torch.randn(6, D, generator=g) * 0.02
    p["scale_shift_table"] = torch.randn(2, D, generator=g) * 0.02
    B = 2
    x = torch.randn(B, T_TOTAL, D, generator=g)
    ctx = torch.randn(B, S_CTX, D, generator=g)
    mod = torch.randn(B, T_TOTAL, 6 * D, generator=g) * 0.02
    pos = torch.from_numpy(np.concatenate([osam.target_positions(LAT_F, LAT_H, LAT_W, B),
                                           osam.reference_positions(LAT_F, LAT_H, LAT_W, B)], axis=2))
    pe = dit.precompute_freqs_cis(pos, cfg)
    t0 = time.time()
    with torch.no_grad():
        for _ in range(blocks):
            dit.block_forward(p, 0, cfg, x, ctx, mod, pe)
    per_block = (time.time() - t0) / blocks
    del x, mod, pe
    # the head: model_forward with no blocks (patchify, per-token adaLN, RoPE tables, output head)
    lat = torch.randn(B, T_TOTAL, 128, generator=g)
    ts = torch.cat([torch.full((B, T_TARGET), 0.9), torch.zeros(B, T_TARGET)], dim=1)
    t0 = time.time()
    with torch.no_grad():
        vel = dit.model_forward(p, cfg, lat, ts, pos, ctx, n_blocks=0).numpy()
    head_s = time.time() - t0
    # the sampler: velocity -> x0, CFG + rescale, post_process, Euler (numpy f32)
    lat_np, ts_np = lat.numpy()[:1], ts.numpy()[:1]
    mask = np.concatenate([np.ones((1, T_TARGET, 1), np.float32), np.zeros((1, T_TARGET, 1), np.float32)], 1)
    t0 = time.time()
    x0c = osam.velocity_to_x0(lat_np, ts_np, vel[:1])
    x0u = osam.velocity_to_x0(lat_np, ts_np, vel[1:])
    x0 = osam.post_process(osam.cfg_combine(x0c, x0u, 3.0, 0.7), mask, lat_np)
    osam.euler_step(lat_np, x0, 0.9, 0.8)
    sampler_s = time.time() - t0
    step_s = per_block * 48 + head_s + sampler_s
    return {"value": T_TOTAL / step_s, "unit": "tokens/s", "cores": threads, "cpu_model": cpu_model(),
            "kind": "port", "blocks_timed": blocks, "extrapolated": True,
            "block_s": per_block, "head_s": head_s, "sampler_s": sampler_s, "step_s": step_s,
            "sample": f"{blocks} full-size block forward(s) (CFG batch 2, T=12288, S=1024) on the torch-f32 "
                      f"oracle: {per_block:.1f} s/block, extrapolated x48 blocks, plus the per-token head "
                      f"({head_s:.1f} s) and the CFG/Euler update ({sampler_s:.2f} s), each timed once"}


def cpu_baseline_dequant(seconds=5.0, threads=None):
    """The oracle (CPU restatement of store.rs:479-521 + 767-793) on all host cores."""
    from oracle.weight_store import LowRankDelta, decode_to_f32, read_raw
    q, scale, a, b = make_config1(1234)
    raw = q.numpy().tobytes()
    d = [LowRankDelta(decode_to_f32("BF16", b.view(__import__("torch").int16).numpy().tobytes()).reshape(4096, 64),
                      decode_to_f32("BF16", a.view(__import__("torch").int16).numpy().tobytes()).reshape(64, 4096),
                      4096, 64, 4096, 1.0)]
    threads = threads or os.cpu_count() or 1
    n, t0 = 0, time.time()
    while True:
        read_raw(raw, "F8_E4M3", True, scale, 4096, 4096, d, "bf16", threads)
        n += 1
        if time.time() - t0 >= seconds:
            break
    dt = (time.time() - t0) / n
    return {"value": CFG1_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} full config-1 reads (4096x4096 fp8 + rank-64 merge -> bf16), {dt * 1e3:.1f} ms each"}


# ── plumbing ─────────────────────────────────────────────────────────────────

def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def sum_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="denoise_step", choices=["denoise_step", "dequant_merge", "chunk_pipeline"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=5.0)
    ap.add_argument("--parallel", default="cfg_tp", choices=["cfg_tp", "tp", "chunk"],
                    help="denoise_step at N>1: one sequence with the CFG batch's two passes on two halves of the "
                         "GPUs, each half tensor-parallel (default; plain tp at odd N), one sequence with every "
                         "GPU a tensor-parallel shard of both passes, or one independent sequence per GPU")
    ap.add_argument("--offload-blocks", type=int, default=0,
                    help="denoise_step: keep the blocks in pinned host memory with this many on the device")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local = dist_env()

    if args.impl == "reference" and args.workload in ("denoise_step", "chunk_pipeline"):
        if rank != 0:
            return
        base = cpu_baseline_step(blocks=1)
        pipe = args.workload == "chunk_pipeline"
        # config 5 is 8 chunks x 8 steps of config 4: on the host cores its
        # tokens/s equals the step's (the chunks run one after another)
        res = {"impl": "reference",
               "metric": ("chunk-parallel pipeline tokens/s (config 5: 8 chunks x 8 Euler steps of config 4, latent "
                          "seam blend)" if pipe else
                          "DiT denoise-step tokens/s (config 4: 48 blocks, T=12288, CFG batch 2 + Euler)"),
               "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus,
               # what ran: one extrapolated step from one timed block, the head and the sampler
               "steps": 1, "warmup": 0, "blocks_timed": base["blocks_timed"], "extrapolated": True,
               "ms_per_step": (64 if pipe else 1) * T_TOTAL / base["value"] * 1e3,
               "higher_is_better": True,
               "scaling": "strong" if pipe or step_mode(args.gpus, args.parallel) in ("tp", "cfg_tp") else "weak",
               "vs_baseline": None,
               "dtype": "f32", "data": "synthetic (random-init weights, N(0,1) activations)",
               "config": ({"workload": "chunk_pipeline_config5"} if pipe else
                          step_config(args.gpus, step_mode(args.gpus, args.parallel))),
               "cpu_baseline": base,
               "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
               "note": "CPU restatement of the reference (oracle/dit.py + oracle/sampler.py, torch/numpy f32): the "
                       "Rust reference cannot be built here.  One full-size block, the head and the sampler update "
                       "are each timed once on the host cores and the 48-block step is extrapolated from them; the "
                       "driver's --steps/--warmup are not repeated (the line's steps/warmup say what ran)."}
        print(json.dumps(res))
        return
    if args.impl == "reference":
        if rank != 0:
            return
        base = cpu_baseline_dequant(seconds=max(args.cpu_seconds, 1.0))
        res = {"impl": "reference", "metric": "dequant+merge HBM GB/s (config 1: FP8 4096x4096 + rank-64 LoRA -> bf16)",
               "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": CFG1_BYTES / base["value"] / 1e6,
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
               "data": "synthetic (seeded N(0,0.02) weight, N(0,0.01) LoRA)",
               "config": {"workload": "dequant_merge_config1"}, "cpu_baseline": base,
               "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
               "note": "CPU restatement of the reference (oracle/fp8_merge.c): the Rust reference cannot be built here"}
        print(json.dumps(res))
        return

    import torch
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    if args.workload == "chunk_pipeline":
        res = run_chunk_pipeline(args, rank, ws, local)
        if rank == 0:
            res.update({"n_gpus": ws, "steps": 1, "warmup": args.warmup, "vs_baseline": None,
                        "data": "synthetic (random-init FP8+LoRA weights, N(0,1) latents/contexts per chunk)"})
            print(json.dumps(res))
    elif args.workload == "dequant_merge":
        res = run_dequant_merge(args, rank, ws, local)
        if rank == 0:
            res.update({"n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "vs_baseline": None,
                        "data": "synthetic (seeded N(0,0.02) weight, N(0,0.01) LoRA)"})
            res["cpu_baseline"] = cpu_baseline_dequant(seconds=args.cpu_seconds) if ws == 1 else None
            print(json.dumps(res))
    else:
        res = run_denoise_step(args, rank, ws, local)
        dq_args = argparse.Namespace(steps=20, warmup=5)
        dq = run_dequant_merge(dq_args, rank, ws, local)
        _log(f"dequant+merge: {dq['value']:.0f} GB/s")
        ffn = run_ffn_config2(local) if ws == 1 else None
        if ffn:
            _log(f"config 2 (linear+FFN): bf16 {ffn['bf16']['ms']:.2f} ms {ffn['bf16']['tflops']:.0f} TFLOP/s "
                 f"rel-L2 {ffn['bf16']['rel_l2_vs_f32']:.2e}; e4m3 {ffn['e4m3']['ms']:.2f} ms "
                 f"{ffn['e4m3']['tflops']:.0f} TFLOP/s rel-L2 {ffn['e4m3']['rel_l2_vs_f32']:.2e}")
        blk = run_block_forward(local) if ws == 1 else None
        if blk:
            _log(f"block forward: bf16 {blk['bf16']['ms']:.2f} ms, e4m3_ffn {blk['e4m3_ffn']['ms']:.2f} ms "
                 f"(rel-L2 {blk['e4m3_ffn']['rel_l2_vs_bf16']:.2e}), e4m3 {blk['e4m3']['ms']:.2f} ms "
                 f"(rel-L2 {blk['e4m3']['rel_l2_vs_bf16']:.2e})")
        if ws > 1:
            mode = step_mode(ws, args.parallel)
            if mode != "replicas":
                rep = run_replicas(args, rank, ws, local)
                _log(f"replicas: {rep['ms_per_step']:.1f} ms/step, {rep['value']:.0f} tokens/s")
                res["replicas"] = rep
            # the other single-sequence layout beside the headline's
            # (plain TP with the fused exchange is not run past 4 GPUs: that
            # path has not been exercised on 8; the NCCL-exchange TP line below
            # covers plain TP there)
            other = ("tp" if ws <= 4 else None) if mode == "cfg_tp" else \
                ("cfg_tp" if mode == "tp" and ws % 2 == 0 else None)
            if other:
                o = run_parallel_step(args, rank, ws, local, other)
                _log(f"{other}: {o['ms_per_step']:.1f} ms/step, {o['value']:.0f} tokens/s ({o['tp_exchange']})")
                res[other] = o
            # the tensor-parallel sums by NCCL allreduce instead of inside the GEMM
            tp_mode = "tp" if mode in ("tp", "cfg_tp") else None
            if tp_mode:
                o = run_parallel_step(args, rank, ws, local, tp_mode, exchange="nccl")
                _log(f"{tp_mode} (NCCL exchange): {o['ms_per_step']:.1f} ms/step, {o['value']:.0f} tokens/s")
                res[f"{tp_mode}_nccl"] = o
            pl_args = argparse.Namespace(warmup=3)
            pl = run_chunk_pipeline(pl_args, rank, ws, local)
            _log(f"config-5 pipeline: {pl['ms_per_step'] / 1e3:.2f} s, {pl['speedup_vs_serial_chunks']:.2f}x the "
                 "serial chunks")
            res["chunk_pipeline"] = {k: pl[k] for k in ("metric", "value", "unit", "ms_per_step", "serial_chunks_ms",
                                                        "speedup_vs_serial_chunks", "clip_finite")}
            res["chunk_pipeline"]["config"] = pl["config"]
        if rank == 0:
            res.update({"n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "vs_baseline": None,
                        "data": "synthetic (random-init FP8+LoRA weights, N(0,1) latent/reference/contexts)"})
            res["dequant_merge"] = {k: dq[k] for k in ("metric", "value", "unit", "ms_per_step", "roofline", "e2e",
                                                       "dequant_only")}
            if ffn:
                res["linear_ffn_config2"] = ffn
            if blk:
                res["block_forward_config3"] = blk
            if ws == 1 and args.cpu_seconds > 0:
                res["cpu_baseline"] = cpu_baseline_step(blocks=1)
                _log(f"CPU baseline (one block): {res['cpu_baseline']['sample']}")
                res["dequant_merge"]["cpu_baseline"] = cpu_baseline_dequant(seconds=min(args.cpu_seconds, 3.0))
                _log("CPU dequant baseline done")
            print(json.dumps(res))
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
