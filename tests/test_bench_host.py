"""bench.py's host-side figures and its CPU reference arm, without a GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_step_flops_match_the_per_block_figures():
    """Config 4: 8.521 TFLOP per block per CFG pass (5.841 of GEMM, 2.680 of attention),
    two passes, 48 blocks, plus the head (patchify, adaLN on the distinct timesteps, proj_out)."""
    import bench
    total, gemm, attn = bench.step_flops()
    assert abs(attn / 1e12 - 2 * 48 * 2.680) < 0.1
    assert abs(gemm / 1e12 - 2 * 48 * 5.841) < 0.2
    assert 2 * 48 * 8.521e12 < total < 2 * 48 * 8.521e12 + 3e12


def test_launch_count_matches_the_profiled_step():
    """The ncu launch list of one config-4 step holds 733 kernels."""
    import bench
    assert bench.launches_per_step(48) == 733


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                        "dequant_merge", "--steps", "1", "--warmup", "1", "--cpu-seconds", "0.5"],
                       capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["warmup"] >= 3
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
