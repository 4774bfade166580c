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


def test_reference_arm_names_what_it_ran_with_the_same_config(monkeypatch, capsys):
    """The denoise-step reference arm extrapolates one timed block (plus head and sampler) to the
    step: its line says so (blocks_timed, extrapolated, steps 1) and carries the same config
    dict as this build's line at the same GPU count."""
    import bench
    canned = {"value": 10.0, "unit": "tokens/s", "cores": 4, "cpu_model": "x", "kind": "port",
              "blocks_timed": 1, "extrapolated": True, "sample": "canned"}
    monkeypatch.setattr(bench, "cpu_baseline_step", lambda blocks=1: dict(canned))
    for gpus, mode in ((1, "single"), (8, "cfg_tp")):
        monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--gpus", str(gpus), "--steps", "20",
                                          "--warmup", "5"])
        bench.main()
        d = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert d["impl"] == "reference" and d["steps"] == 1 and d["blocks_timed"] == 1 and d["extrapolated"]
        assert d["config"] == bench.step_config(gpus, mode)
        assert d["cpu_baseline"]["cpu_model"] == "x"


def test_step_layouts():
    """How config 4 uses N GPUs: one GPU; at even N the CFG pair over two
    tensor-parallel halves (the default); plain TP at odd N or on request; one
    sequence per GPU with --parallel chunk.  The config names the layout."""
    import bench
    assert bench.step_mode(1, "cfg_tp") == "single"
    assert bench.step_mode(2, "cfg_tp") == "cfg_tp"
    assert bench.step_mode(3, "cfg_tp") == "tp"
    assert bench.step_mode(8, "tp") == "tp"
    assert bench.step_mode(8, "chunk") == "replicas"
    par = bench.step_config(8, "cfg_tp")["parallelism"]
    assert par.startswith("cfg2 x tp4") and "allreduce" in par
    assert "allreduce" not in bench.step_config(2, "cfg_tp")["parallelism"]
    assert bench.step_config(4, "tp")["parallelism"].startswith("tp4")
    assert bench.step_config(1, "single")["workload"] == "denoise_step_config4"
