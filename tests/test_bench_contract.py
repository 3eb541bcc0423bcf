"""bench.py's reference arm on the CPU: one JSON line with the contract's keys (the GPU arm
needs a B200 and is exercised by the benchmark runs themselves)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("qwen3-30b-a3b")


def test_reference_arm_config_equals_gpu_arm_config():
    """Both arms describe the default workload with the same `config` object (the GPU
    arm builds it with the same function from the same workload table)."""
    import argparse
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    import mlx_rs_b200.synth as S
    args = argparse.Namespace(workload="decode", tokens=None)
    cfg, _, T, regime, layers = bench.make_workload(args, S, host=False)
    want = bench.workload_config(cfg, regime, T, 1, layers)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][0])
    assert d["config"] == want
    assert [c[1] for c in bench.CONFIG_RECORDS if c[1] in bench.WORKLOADS] == [c[1] for c in bench.CONFIG_RECORDS]
