"""bench.py's reference arm (the reference's CPU math path on the host cores) runs without a
GPU: its JSON line must carry the keys of the benchmark contract, and under torchrun only
rank 0 prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(args, extra_env=None, timeout=300):
    env = dict(os.environ)
    env.update(extra_env or {})
    env.setdefault("OMP_NUM_THREADS", str(min(8, os.cpu_count() or 1)))
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True,
                          text=True, timeout=timeout, cwd=ROOT, env=env)


def test_reference_arm_prints_one_contract_line():
    r = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "3", "--cpu-budget", "2"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "dtype", "data", "config", "cpu_baseline", "e2e", "vs_baseline"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference") and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    r = run_bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--cpu-budget", "1"],
                  extra_env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def _contract_line(r):
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_config_is_the_gpu_arms():
    """Both arms describe the same workload with the same config dict, so a driver can
    pair their lines; the reference line also gives ms_per_step for the whole workload."""
    sys.path.insert(0, ROOT)
    import bench
    d = _contract_line(run_bench(["--impl", "reference", "--steps", "1", "--cpu-budget", "2"]))
    assert d["config"] == bench.config_single()
    assert d["ms_per_step"] > 0


def test_torchrun_world_one_times_the_c5_slice():
    """Under torchrun every WORLD_SIZE, 1 included, times 64 C5 heads per rank, so a 1->8
    scaling run divides like by like (the reference arm follows the same rule)."""
    sys.path.insert(0, ROOT)
    import bench
    d = _contract_line(run_bench(["--impl", "reference", "--steps", "1", "--cpu-budget", "2"],
                                 extra_env={"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"}))
    assert d["config"] == bench.config_multi(1) and d["n_gpus"] == 1
    assert "C5 slice" in d["config"]["workload"]
