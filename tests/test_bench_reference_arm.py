"""CPU check of bench.py's reference arm (`--impl reference`: the CPU oracle
port timed on the host cores): one run prints one JSON line with the keys
the driver reads, and a non-zero rank under torchrun exits 0 without work."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, args=()):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                           *args], cwd=REPO, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    res = _run()
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["unit"] == "TFLOPS" and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_without_work():
    res = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1", "MASTER_ADDR": "127.0.0.1",
                "MASTER_PORT": "29598"}, ("--gpus", "2"))
    assert res.returncode == 0, res.stderr[-2000:]
    assert not [ln for ln in res.stdout.splitlines() if ln.startswith("{")]


def test_packed_flag_is_validated():
    """--packed applies to the decode workloads only, and the fused one takes
    at most 16 rows (one launch per call)."""
    for args in (["--workload", "prefill", "--packed"], ["--workload", "decode-fused", "--packed", "--m", "32"]):
        res = subprocess.run([sys.executable, "bench.py", *args], cwd=REPO, capture_output=True, text=True,
                             timeout=300)
        assert res.returncode == 2 and "--packed" in res.stderr, (args, res.stderr[-500:])
