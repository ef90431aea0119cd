"""bench.py's reference arm (CPU): the JSON line keeps the contract's keys for
the large CNN (the reference's C library, built under oracle/_ref) and the LM
(the float64 restatement), and a rank other than 0 exits 0 without work."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, env=e, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]


@pytest.mark.parametrize("workload", ["large_cnn", "char_transformer_lm"])
def test_reference_arm_line(workload):
    lines = run("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "0")
    assert len(lines) == 1
    d = lines[0]
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["metric"] == "train samples/s (fwd+bwd+step)" and d["unit"] == "samples/s"
    assert d["config"]["workload"] == workload
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    assert run("--impl", "reference", "--steps", "1", "--warmup", "0",
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
