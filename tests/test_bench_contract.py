"""The reference arm of `bench.py` on the host (no GPU): one JSON line on rank
0 with the keys of the device arm's line, the CPU restatement timed on a
bounded sample, and nothing printed by the other ranks of a torchrun launch."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*argv, env=None):
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *argv], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    return [ln for ln in p.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("workload", ["mlp", "ref-forward"])
def test_reference_arm_line(workload):
    lines = _bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "0")
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == ("samples/s" if workload == "mlp" else "tokens/s")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_are_silent():
    # under torchrun with N > 1 only rank 0 times and prints
    lines = _bench("--impl", "reference", "--workload", "mlp", "--steps", "1", "--warmup", "0",
                   env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert lines == []
