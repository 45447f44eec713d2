"""bench.py's reference arm runs on the host cores (the numpy port of reference.py), so its JSON line
can be checked here without a GPU: the keys and types the driver reads, and the e2e / cpu_baseline
objects this tier asks of the reference arm. CPU only."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_line(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--ref-step-seconds", "0.2", *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("args,unit,higher", [((), "TOP/s", True), (("--workload", "act_quant"), "GB/s", True),
                                              (("--workload", "index_prefill"), "ms", False)])
def test_reference_arm_json_contract(args, unit, higher):
    d = _ref_line(*args)
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["unit"] == unit and d["higher_is_better"] is higher and d["n_gpus"] == 1
    assert isinstance(d["value"], (int, float)) and d["value"] > 0 and d["warmup"] >= 3
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == unit
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
