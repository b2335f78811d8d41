"""bench.py's reference arm (`--impl reference`) on the host cores: one JSON
line with the contract's keys, the same metric and unit as the product arm,
an e2e entry that moves no bytes, a described cpu_baseline, and no product
library loaded (the arm times the CPU restatement of the reference's path on
inputs from the oracle's own generator)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROBE = r"""
import json, os, sys
sys.path.insert(0, {root!r})
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"]
import bench
bench.main()
maps = open("/proc/self/maps").read()
print("LOADED_PRODUCT=" + str("libce_b200" in maps))
"""


def test_reference_arm_line():
    out = subprocess.run([sys.executable, "-c", _PROBE.format(root=ROOT)], cwd=ROOT, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert "LOADED_PRODUCT=False" in out.stdout
