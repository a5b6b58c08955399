"""bench.py's reference arm on the CPU: it runs without a GPU and prints the contract's JSON line.

The driver launches `bench.py --impl reference` beside the product's own line and compares
the two; this checks the reference line's shape: the shared keys, `impl`, a `cpu_baseline`
describing the run, and an `e2e` with no host-device bytes.
"""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--tokens", "2048", "--pool-blocks", "300"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 1 and line["warmup"] == 1
    assert line["config"]["session_blocks"] == 128 and line["config"]["pool_blocks"] == 300
    assert line["value"] > 0 and line["higher_is_better"] is True and line["scaling"] == "weak"
    base = line["cpu_baseline"]
    assert base["value"] == line["value"] and base["cores"] >= 1 and base["kind"] in ("reference", "port")
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
