"""bench.py's reference arm on the host CPU: the JSON line the driver pairs with ours.

`bench.py --impl reference` times the reference's CPU path (the oracle port, since the
Rust / ANE reference cannot run on Linux) on the same metric, unit and direction as the
B200 arm, with the `cpu_baseline` and zero-copy `e2e` objects the contract asks for.
One timed step of one 512-token sequence of the 600M train step keeps this under a minute.
"""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    sys.path.insert(0, str(ROOT))
    import bench  # the metric string both arms print
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "sample" in cb and cb["unit"] == "tok/s"
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == "tok/s"
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
