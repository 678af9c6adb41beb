"""The reference arm of bench.py (the CPU oracle on every host core) runs on CPU and prints the
contract's JSON line: impl, the arm's metric and unit, a cpu_baseline naming its cores, and an e2e
object with no host-device traffic."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_its_line():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup",
                          "0", "--gaussians", "20000", "--channels", "32"],
                         capture_output=True, text=True, timeout=300, check=True).stdout
    line = json.loads(out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "views/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 0
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "views/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
