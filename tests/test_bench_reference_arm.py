"""The reference arm of bench.py (the CPU oracle on every host core) runs on CPU and prints the
contract's JSON line: impl, the arm's metric and unit, the GPU arm's config, a cpu_baseline naming
its cores, and an e2e object with no host-device traffic.  The arm maps none of this library's
native code (importing the package loads libhds_b200.so only on the first entry-point call)."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]

RUN_AND_CHECK_MAPS = """
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--gaussians", "20000",
            "--channels", "32"]
runpy.run_path(sys.argv[0], run_name="__main__")
maps = open("/proc/self/maps").read()
print("MAPS_HAVE_LIB", "libhds_b200" in maps)
"""


def test_reference_arm_prints_its_line():
    out = subprocess.run([sys.executable, "-c", RUN_AND_CHECK_MAPS], cwd=REPO, capture_output=True, text=True,
                         timeout=300, check=True).stdout
    lines = out.strip().splitlines()
    assert lines[-1] == "MAPS_HAVE_LIB False", "the reference arm loaded libhds_b200.so"
    line = json.loads(lines[-2])
    assert line["impl"] == "reference" and line["unit"] == "views/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 0
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "views/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"].startswith("config2 scene") and line["config"]["channels"] == 32
    assert line["config"]["parallelism"] == "dp1"
