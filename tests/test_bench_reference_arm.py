"""bench.py's reference arm (`--impl reference`): the reference's CPU path (the oracle port) timed on the host cores,
on the same config as the GPU arm. It must not load this repository's CUDA library or import its package, or the
comparison between the two arms would not be between the reference and this code. Run in a fresh process; CPU only
(one bounded step of config 2, a few seconds)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit:
    pass
maps = open("/proc/self/maps").read()
print(json.dumps({"probe": True, "libtrnopt_loaded": "libtrnopt" in maps,
                  "trnopt_modules": sorted(m for m in sys.modules if m == "trnopt" or m.startswith("trnopt."))}))
"""


def test_reference_arm_runs_the_cpu_path_without_this_library():
    out = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    line = next(l for l in lines if l.get("impl") == "reference")
    probe = next(l for l in lines if l.get("probe"))
    assert line["config"]["workload"] == "cfg2" and line["unit"] == "ms/iter" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert not probe["libtrnopt_loaded"], "the reference arm mapped this repository's CUDA library"
    assert probe["trnopt_modules"] == [], probe["trnopt_modules"]
