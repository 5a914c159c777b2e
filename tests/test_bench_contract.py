"""bench.py's output contract on the CPU: the reference arm (the oracle port timed on the host
cores) prints exactly one line on standard output, a JSON object with the keys a driver reads."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# Runs bench.py's reference arm as __main__, then reports on standard error whether any of the
# package's compiled libraries was mapped into the process (the arm must load none of them).
_WRAPPER = """
import runpy, sys
sys.argv = [sys.argv[1], "--impl", "reference", "--steps", "1", "--warmup", "3"]
runpy.run_path(sys.argv[0], run_name="__main__")
maps = open("/proc/self/maps").read()
sys.stderr.write("PACKAGE_SO_MAPPED=%d\\n" % ("15642_moe_b200/lib" in maps))
"""


def test_reference_arm_prints_one_json_line():
    res = subprocess.run([sys.executable, "-c", _WRAPPER, os.path.join(REPO, "bench.py")],
                         capture_output=True, text=True, timeout=900, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = res.stdout.splitlines()
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3 and d["value"] > 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # same configuration object as this package's arm at N = 1, no compiled package code loaded
    sys.path.insert(0, REPO)
    import bench
    assert d["config"] == bench.config_1gpu()
    assert "PACKAGE_SO_MAPPED=0" in res.stderr, res.stderr[-2000:]
