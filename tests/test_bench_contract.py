"""bench.py's reference arm prints the one JSON line the driver reads (CPU only).

The reference arm times the reference's eager PyTorch path on the host cores;
this runs it on a short sequence and checks the line's contract keys, and that
the arm loads nothing of this library (its path must be the reference's own)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0', '--seq', '4128']\n"
        "try:\n"
        "    runpy.run_path('bench.py', run_name='__main__')\n"
        "finally:\n"
        "    print('LIBH3B_LOADED', 'libh3b' in open('/proc/self/maps').read(), file=sys.stderr)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is False
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "LIBH3B_LOADED False" in r.stderr
