"""The bench's reference arm on the CPU: the JSON line's contract, and that the
process times the oracle only (libobn.so never mapped), as the driver checks."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROBE = """
import runpy, sys
sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0']
try:
    runpy.run_path('bench.py', run_name='__main__')
except SystemExit as e:
    if e.code not in (None, 0):
        raise
print('LIBOBN_MAPPED', 'libobn.so' in open('/proc/self/maps').read())
"""


def test_reference_arm_json_line_and_no_libobn():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", _PROBE], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    j = json.loads(lines[0])
    assert j["impl"] == "reference"
    assert j["metric"] == "ternary decode GEMV GB/s" and j["unit"] == "GB/s"
    assert j["value"] > 0 and j["higher_is_better"] is True
    assert j["steps"] == 1 and j["warmup"] == 0 and j["n_gpus"] == 1
    assert "cfg1 decode GEMV sweep" in j["config"]["workload"]
    cb = j["cpu_baseline"]
    assert cb["value"] == j["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["sample"]
    e2e = j["e2e"]
    assert e2e["value"] == j["value"] and e2e["unit"] == j["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "LIBOBN_MAPPED False" in r.stdout
