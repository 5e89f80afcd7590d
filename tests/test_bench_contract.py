"""bench.py's output contract, checked on CPU through its reference arm (the reference's CPU path): exactly one
line on stdout, JSON, with the keys the driver reads, for each workload."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload", ["gemm", "fp8", "elementwise"])
def test_reference_arm_json_line(workload):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", workload,
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3
    assert {"value", "unit", "cores", "kind", "sample"} <= set(d["cpu_baseline"])
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_reference_arm_loads_no_product_code():
    """The reference arm times the reference's own CPU arithmetic: it imports nothing of hy_nomas_b200 and maps no
    library of this repository (only torch and oracle/torch_ref.py)."""
    code = ("import runpy, sys\n"
            "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'gemm', '--steps', '1', '--warmup', '3']\n"
            "runpy.run_path('bench.py', run_name='__main__')\n"
            "maps = open('/proc/self/maps').read()\n"
            "assert not any(m.startswith('hy_nomas_b200') for m in sys.modules), 'product imported'\n"
            "assert 'libhynomas' not in maps and 'liboracle' not in maps, 'repository library mapped'\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert json.loads(r.stdout.strip().splitlines()[-1])["impl"] == "reference"
