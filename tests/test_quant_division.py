"""The quantizers' fast division (hn_common.cuh: x2_quot) gives the same int8 codes and e4m3 bytes as the IEEE
quotient over the whole bf16 input domain: tests/division_check.c enumerates every bf16 absmax and every bf16
value within it (1.07e9 pairs, both signs) and compares; it also checks the scales absmax/127 and absmax/448 that
the kernels form by the same fma-corrected quotient (quot_const) for every bf16 absmax. CPU only; about 20 s on 8 threads."""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.mark.slow
def test_fast_division_exhaustive(tmp_path):
    exe = os.path.join(tmp_path, "division_check")
    subprocess.check_call(["gcc", "-O2", "-march=native", "-ffp-contract=off", "-fopenmp", "-o", exe,
                           os.path.join(HERE, "division_check.c"), os.path.join(ROOT, "oracle", "hn_oracle.c"), "-lm"])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "int8 code mismatches 0, e4m3 byte mismatches 0" in r.stdout
    assert "scale mismatches 0" in r.stdout
