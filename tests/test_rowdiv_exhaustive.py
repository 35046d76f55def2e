"""The rowwise quantisers replace the IEEE divide x / s by a reciprocal product with one
fused-multiply-add correction (e4m3_quotient, fastforward_b200/csrc/common.cuh).  This CPU
test compiles tests/rowdiv_exhaustive.c and runs it over the callers' whole domain (every
bf16 row maximum a, every bf16 x with |x| <= a, both signs): every e4m3 byte must equal the
divide's.  The GPU parity tests then compare the device bytes with the oracle, which
divides."""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_rowwise_quotient_matches_ieee_divide_on_every_bf16_pair(tmp_path):
    exe = tmp_path / "rowdiv_exhaustive"
    base = ["gcc", "-O2", "-ffp-contract=off", str(HERE / "rowdiv_exhaustive.c"), "-o", str(exe), "-lm"]
    if subprocess.run(base[:1] + ["-fopenmp"] + base[1:], capture_output=True).returncode != 0:
        subprocess.run(base, check=True, capture_output=True)  # no OpenMP: one thread
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900)
    fields = r.stdout.split()
    counts = dict(zip(fields[0::2], map(int, fields[1::2])))
    assert counts["pairs"] == 1_065_402_240  # sum over a of (a's index + 1) x 2 signs
    assert counts["byte_differs"] == 0, r.stdout
    assert r.returncode == 0
