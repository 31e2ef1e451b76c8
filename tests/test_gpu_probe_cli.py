"""mpp41probe, the C++ mirror of the reference CLI (main.swift:80-162), run as a
subprocess on the GPU: roundtrip checks pass, and the MXFP4 MLP rows print the
reference's published checksum (403573 over 32 samples, README.md:292-295) to
within one unit of the last printed digit."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

PROBE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mpp-4.1-fp4-fp8-block_b200", "bin",
                     "mpp41probe")


def test_probe_roundtrips_pass():
    r = subprocess.run([PROBE], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().endswith("PASS")
    assert r.stdout.count(": pass") == 3


def test_probe_mlp_rows_and_checksum():
    r = subprocess.run([PROBE, "--mlp-benchmark", "--iterations", "3"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rows = re.findall(r"  (MXFP4[^\n]*):\n    [0-9.]+ ms/MLP, [0-9.]+ effective TOPS\n    checksum: ([-0-9.e+]+) over 32 samples",
                      r.stdout)
    assert len(rows) == 7, r.stdout
    for name, value in rows:
        assert abs(float(value) - 403573.0) <= 1.0, (name, value)
    assert "W8A8" in r.stdout and "W2A8" in r.stdout
