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
    r = subprocess.run([PROBE, "--mlp-benchmark", "--mlp-iterations=3"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rows = re.findall(r"  (MXFP4[^\n]*):\n    [0-9.]+ ms/MLP, [0-9.]+ effective TOPS\n    checksum: ([-0-9.e+]+) over 32 samples",
                      r.stdout)
    assert len(rows) == 7, r.stdout
    for name, value in rows:
        assert abs(float(value) - 403573.0) <= 1.0, (name, value)
    assert "W8A8" in r.stdout and "W2A8" in r.stdout


def _json_rows(stdout):
    import json
    return [json.loads(l) for l in stdout.splitlines() if l.startswith("{")]


def test_probe_new_rows_as_json():
    """--w4a4 and --moe rows (no reference counterpart) print JSON lines with --json."""
    r = subprocess.run([PROBE, "--w4a4", "--moe", "--json", "--mlp-iterations=2", "--seed", "3"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rows = _json_rows(r.stdout)
    names = [d["row"] for d in rows]
    assert any(n.startswith("W4A4 MXFP4") for n in names) and any(n.startswith("W4A4 NVFP4") for n in names)
    assert any(n.startswith("MoE W4A4") for n in names)
    assert all(d["ms"] > 0 and d["tops"] > 0 for d in rows)


def test_probe_mode_baseline_changes_only_the_mxfp4_rows():
    base = subprocess.run([PROBE, "--mlp-benchmark", "--json", "--mlp-iterations=2"], capture_output=True, text=True,
                          timeout=300)
    modeb = subprocess.run([PROBE, "--mlp-benchmark", "--json", "--mlp-iterations=2", "--mode", "baseline"],
                           capture_output=True, text=True, timeout=300)
    assert base.returncode == 0 and modeb.returncode == 0, base.stderr + modeb.stderr
    a = {d["row"]: d["checksum"] for d in _json_rows(base.stdout)}
    b = {d["row"]: d["checksum"] for d in _json_rows(modeb.stdout)}
    assert a.keys() == b.keys() and len(a) == 18 + 5   # MPP/MXFP4 rows + scalar half rows
    for name in a:
        if name.startswith("MXFP4"):
            assert a[name] != b[name], name          # mode B inputs
        else:
            assert a[name] == b[name], name          # reference seeds unchanged


def test_probe_rejects_several_gpus():
    r = subprocess.run([PROBE, "--gpus", "2"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "one process per GPU" in r.stderr


def test_probe_reference_flag_surface():
    """--name=value sizes, the FP4 group sweep rows of both sections, and the
    relative slowdown table (main.swift:2772-2783); unknown flags are ignored."""
    r = subprocess.run([PROBE, "--benchmark", "--mlp-benchmark", "--fp4-group-sweep", "--matmul-size=512",
                        "--iterations=2", "--mlp-tokens=32", "--mlp-hidden=512", "--mlp-iterations=1",
                        "--no-such-flag"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "ignoring argument --no-such-flag" in r.stderr
    assert "shape: A 512x512, B 512x512, C 512x512" in r.stdout
    assert "shape: tokens=32, hidden=512, intermediate=2048" in r.stdout
    assert "FP4 E2M1 g8 -> FP32 accumulate:" in r.stdout
    assert "half MLP with FP4 E2M1 g8 weights: half x FP4 -> half:" in r.stdout
    assert "half MLP with INT2 weights: half x int2b_format -> half:" in r.stdout
    assert r.stdout.count("relative slowdown, best = ") == 2
    assert r.stdout.strip().endswith("PASS")
