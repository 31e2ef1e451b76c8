"""Regenerate tests/golden/reference_kats.json from the reference's own text.

The reference (Swift + Metal) cannot run here, so its golden values are
read as text:
  * the three packed-roundtrip known-answer cases of main.swift:108-132
    (inputs, expected unpacked values, kernel names), and
  * the published MXFP4 MLP checksum "403573 over 32 samples"
    (README.md:292-295) for tokens=128, hidden=1024, intermediate=4096.
Run once in a container that has the reference mounted:
    python tests/golden/make_golden.py /path/to/reference
The JSON it writes is committed; tests never read the reference itself.
"""
from __future__ import annotations

import json
import os
import re
import sys


def _floats(text: str) -> list[float]:
    return [float(t.replace("_", "")) for t in re.findall(r"-?[0-9][0-9_]*\.?[0-9]*", text)]


def main(ref_root: str) -> None:
    main_swift = open(os.path.join(ref_root, "Sources/MetalFP41Probe/main.swift")).read()
    readme = open(os.path.join(ref_root, "README.md")).read()
    cases = []
    pat = re.compile(r'PackedNumericCase\(\s*name:\s*"([^"]+)",\s*kernelName:\s*"([^"]+)",\s*'
                     r'inputs:\s*\[([^\]]*)\],\s*expected:\s*\[([^\]]*)\],\s*packedByteCount:\s*(\d+)', re.S)
    for m in pat.finditer(main_swift):
        cases.append({"name": m.group(1), "kernel": m.group(2), "inputs": _floats(m.group(3)),
                      "expected": _floats(m.group(4)), "packed_bytes": int(m.group(5))})
    assert len(cases) == 3, cases
    tol = re.search(r"abs\(lhs - rhs\) <= ([0-9._]+)", main_swift).group(1).replace("_", "")
    cks = re.search(r"produce the same checksum \((\d+)\)", readme)
    out = {
        "source": "reference main.swift PackedNumericCase list and README MXFP4 checksum",
        "roundtrip_tolerance": float(tol),
        "roundtrip_cases": cases,
        "mxfp4_mlp_checksum": {"tokens": 128, "hidden": 1024, "intermediate": 4096,
                               "value": cks.group(1) + " over 32 samples",
                               "rows": ["mxfp4_native_sp_h_f_n64", "mxfp4_native_sp_h_f_n128",
                                        "mxfp4_native_sph_h_f_n64", "mxfp4_fused_ci_h_f_sg_k64",
                                        "mxfp4_fused_ci_h_f_sg_k32"]},
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
