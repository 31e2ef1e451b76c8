"""Seeded operands for the GPU parity tests (reference generators, main.swift:2785-2842)."""
import numpy as np

import oracle as O

SCALE_PATTERN = O.MXFP4_SCALE_PATTERN
# E8M0 codes spanning the fp16-exact window and both slow paths of the decoder
WIDE_SCALES = bytes(range(90, 150)) + bytes([0, 1, 60, 200])


def weights(wfmt: int, n: int, k: int, seed: int, wide_scales: bool = False):
    """Packed weight bytes [n][...] and (for MXFP4) scales [n][k/32]."""
    if wfmt == O.W_F16:
        w = O.half_values(n * k, seed, 1.0 / 64).view(np.uint16).reshape(n, k)
    elif wfmt == O.W_I8:
        w = O.int8_values(n * k, seed).reshape(n, k)
    elif wfmt in (O.W_I4, O.W_FP4, O.W_MXFP4):
        w = O.packed_bytes(n * k // 2, seed).reshape(n, k // 2)
    elif wfmt == O.W_I2:
        w = O.packed_bytes(n * k // 4, seed).reshape(n, k // 4)
    else:
        w = O.fp8_bytes(n * k, seed, e5m2=(wfmt == O.W_E5M2)).reshape(n, k)
    s = None
    if wfmt == O.W_MXFP4:
        s = O.pattern_bytes(n * k // 32, seed ^ 0x5A5A5A5A, WIDE_SCALES if wide_scales else SCALE_PATTERN)
        s = s.reshape(n, k // 32)
    return w, s


def activations(m: int, k: int, seed: int = 0x11112222, scale: float = 0.125):
    return O.half_values(m * k, seed, scale).reshape(m, k)


def rel_fro(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(got - ref) / (den if den > 0 else 1.0))
