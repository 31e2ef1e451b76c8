"""Property checks of the oracle's quantizers (CPU, hypothesis): MXFP4 and
NVFP4 round trips stay within half a code step of the input, re-quantizing a
decoded tensor is the identity, and scaling a block by a power of two moves
only its MXFP4 scale byte."""
import numpy as np
from hypothesis import given, settings, strategies as st

import oracle as O

E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6])


def _half_step(a):
    """Largest distance of |a| (in code units) to its nearest E2M1 neighbours / 2."""
    idx = np.clip(np.searchsorted(E2M1, a), 1, 7)
    return (E2M1[idx] - E2M1[idx - 1]) / 2


blocks = st.lists(st.floats(-1e3, 1e3, allow_nan=False, width=32), min_size=32, max_size=32)


@settings(max_examples=60, deadline=None)
@given(st.lists(blocks, min_size=1, max_size=4))
def test_mxfp4_round_trip_bound_and_idempotence(rows):
    w = np.array(rows, np.float32)
    q, s = O.quantize_mxfp4(w)
    d = O.decode_weights(O.W_MXFP4, q, s, w.shape[0], 32)
    scale = np.ldexp(1.0, s.astype(np.int64) - 127)[:, :1]
    a = np.minimum(np.abs(w) / scale, 6.0)
    assert np.all(np.abs(d - w) <= (_half_step(a) + np.maximum(np.abs(w) / scale - 6.0, 0)) * scale + 1e-30)
    q2, s2 = O.quantize_mxfp4(d.astype(np.float32))
    assert np.array_equal(O.decode_weights(O.W_MXFP4, q2, s2, w.shape[0], 32), d)


@settings(max_examples=40, deadline=None)
@given(blocks, st.integers(-20, 20))
def test_mxfp4_power_of_two_scaling_moves_only_the_scale(block, e):
    w = np.array([block], np.float32)
    if np.abs(w).max() < 1e-20:
        return
    q, s = O.quantize_mxfp4(w)
    q2, s2 = O.quantize_mxfp4(np.ldexp(w, e).astype(np.float32))
    code = int(s[0, 0]) + e
    if 0 < code < 254 and 0 < int(s[0, 0]) < 254:
        assert int(s2[0, 0]) == code and np.array_equal(q2, q)


@settings(max_examples=40, deadline=None)
@given(st.lists(st.floats(-50, 50, allow_nan=False, width=32), min_size=64, max_size=64))
def test_nvfp4_round_trip_bound(vals):
    w = np.array([vals], np.float32)
    q, s, ts = O.quantize_nvfp4(w)
    d = O.decode_nvfp4(q, s, ts, 1, 64)
    amax = np.abs(w).max()
    # each block: at most half an E2M1 step of its decoded scale, plus the UE4M3 rounding of the scale
    # (relative 2^-4) applied to a value of at most 6 code units
    for b in range(4):
        blk = slice(16 * b, 16 * b + 16)
        sc = float(O.lib().orc_e4m3_decode(int(s[0, b]))) * ts
        if sc == 0:
            assert np.all(d[0, blk] == 0)
            continue
        a = np.minimum(np.abs(w[0, blk]) / sc, 6.0)
        over = np.maximum(np.abs(w[0, blk]) / sc - 6.0, 0)
        assert np.all(np.abs(d[0, blk] - w[0, blk]) <= (_half_step(a) + over) * sc + 1e-6 * (amax + 1))
