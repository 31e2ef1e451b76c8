"""BASELINE config 2's scaled weight rows on the CPU oracle (no GPU): the
per-row INT quantizer and the MXFP8 (E4M3 / E5M2 + E8M0 per 32) quantizer, the
MXFP8 decode rule half(value * 2^(scale - 127)) cross-checked against
ml_dtypes, and the row-scaled MLP restatement against the unscaled one."""
import ml_dtypes
import numpy as np
import pytest

import oracle as O


@pytest.mark.parametrize("wfmt", [O.W_I8, O.W_I4, O.W_I2])
def test_int_rowscale_quantizer_error_bound(wfmt):
    rng = np.random.default_rng(wfmt)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[5] = 0.0
    q, s = O.quantize_int_rowscale(w, wfmt)
    assert s.dtype == np.float16 and s.shape == (64,)
    deq = O.decode_weights(wfmt, q, None, 64, 256) * s.astype(np.float64)[:, None]
    qmax = O.INT_QMAX[wfmt]
    # every element within half a step, except the clipped top of the negative side
    step = s.astype(np.float64)[:, None]
    assert np.all(np.abs(deq - w) <= 0.5 * step * (1 + 1e-3) + np.abs(w) * 2e-3 / qmax + 1e-12)
    assert np.all(deq[5] == 0.0)


@pytest.mark.parametrize("e5m2", [False, True])
def test_mxfp8_decode_matches_ml_dtypes(e5m2):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0
    q, s = O.quantize_mxfp8(w, e5m2)
    wfmt = O.W_E5M2_MX if e5m2 else O.W_E4M3_MX
    got = O.decode_weights(wfmt, q, s, 32, 512)
    dt = ml_dtypes.float8_e5m2 if e5m2 else ml_dtypes.float8_e4m3fn
    elem = q.view(dt).astype(np.float64)
    scale = np.exp2(s.astype(np.float64) - 127.0)
    ref = (elem * np.repeat(scale, 32, axis=1)).astype(np.float16).astype(np.float64)
    assert np.array_equal(got, ref)
    # quantization error of the block-scaled elements (2 or 3 mantissa bits)
    rel = np.linalg.norm(got - w) / np.linalg.norm(w)
    assert rel < (0.1 if e5m2 else 0.05)


def test_row_scaled_mlp_with_unit_scales_equals_plain_row():
    rng = np.random.default_rng(3)
    T, H, I = 8, 64, 128
    x = (rng.standard_normal((T, H)) * 0.5).astype(np.float16)
    wg, wu, wd = (rng.integers(-4, 4, (r, c)).astype(np.int8) for r, c in ((I, H), (I, H), (H, I)))
    ones_i, ones_h = np.ones(I, np.float16), np.ones(H, np.float16)
    _, a = O.mlp(0, O.W_I8, 4, 0, T, H, I, x.view(np.uint16), wg, wu, wd)
    _, b = O.mlp(0, O.W_I8, 4, 0, T, H, I, x.view(np.uint16), wg, wu, wd, ones_i, ones_i, ones_h,
                 row_scales=True)
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)


def test_row_scaled_mlp_scales_each_row():
    rng = np.random.default_rng(4)
    T, H, I = 4, 64, 64
    x = (rng.standard_normal((T, H)) * 0.5).astype(np.float16)
    wg, wu, wd = (rng.integers(-8, 8, (r, c)).astype(np.int8) for r, c in ((I, H), (I, H), (H, I)))
    sd = np.full(H, 2.0, np.float16)
    ones = np.ones(I, np.float16)
    _, a = O.mlp(0, O.W_I8, 4, 0, T, H, I, x.view(np.uint16), wg, wu, wd, ones, ones, np.ones(H, np.float16),
                 row_scales=True)
    _, b = O.mlp(0, O.W_I8, 4, 0, T, H, I, x.view(np.uint16), wg, wu, wd, ones, ones, sd, row_scales=True)
    assert np.array_equal(2.0 * a, b)
