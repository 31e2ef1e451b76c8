"""Tensor-core GEMM rows through the C ABI (mpp41_gemm by reference kernel
name) against the FP64 dequantize-then-matmul oracle.

The reference's matmul2d accumulates full width (README.md:342-347); ours
accumulates the exact fp16 x fp16 products in fp32 TMEM. Tolerance: relative
Frobenius error <= 1e-5 for fp32 outputs (north_star allows 1e-2), and one
final rounding for fp16 outputs."""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import activations, rel_fro, weights

pytestmark = pytest.mark.gpu

ROWS = [
    ("mpp_mlp_h_h_f_n128", O.W_F16),
    ("mpp_mlp_h_i8_f_n128", O.W_I8),
    ("mpp_mlp_h_i4_f_n128", O.W_I4),
    ("mpp_mlp_h_fp4_f_n128", O.W_FP4),
    ("mpp_mlp_h_fp8e4m3_f_n128", O.W_E4M3),
    ("mpp_mlp_h_fp8e5m2_f_n128", O.W_E5M2),
    ("mpp_mlp_h_i2_f_n128", O.W_I2),
    ("mxfp4_native_sp_h_f_n64", O.W_MXFP4),
    ("mxfp4_native_sp_h_f_n128", O.W_MXFP4),
    ("mxfp4_fused_h_f_n64", O.W_MXFP4),
    ("mxfp4_native_sph_h_f_n64", O.W_MXFP4),
    ("mxfp4_fused_ci_h_f_sg_k32", O.W_MXFP4),
]


def run_gemm(ctx, kernel, wfmt, m, n, k, out_dt=np.float32, wide=False, seed=0x13572468):
    a = activations(m, k)
    w, s = weights(wfmt, n, k, seed, wide_scales=wide)
    d_c = empty_dev(m * n * np.dtype(out_dt).itemsize)
    ctx.gemm(kernel, to_dev(a), to_dev(w), d_c, m, n, k, to_dev(s) if s is not None else None)
    ctx.synchronize()
    got = from_dev(d_c, out_dt, (m, n))
    ref = a.astype(np.float64) @ O.decode_weights(wfmt, w, s, n, k).T
    return got, ref


@pytest.mark.parametrize("kernel,wfmt", ROWS)
@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (64, 128, 1024), (200, 192, 256)])
def test_gemm_rows(ctx, kernel, wfmt, m, n, k):
    got, ref = run_gemm(ctx, kernel, wfmt, m, n, k)
    assert np.isfinite(got).all()
    assert rel_fro(got, ref) <= 1e-5, kernel


@pytest.mark.parametrize("m", [1, 16, 127, 129, 384])
def test_mxfp4_ragged_tokens(ctx, m):
    got, ref = run_gemm(ctx, "mxfp4_native_sp_h_f_n64", O.W_MXFP4, m, 256, 2048)
    assert rel_fro(got, ref) <= 1e-5


def test_mxfp4_scales_outside_fp16_window(ctx):
    """E8M0 codes where 2^(s-127) * E2M1 leaves the fp16-exact range take the
    fp32 decode path; compare against half(float(lut) * scale) then FP64."""
    m, n, k = 128, 128, 512
    a = activations(m, k)
    w, s = weights(O.W_MXFP4, n, k, 0x2468BDF0, wide_scales=True)
    d_c = empty_dev(m * n * 4)
    ctx.gemm("mxfp4_native_sp_h_f_n64", to_dev(a), to_dev(w), d_c, m, n, k, to_dev(s))
    ctx.synchronize()
    got = from_dev(d_c, np.float32, (m, n))
    wh = O.mxfp4_dequant_half(np.ascontiguousarray(w), np.ascontiguousarray(s), n, k).astype(np.float64)
    ref = a.astype(np.float64) @ wh.T
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    assert rel_fro(got[fin], ref[fin]) <= 1e-5


def test_fp8_half_destination_rounds_once(ctx):
    got, ref = run_gemm(ctx, "mpp_mlp_h_fp8e4m3_h_n128", O.W_E4M3, 128, 256, 512, out_dt=np.float16)
    want = ref.astype(np.float16)
    assert np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)) /
                  np.maximum(np.abs(want.astype(np.float64)), 1e-3)) <= 2 ** -10


def test_half_destination_overflows_to_inf(ctx):
    """README.md:342-356: a half destination overflows to inf past 65520 and
    never saturates; the fp32 accumulator itself stays exact."""
    m, n, k = 128, 128, 256
    a = np.full((m, k), 16.0, np.float16)
    w = np.full((n, k), 0x58, np.uint8)          # E4M3 0x58 = 16.0; 256 * 16 * 16 = 65536
    d_c = empty_dev(m * n * 2)
    ctx.gemm("mpp_mlp_h_fp8e4m3_h_n128", to_dev(a), to_dev(w), d_c, m, n, k)
    got = from_dev(d_c, np.float16, (m, n))
    assert np.all(np.isinf(got)) and np.all(got > 0)
    d_f = empty_dev(m * n * 4)
    ctx.gemm("mpp_mlp_h_fp8e4m3_f_n128", to_dev(a), to_dev(w), d_f, m, n, k)
    assert np.all(from_dev(d_f, np.float32, (m, n)) == 65536.0)


def test_unsupported_shape_is_reported(ctx):
    import mpp41
    d = empty_dev(1 << 16)
    with pytest.raises(mpp41.MPP41Error) as e:
        ctx.gemm("mpp_mlp_h_i4_f_n128", d, d, d, 64, 100, 512)
    assert e.value.status == mpp41.ERR_UNSUPPORTED_SHAPE
    with pytest.raises(mpp41.MPP41Error) as e:
        ctx.gemm("mxfp4_probe_noscale_h_f_n64", d, d, d, 64, 128, 512)
    assert e.value.status == mpp41.ERR_MISSING_KERNEL


@pytest.mark.parametrize("kernel,wfmt", [("mpp_mlp_f_h_f_n128", O.W_F16), ("mpp_mlp_f_i8_f_n128", O.W_I8)])
@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (64, 128, 4096), (200, 192, 256)])
def test_fp32_activation_rows(ctx, kernel, wfmt, m, n, k):
    """fp32 A (the swiglu_float mid) on kind::tf32 with A split into a tf32 head
    and its fp32 remainder: ~2^-21 relative per product, checked at 1e-5."""
    a = (np.random.default_rng(m + n).standard_normal((m, k)) * 0.5).astype(np.float32)
    w, _ = weights(wfmt, n, k, 0x7777 + k)
    d_c = empty_dev(m * n * 4)
    ctx.gemm(kernel, to_dev(a), to_dev(w), d_c, m, n, k, None)
    ctx.synchronize()
    got = from_dev(d_c, np.float32, (m, n))
    ref = a.astype(np.float64) @ O.decode_weights(wfmt, w, None, n, k).T
    assert rel_fro(got, ref) <= 1e-5, kernel


# README.md:342-352 accumulator semantics, as device tests: constant fills so
# every output element has the same exact integer value.
def _ones_gemm(ctx, kernel, wfmt_byte, k, zeros, out_dt):
    m = n = 128
    a = np.ones((m, k), np.float16)
    if wfmt_byte == "fp4":
        w = np.full((n, k // 2), 0x22, np.uint8)          # E2M1 nibble 0x2 = 1.0
        if zeros:
            w[:, :zeros // 2] = 0
    else:
        w = np.full((n, k), 0x38, np.uint8)               # E4M3 0x38 = 1.0
        w[:, :zeros] = 0
    d_c = empty_dev(m * n * np.dtype(out_dt).itemsize)
    ctx.gemm(kernel, to_dev(a), to_dev(w), d_c, m, n, k)
    return from_dev(d_c, out_dt, (m, n))


@pytest.mark.parametrize("kernel,fmt", [("mpp_mlp_h_fp8e4m3_f_n128", "e4m3"), ("mpp_mlp_h_fp4_f_n128", "fp4")])
def test_sum_of_ones_exact_through_131072_float_destination(ctx, kernel, fmt):
    got = _ones_gemm(ctx, kernel, fmt, 131072, 0, np.float32)
    assert np.all(got == 131072.0)


def test_sum_of_ones_exact_to_65504_half_destination(ctx):
    # K = 65536 with 32 zero weights: exact sum 65504, the largest finite half
    got = _ones_gemm(ctx, "mpp_mlp_h_fp8e4m3_h_n128", "e4m3", 65536, 32, np.float16)
    assert np.all(got.astype(np.float64) == 65504.0)


def test_half_destination_rounds_once_65448_to_65440(ctx):
    # K = 65472 with 24 zero weights: exact sum 65448, one rounding to half -> 65440
    got = _ones_gemm(ctx, "mpp_mlp_h_fp8e4m3_h_n128", "e4m3", 65472, 24, np.float16)
    assert np.all(got.astype(np.float64) == 65440.0)
