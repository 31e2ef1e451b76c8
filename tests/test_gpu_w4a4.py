"""W4A4 (activations and weights MXFP4, kind::mxf4 block-scaled MMA) against
the oracle.

- The GEMM is bit-exact when every partial sum is representable in fp32
  (scales 2^-1..2^1, K <= 1536), and within 1e-5 of sum |a||b| otherwise.
- The layer: x's quantization is bit-exact; the mid's quantization matches
  the oracle's on all but a few elements (silu in fp32 hardware exp versus
  fp64 can move a value across an E2M1 rounding boundary: at most one E2M1
  step, at most 0.2 % of elements); the down GEMM on the kernel's own mid
  matches fp64 within 1e-5 relative to the row scale.
- The W4A4 error against the unquantized-activation layer is reported as a
  separate number, bounded loosely (MXFP4 activations lose about 2-3 bits).
"""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu


def _rand_mx(rng, rows, K, lo=126, hi=128):
    packed = rng.integers(0, 256, (rows, K // 2), dtype=np.uint8)
    scales = rng.integers(lo, hi + 1, (rows, K // 32), dtype=np.uint8)
    return packed, scales


def _layer(T, H, I, seed):
    d = O.baseline_mlp_inputs(T, H, I, seed=seed)
    return d["x"], d["wg"], d["wu"], d["wd"], d["sg"], d["su"], d["sd"]


# ragged row tiles (200, 300) and several full row tiles (1024)
@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (200, 96, 1536), (1, 512, 1024), (300, 544, 512), (1024, 768, 2048)])
def test_mxf4_gemm_bit_exact(ctx, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    a, sa = _rand_mx(rng, M, K)
    b, sb = _rand_mx(rng, N, K)
    c = empty_dev(M * N * 4)
    ctx.matmul_mxf4(to_dev(a), to_dev(sa), to_dev(b), to_dev(sb), c, M, N, K)
    got = from_dev(c, np.float32, (M, N)).astype(np.float64)
    ref = O.decode_weights(O.W_MXFP4, a, sa, M, K) @ O.decode_weights(O.W_MXFP4, b, sb, N, K).T
    assert np.array_equal(got, ref)


def test_mxf4_gemm_wide_scales_f16(ctx):
    M, N, K = 256, 512, 4096
    rng = np.random.default_rng(5)
    a, sa = _rand_mx(rng, M, K, 110, 140)
    b, sb = _rand_mx(rng, N, K, 110, 140)
    c32, c16 = empty_dev(M * N * 4), empty_dev(M * N * 2)
    da, dsa, db, dsb = to_dev(a), to_dev(sa), to_dev(b), to_dev(sb)
    ctx.matmul_mxf4(da, dsa, db, dsb, c32, M, N, K)
    ctx.matmul_mxf4(da, dsa, db, dsb, c16, M, N, K, c_f16=True)
    ref = O.decode_weights(O.W_MXFP4, a, sa, M, K) @ O.decode_weights(O.W_MXFP4, b, sb, N, K).T
    absref = np.abs(O.decode_weights(O.W_MXFP4, a, sa, M, K)) @ np.abs(O.decode_weights(O.W_MXFP4, b, sb, N, K)).T
    got = from_dev(c32, np.float32, (M, N)).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absref + 1e-30)
    h = from_dev(c16, np.float16, (M, N))
    with np.errstate(over="ignore"):   # out-of-range sums saturate to inf on both sides
        assert np.array_equal(h, got.astype(np.float32).astype(np.float16))


def test_mxf4_gemm_rejects_bad_shapes(ctx):
    import mpp41
    d = empty_dev(1 << 16)
    with pytest.raises(mpp41.MPP41Error):
        ctx.matmul_mxf4(d, d, d, d, d, 128, 256, 256)   # K % 512
    with pytest.raises(mpp41.MPP41Error):
        ctx.matmul_mxf4(d, d, d, d, d, 128, 100, 512)   # N % 32


@pytest.mark.parametrize("T,H,I", [(128, 1024, 4096), (77, 512, 1024), (1, 1024, 512), (384, 1024, 1024)])
def test_w4a4_mlp(ctx, T, H, I):
    import mpp41
    x, wg, wu, wd, sg, su, sd = _layer(T, H, I, seed=T + H)
    scratch = empty_dev(mpp41.w4a4_scratch_bytes(T, H, I))
    out = empty_dev(T * H * 4)
    ctx.mlp_w4a4(T, H, I, to_dev(x), to_dev(wg), to_dev(sg), to_dev(wu), to_dev(su), to_dev(wd), to_dev(sd), out,
                 scratch)
    ctx.synchronize()
    xq, xs, mq, ms, ref_out = O.w4a4_mlp(x, wg, sg, wu, su, wd, sd)
    raw = from_dev(scratch, np.uint8, (scratch.numel(),))
    o0, o1, o2, o3 = mpp41.w4a4_scratch_layout(T, H, I)
    assert np.array_equal(raw[o0:o0 + T * H // 2].reshape(T, H // 2), xq)
    assert np.array_equal(raw[o1:o1 + T * H // 32].reshape(T, H // 32), xs)
    g_mq = raw[o2:o2 + T * I // 2].reshape(T, I // 2)
    g_ms = raw[o3:o3 + T * I // 32].reshape(T, I // 32)
    gm = O.decode_weights(O.W_MXFP4, g_mq, g_ms, T, I)
    rm = O.decode_weights(O.W_MXFP4, mq, ms, T, I)
    diff = gm != rm
    assert diff.mean() <= 2e-3
    # a flipped rounding moves one element by at most one E2M1 step (2 units of the block's scale)
    blk_scale = np.repeat(np.ldexp(1.0, ms.astype(np.int64) - 127), 32, axis=1)
    assert np.all(np.abs(gm - rm) <= 2.0 * blk_scale + 1e-30)
    got = from_dev(out, np.float32, (T, H)).astype(np.float64)
    own = gm @ O.decode_weights(O.W_MXFP4, wd, sd, H, I).T
    row = np.abs(own).max(axis=1, keepdims=True) + 1e-30
    assert np.all(np.abs(got - own) <= 1e-5 * row)
    # end to end against the oracle (including its own mid), loosely
    assert np.abs(got - ref_out).max() <= 0.05 * np.abs(ref_out).max()


def test_w4a4_error_vs_w4a16(ctx):
    """The cost of quantizing activations, as a number: relative Frobenius error
    of the W4A4 layer against the exact fp16-activation (W4A16) layer."""
    import mpp41
    T, H, I = 128, 1024, 4096
    x, wg, wu, wd, sg, su, sd = _layer(T, H, I, seed=0)
    scratch = empty_dev(mpp41.w4a4_scratch_bytes(T, H, I))
    out = empty_dev(T * H * 4)
    ctx.mlp_w4a4(T, H, I, to_dev(x), to_dev(wg), to_dev(sg), to_dev(wu), to_dev(su), to_dev(wd), to_dev(sd), out,
                 scratch)
    got = from_dev(out, np.float32, (T, H)).astype(np.float64)
    xd = x.astype(np.float64)
    g = xd @ O.decode_weights(O.W_MXFP4, wg, sg, I, H).T
    u = xd @ O.decode_weights(O.W_MXFP4, wu, su, I, H).T
    exact = (g / (1.0 + np.exp(-g)) * u) @ O.decode_weights(O.W_MXFP4, wd, sd, H, I).T
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    print(f"W4A4 relative error vs W4A16 (fp64): {rel:.4f}")
    assert rel < 0.3
