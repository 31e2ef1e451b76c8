"""NVFP4 (E2M1 + UE4M3 per 16 + fp32 tensor scale, kind::mxf4nvf4) against the
oracle:
- the quantizers (fp32 weights, fp16 activations) are bit-exact, tensor
  scale included;
- the GEMM is bit-exact when every partial sum is representable in fp32 (the
  tensor scales are powers of two and the block scales small), and within
  1e-5 of sum |a||b| otherwise;
- the layer: x's quantization bit-exact; the fp16 mid within fp16 rounding of
  the fp64 mid computed from the same quantized x (silu on hardware exp);
  the mid's NVFP4 quantization bit-exact given the kernel's own fp16 mid; the
  down GEMM within 1e-5 of the row scale.
"""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu


def _f32(v):
    return to_dev(np.array([v], np.float32))


@pytest.mark.parametrize("rows,depth", [(256, 1024), (3, 4096), (1, 16)])
def test_quantize_nvfp4_bit_exact(ctx, rows, depth):
    rng = np.random.default_rng(rows + depth)
    w = (rng.standard_normal((rows, depth)) * rng.choice([1e-3, 0.02, 3.0], (rows, 1))).astype(np.float32)
    if rows > 1:
        w[1, :16] = 0
    d_p, d_s, d_t = empty_dev(rows * depth // 2), empty_dev(rows * depth // 16), empty_dev(4)
    ctx.quantize_nvfp4(to_dev(w), rows, depth, d_p, d_s, d_t)
    pk, sc, ts = O.quantize_nvfp4(w)
    assert from_dev(d_t, np.float32, (1,))[0] == np.float32(ts)
    assert np.array_equal(from_dev(d_s, np.uint8, sc.shape), sc)
    assert np.array_equal(from_dev(d_p, np.uint8, pk.shape), pk)
    x16 = (rng.standard_normal((rows, depth)) * 4).astype(np.float16)
    ctx.quantize_act_nvfp4(to_dev(x16), rows, depth, d_p, d_s, d_t)
    pk, sc, ts = O.quantize_nvfp4(x16.astype(np.float32))
    assert from_dev(d_t, np.float32, (1,))[0] == np.float32(ts)
    assert np.array_equal(from_dev(d_s, np.uint8, sc.shape), sc)
    assert np.array_equal(from_dev(d_p, np.uint8, pk.shape), pk)


def _rand_nv(rng, rows, K, lo=None, hi=None):
    packed = rng.integers(0, 256, (rows, K // 2), dtype=np.uint8)
    if lo is None:   # UE4M3 0.5, 1, 2: every partial sum stays exact in fp32
        scales = rng.choice(np.array([0x30, 0x38, 0x40], np.uint8), (rows, K // 16))
    else:
        scales = rng.integers(lo, hi + 1, (rows, K // 16), dtype=np.uint8)
    return packed, scales


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (200, 96, 768), (1, 512, 1024), (640, 512, 1024)])
def test_nvf4_gemm_bit_exact(ctx, M, N, K):
    rng = np.random.default_rng(M + N * 3 + K)
    a, sa = _rand_nv(rng, M, K)
    b, sb = _rand_nv(rng, N, K)
    ta, tb = 0.5, 4.0
    c = empty_dev(M * N * 4)
    ctx.matmul_nvf4(to_dev(a), to_dev(sa), _f32(ta), to_dev(b), to_dev(sb), _f32(tb), c, M, N, K)
    got = from_dev(c, np.float32, (M, N)).astype(np.float64)
    ref = O.decode_nvfp4(a, sa, ta, M, K) @ O.decode_nvfp4(b, sb, tb, N, K).T
    assert np.array_equal(got, ref)


def test_nvf4_gemm_wide_scales(ctx):
    M, N, K = 256, 512, 4096
    rng = np.random.default_rng(9)
    a, sa = _rand_nv(rng, M, K, 0x01, 0x7E)   # subnormal .. 448
    b, sb = _rand_nv(rng, N, K, 0x01, 0x7E)
    ta, tb = 1.7e-3, 3.1e-2
    c32, c16 = empty_dev(M * N * 4), empty_dev(M * N * 2)
    args = (to_dev(a), to_dev(sa), _f32(ta), to_dev(b), to_dev(sb), _f32(tb))
    ctx.matmul_nvf4(*args, c32, M, N, K)
    ctx.matmul_nvf4(*args, c16, M, N, K, c_f16=True)
    da, db = O.decode_nvfp4(a, sa, ta, M, K), O.decode_nvfp4(b, sb, tb, N, K)
    ref, absref = da @ db.T, np.abs(da) @ np.abs(db).T
    got = from_dev(c32, np.float32, (M, N)).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * absref + 1e-30)
    h = from_dev(c16, np.float16, (M, N)).astype(np.float64)
    assert np.all(np.abs(h - ref) <= 1e-3 * np.abs(ref) + 1e-5 * absref + 6e-8)


def _weights(rng, rows, cols):
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    return O.quantize_nvfp4(w)


@pytest.mark.parametrize("T,H,I", [(128, 1024, 4096), (77, 512, 768), (300, 512, 512)])
def test_nvfp4_mlp(ctx, T, H, I):
    import mpp41
    rng = np.random.default_rng(T + I)
    x = rng.standard_normal((T, H)).astype(np.float16)
    (wg, sg, tg), (wu, su, tu), (wd, sd, td) = _weights(rng, I, H), _weights(rng, I, H), _weights(rng, H, I)
    scratch = empty_dev(mpp41.nvfp4_scratch_bytes(T, H, I))
    out = empty_dev(T * H * 4)
    ctx.mlp_nvfp4(T, H, I, to_dev(x), to_dev(wg), to_dev(sg), _f32(tg), to_dev(wu), to_dev(su), _f32(tu),
                  to_dev(wd), to_dev(sd), _f32(td), out, scratch)
    ctx.synchronize()
    xq, xs, tx, mid_ref, out_ref = O.nvfp4_mlp(x, wg, sg, tg, wu, su, tu, wd, sd, td)
    raw = from_dev(scratch, np.uint8, (scratch.numel(),))
    o_xq, o_xs, o_mid, o_mq, o_ms, o_ts = mpp41.nvfp4_scratch_layout(T, H, I)
    assert np.array_equal(raw[o_xq:o_xq + T * H // 2].reshape(T, H // 2), xq)
    assert np.array_equal(raw[o_xs:o_xs + T * H // 16].reshape(T, H // 16), xs)
    ts = raw[o_ts:o_ts + 8].view(np.float32)
    assert ts[0] == np.float32(tx)
    mid = raw[o_mid:o_mid + T * I * 2].view(np.float16).reshape(T, I)
    m64, r64 = mid.astype(np.float64), mid_ref.astype(np.float64)
    assert np.all(np.abs(m64 - r64) <= 2e-3 * np.abs(r64) + 1e-6 * np.abs(r64).max())
    mq, ms, tm = O.quantize_nvfp4(mid.astype(np.float32))
    assert ts[1] == np.float32(tm)
    assert np.array_equal(raw[o_mq:o_mq + T * I // 2].reshape(T, I // 2), mq)
    assert np.array_equal(raw[o_ms:o_ms + T * I // 16].reshape(T, I // 16), ms)
    got = from_dev(out, np.float32, (T, H)).astype(np.float64)
    own = O.decode_nvfp4(mq, ms, tm, T, I) @ O.decode_nvfp4(wd, sd, td, H, I).T
    row = np.abs(own).max(axis=1, keepdims=True) + 1e-30
    assert np.all(np.abs(got - own) <= 1e-5 * row)
    assert np.abs(got - out_ref).max() <= 0.05 * np.abs(out_ref).max()
