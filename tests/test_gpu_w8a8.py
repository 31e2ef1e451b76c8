"""Scaled integer layers (W8A8 / W4A8 / W2A8) against the oracle:
- per-row symmetric weight quantization bit-exact (packed bytes and fp32 scales);
- per-token x quantization bit-exact;
- fp16 mid within two fp16 ulps of the fp32 dequant + SwiGLU computed from the
  exact int32 sums (the kernel's silu uses the hardware exp);
- the mid's quantization and the dequantized down GEMM bit-exact given the
  kernel's own fp16 mid (int32 sums are exact, dequant is two fp32 products).
"""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu

BITS = {1: 8, 2: 4, 3: 2}   # MPP41_W_I8 / I4 / I2


@pytest.mark.parametrize("wfmt", [1, 2, 3])
def test_quantize_weights_int(ctx, wfmt):
    bits = BITS[wfmt]
    rng = np.random.default_rng(bits)
    w = (rng.standard_normal((96, 512)) * rng.choice([0.01, 1.0], (96, 1))).astype(np.float32)
    w[3] = 0
    d_p, d_s = empty_dev(96 * 512 * bits // 8), empty_dev(96 * 4)
    ctx.quantize_weights_int(to_dev(w), 96, 512, bits, d_p, d_s)
    pk, sc = O.quantize_int_rows(w, bits)
    assert np.array_equal(from_dev(d_s, np.float32, sc.shape), sc)
    assert np.array_equal(from_dev(d_p, np.uint8, pk.shape), pk)


@pytest.mark.parametrize("wfmt,T,H,I", [(1, 128, 1024, 4096), (2, 77, 512, 1024), (3, 200, 1024, 512), (1, 1, 256, 256)])
def test_mlp_w8a8(ctx, wfmt, T, H, I):
    import mpp41
    bits = BITS[wfmt]
    rng = np.random.default_rng(T + wfmt)
    x = rng.standard_normal((T, H)).astype(np.float16)
    ws = [(rng.standard_normal((r, c)) * 0.05).astype(np.float32) for r, c in ((I, H), (I, H), (H, I))]
    q = [O.quantize_int_rows(w, bits) for w in ws]
    (wg, sg), (wu, su), (wd, sd) = q
    scratch = empty_dev(mpp41.w8a8_scratch_bytes(T, H, I))
    out = empty_dev(T * H * 2)
    ctx.mlp_w8a8(wfmt, T, H, I, to_dev(x), to_dev(wg), to_dev(sg), to_dev(wu), to_dev(su), to_dev(wd), to_dev(sd),
                 out, scratch)
    ctx.synchronize()
    raw = from_dev(scratch, np.uint8, (scratch.numel(),))
    o_xq, o_xs, o_mid, o_mq, o_ms = mpp41.w8a8_scratch_layout(T, H, I)
    xq, xs = O.quantize_act_s8(x)
    assert np.array_equal(raw[o_xq:o_xq + T * H].view(np.int8).reshape(T, H), xq)
    assert np.array_equal(raw[o_xs:o_xs + T * 4].view(np.float32), xs)
    dec = lambda p, r, c: O.decode_weights(wfmt, p, None, r, c).astype(np.int64)
    g = xq.astype(np.int64) @ dec(wg, I, H).T
    u = xq.astype(np.int64) @ dec(wu, I, H).T
    gf = (g.astype(np.float32) * xs[:, None]) * sg[None, :]
    uf = (u.astype(np.float32) * xs[:, None]) * su[None, :]
    mid_ref = (gf.astype(np.float64) / (1 + np.exp(-gf.astype(np.float64))) * uf).astype(np.float16)
    mid = raw[o_mid:o_mid + T * I * 2].view(np.float16).reshape(T, I)
    m64, r64 = mid.astype(np.float64), mid_ref.astype(np.float64)
    assert np.all(np.abs(m64 - r64) <= 2 * np.abs(r64) * 2.0 ** -10 + 1e-7)
    mq, ms = O.quantize_act_s8(mid)
    assert np.array_equal(raw[o_mq:o_mq + T * I].view(np.int8).reshape(T, I), mq)
    assert np.array_equal(raw[o_ms:o_ms + T * 4].view(np.float32), ms)
    acc = mq.astype(np.int64) @ dec(wd, H, I).T
    ref = ((acc.astype(np.float32) * ms[:, None]) * sd[None, :]).astype(np.float16)
    assert np.array_equal(from_dev(out, np.float16, (T, H)), ref)
