"""Activation quantization epilogue kernels against their definitions:
fp16 -> MXFP4 equals the oracle's OCP-MX quantizer bit for bit (fp16 is exact
in fp32); per-token int8 matches q = rint(x * 127 / absmax) computed in fp32."""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H", [(128, 1024), (3, 4096), (1, 32)])
def test_act_mxfp4_bit_exact(ctx, T, H):
    x = (np.random.default_rng(T + H).standard_normal((T, H)) * 3).astype(np.float16)
    x[0, :32] = 0
    d_p, d_s = empty_dev(T * H // 2), empty_dev(T * H // 32)
    ctx.quantize_act_mxfp4(to_dev(x), T, H, d_p, d_s)
    ctx.synchronize()
    pk, sc = O.quantize_mxfp4(x.astype(np.float32))
    assert np.array_equal(from_dev(d_p, np.uint8, pk.shape), pk)
    assert np.array_equal(from_dev(d_s, np.uint8, sc.shape), sc)


@pytest.mark.parametrize("T,H", [(128, 1024), (7, 4096), (2, 100)])
def test_act_s8_per_token(ctx, T, H):
    x = (np.random.default_rng(T * H).standard_normal((T, H)) * 2).astype(np.float16)
    x[-1] = 0
    d_q, d_s = empty_dev(T * H), empty_dev(T * 4)
    ctx.quantize_act_s8(to_dev(x), T, H, d_q, d_s)
    ctx.synchronize()
    xf = x.astype(np.float32)
    amax = np.abs(xf).max(axis=1)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    q = np.rint(np.clip(xf * inv[:, None], -127, 127)).astype(np.int8)
    assert np.array_equal(from_dev(d_q, np.int8, (T, H)), q)
    assert np.array_equal(from_dev(d_s, np.float32, (T,)), (amax / np.float32(127)).astype(np.float32))
