"""The reference's scalar half-accumulate rows (PackedNumericKernels.metal:
98-832) through mpp41_matmul_scalar / mpp41_mlp_scalar, bit for bit against
the oracle's restatement (serial fused half fma, one rounding each)."""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu

MM = [("fp4_e2m1_matmul_benchmark", 0), ("fp4_e2m1_matmul_g8_benchmark", 0),
      ("half_fp4_matmul_half_benchmark", 1), ("half_fp4_matmul_half_g8_benchmark", 1),
      ("half_int4_matmul_half_benchmark", 2), ("int8_half_matmul_half_benchmark", 3),
      ("int4_int8_matmul_benchmark", 4)]


@pytest.mark.parametrize("kernel,kind", MM)
def test_scalar_matmul_bit_exact(ctx, kernel, kind):
    M, N, K = 64, 96, 256
    s = O.MATMUL_SEEDS
    if kind in (0, 4):
        a = O.packed_bytes(M * K // 2, s["a_packed"])
    elif kind in (1, 2):
        a = O.half_values(M * K, s["a_half"]).view(np.uint16)
    else:
        a = O.int8_values(M * K, s["a_int8"])
    b = O.half_values(N * K, s["b_half"], 0.03125).view(np.uint16) if kind == 3 else O.packed_bytes(N * K // 2, s["b_packed"])
    ref = O.scalar_matmul(kind, M, N, K, a, b)
    d_c = empty_dev(ref.nbytes)
    ctx.matmul_scalar(kernel, to_dev(a), to_dev(b), d_c, M, N, K)
    got = from_dev(d_c, ref.dtype, ref.shape)
    assert np.array_equal(got.view(np.uint8), np.ascontiguousarray(ref).view(np.uint8))


SCALAR_MLP = [("half_mlp_gate_up_benchmark", "half_mlp_down_benchmark", O.W_F16),
              ("half_int8_mlp_gate_up_benchmark", "half_int8_mlp_down_benchmark", O.W_I8),
              ("half_int4_mlp_gate_up_benchmark", "half_int4_mlp_down_benchmark", O.W_I4),
              ("half_int2_mlp_gate_up_benchmark", "half_int2_mlp_down_benchmark", O.W_I2),
              ("half_fp4_mlp_gate_up_benchmark", "half_fp4_mlp_down_benchmark", O.W_FP4),
              ("half_fp4_mlp_gate_up_g8_benchmark", "half_fp4_mlp_down_g8_benchmark", O.W_FP4)]


@pytest.mark.parametrize("gk,dk,wfmt", SCALAR_MLP)
def test_scalar_mlp_bit_exact(ctx, gk, dk, wfmt):
    from gpu_data import weights
    T, H, I = 32, 128, 256
    sd = O.MLP_SEEDS
    x = O.half_values(T * H, sd["x_half"], 0.125).view(np.uint16)
    wg, _ = weights(wfmt, I, H, 0x5555_6666)
    wu, _ = weights(wfmt, I, H, 0x7777_8888)
    wd, _ = weights(wfmt, H, I, 0x9999_AAAA)
    mid_ref, out_ref = O.scalar_mlp(wfmt, T, H, I, x, wg, wu, wd)
    d_mid, d_out = empty_dev(T * I * 2), empty_dev(T * H * 2)
    ctx.mlp_scalar(gk, dk, to_dev(x), to_dev(wg), to_dev(wu), d_mid, to_dev(wd), d_out, T, H, I)
    assert np.array_equal(from_dev(d_mid, np.uint16, (T, I)), mid_ref.view(np.uint16))
    assert np.array_equal(from_dev(d_out, np.uint16, (T, H)), out_ref.view(np.uint16))
