"""Tensor-core formulation of the big-matmul rows (mpp41_matmul), BASELINE
config 1: FP4 x FP4 -> fp32 and INT4 x INT4 -> int32 are exact (every partial
sum is representable), so they must equal the FP64 product bit for bit, also
at the full 2048^3 size; the half-output rows are the exactly rounded sum to
within one fp16 ulp (fp32 accumulation, one rounding)."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu

MM = [("fp4_e2m1_matmul_benchmark", 0), ("fp4_e2m1_matmul_g8_benchmark", 0),
      ("half_fp4_matmul_half_benchmark", 1), ("half_fp4_matmul_half_g8_benchmark", 1),
      ("half_int4_matmul_half_benchmark", 2), ("int8_half_matmul_half_benchmark", 3),
      ("int4_int8_matmul_benchmark", 4)]


def operands(kind, M, N, K):
    s = O.MATMUL_SEEDS
    if kind in (0, 4):
        a = O.packed_bytes(M * K // 2, s["a_packed"]).reshape(M, K // 2)
        ad = O.decode_weights(O.W_FP4 if kind == 0 else O.W_I4, a, None, M, K)
    elif kind in (1, 2):
        a = O.half_values(M * K, s["a_half"]).reshape(M, K)
        ad = a.astype(np.float64)
    else:
        a = O.int8_values(M * K, s["a_int8"]).reshape(M, K)
        ad = a.astype(np.float64)
    if kind == 3:
        b = O.half_values(N * K, s["b_half"], 0.03125).reshape(N, K)
        bd = b.astype(np.float64)
    else:
        b = O.packed_bytes(N * K // 2, s["b_packed"]).reshape(N, K // 2)
        bd = O.decode_weights({0: O.W_FP4, 1: O.W_FP4, 2: O.W_I4, 4: O.W_I4}[kind], b, None, N, K)
    return a, b, ad @ bd.T


def run(ctx, kernel, kind, M, N, K):
    a, b, ref = operands(kind, M, N, K)
    out_dt = {0: np.float32, 4: np.int32}.get(kind, np.float16)
    d_c = empty_dev(M * N * np.dtype(out_dt).itemsize)
    wsb = mpp41.Context.matmul_workspace_bytes(kernel, M, N, K)
    ws = empty_dev(wsb) if wsb else None
    ctx.matmul(kernel, to_dev(a), to_dev(b), d_c, M, N, K, ws)
    ctx.synchronize()
    return from_dev(d_c, out_dt, (M, N)), ref


@pytest.mark.parametrize("kernel,kind", MM)
@pytest.mark.parametrize("M,N,K", [(256, 192, 512), (100, 128, 1024)])
def test_tensor_matmul_rows(ctx, kernel, kind, M, N, K):
    got, ref = run(ctx, kernel, kind, M, N, K)
    if kind == 0:
        assert np.array_equal(got.astype(np.float64), ref)
    elif kind == 4:
        assert np.array_equal(got.astype(np.int64), ref.astype(np.int64))
    else:
        r16 = ref.astype(np.float16)
        fin = np.isfinite(r16)
        assert np.array_equal(np.isfinite(got), fin)
        ulp = np.abs(got[fin].view(np.int16).astype(np.int32) - r16[fin].view(np.int16).astype(np.int32))
        assert ulp.max() <= 1 and (ulp == 0).mean() > 0.99, kernel


@pytest.mark.parametrize("kernel,kind", [("fp4_e2m1_matmul_benchmark", 0), ("int4_int8_matmul_benchmark", 4)])
def test_exact_rows_at_2048_cubed(ctx, kernel, kind):
    got, ref = run(ctx, kernel, kind, 2048, 2048, 2048)
    assert np.array_equal(got.astype(np.float64), ref)
