"""int8-activation rows (W8A8 / W4A8 / W2A8) on tcgen05 kind::i8 through the C
ABI, against the oracle. Integer accumulation is exact, so GEMM outputs are
compared bit for bit; the MLP rows (gate/up -> mpp_mlp_swiglu_i8 -> down) use
exp in double on both sides and must also match exactly (mismatch count 0)."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import weights

pytestmark = pytest.mark.gpu

ROWS = [("mpp_mlp_i8_i8_i32_n128", O.W_I8), ("mpp_mlp_i8_i4_i32_n128", O.W_I4), ("mpp_mlp_i8_i2_i32_n128", O.W_I2)]


def int8_acts(m, k, seed):
    return np.random.default_rng(seed).integers(-128, 128, (m, k), dtype=np.int8)


@pytest.mark.parametrize("kernel,wfmt", ROWS)
@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (64, 128, 1024), (200, 192, 256), (1, 128, 4096)])
def test_int8_gemm_exact(ctx, kernel, wfmt, m, n, k):
    a = int8_acts(m, k, 0x1234 + m)
    w, _ = weights(wfmt, n, k, 0x5151 + n)
    d_c = empty_dev(m * n * 4)
    ctx.gemm(kernel, to_dev(a), to_dev(w), d_c, m, n, k, None)
    ctx.synchronize()
    got = from_dev(d_c, np.int32, (m, n))
    ref = (a.astype(np.float64) @ O.decode_weights(wfmt, w, None, n, k).T).astype(np.int64)
    assert np.array_equal(got.astype(np.int64), ref), kernel


@pytest.mark.parametrize("kernel,wfmt", ROWS)
@pytest.mark.parametrize("T,H,I", [(128, 256, 512), (128, 1024, 4096), (5, 512, 1024)])
def test_int8_mlp_rows_exact(ctx, kernel, wfmt, T, H, I):
    desc = mpp41.describe(kernel, T, H, I)
    assert desc.afmt == mpp41.A_S8 and desc.out_dtype == mpp41.S32
    x = O.int8_values(T * H, O.MLP_SEEDS["x_int8"]).reshape(T, H)
    wg, _ = weights(wfmt, I, H, 0x33334444)
    wu, _ = weights(wfmt, I, H, 0x44445555)
    wd, _ = weights(wfmt, H, I, 0x55557777)
    d_out, d_scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, to_dev(x), to_dev(wg), to_dev(wu), to_dev(wd), None, None, None, d_scr, d_out)
    ctx.synchronize()
    got = from_dev(d_out, np.int32, (T, H))
    mid = from_dev(d_scr, np.int8, (T, I))
    mid_ref, ref = O.mlp(1, wfmt, 3, 2, T, H, I, x, wg, wu, wd)
    assert int((mid != mid_ref).sum()) == 0, "int8 mid mismatches"
    assert np.array_equal(got, ref), "int32 output mismatches"


def test_int8_two_stage_matches_one_call(ctx):
    T, H, I = 128, 512, 1024
    desc = mpp41.describe("mpp_mlp_i8_i4_i32_n128", T, H, I)
    x = O.int8_values(T * H, 7).reshape(T, H)
    wg, _ = weights(O.W_I4, I, H, 1)
    wu, _ = weights(O.W_I4, I, H, 2)
    wd, _ = weights(O.W_I4, H, I, 3)
    dv = [to_dev(a) for a in (x, wg, wu, wd)]
    a_out, b_out = empty_dev(T * H * 4), empty_dev(T * H * 4)
    scr = empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, dv[0], dv[1], dv[2], dv[3], None, None, None, scr, a_out)
    ctx.mlp_gate_up(desc, dv[0], dv[1], dv[2], None, None, scr)
    ctx.mlp_down(desc, scr, dv[3], None, b_out, False)
    ctx.synchronize()
    assert np.array_equal(from_dev(a_out, np.int32, (T, H)), from_dev(b_out, np.int32, (T, H)))
