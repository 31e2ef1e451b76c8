"""BASELINE config 2's scaled weight rows on the GPU against the FP64 oracle:
INT8 / INT4 / INT2 weights with a per-output-channel fp16 scale
(MPP41_MLP_ROW_SCALES) and FP8 E4M3 / E5M2 weights with an E8M0 scale per 32
along K (MPP41_W_E4M3_MX / MPP41_W_E5M2_MX), at tokens=128, hidden=1024,
intermediate=4096 (and other token counts) with x ~ N(0,1) fp16 and weights
quantized from N(0, 0.02), as config 0. The reference runs these formats
unscaled only (MPPMLPKernels.metal:50-60, 72-82, 94-138); the scaled rows have
no reference counterpart and are pinned by the oracle restatement.

Tolerance: relative Frobenius error <= 1e-3 against the oracle of the same
quantized weights (north_star allows 1e-2). The error of each quantized layer
against the unquantized fp32 layer is printed."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-3


def config2_inputs(wfmt, T, H, I, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    out = {"x": x, "f32": {}}
    for name, (r, c) in (("g", (I, H)), ("u", (I, H)), ("d", (H, I))):
        w = (rng.standard_normal((r, c), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        out["f32"][name] = w
        if wfmt in (O.W_I8, O.W_I4, O.W_I2):
            out["w" + name], out["s" + name] = O.quantize_int_rowscale(w, wfmt)
        else:
            out["w" + name], out["s" + name] = O.quantize_mxfp8(w, e5m2=(wfmt == O.W_E5M2_MX))
    return out


def fp32_layer(x, f):
    xf = x.astype(np.float64)
    g, u = xf @ f["g"].T.astype(np.float64), xf @ f["u"].T.astype(np.float64)
    mid = (g / (1.0 + np.exp(-g)) * u).astype(np.float16).astype(np.float64)
    return mid @ f["d"].T.astype(np.float64)


@pytest.mark.parametrize("wfmt", [O.W_I8, O.W_I4, O.W_I2, O.W_E4M3_MX, O.W_E5M2_MX])
@pytest.mark.parametrize("T", [128, 77])
def test_config2_scaled_rows(ctx, wfmt, T):
    H, I = 1024, 4096
    d = config2_inputs(wfmt, T, H, I, seed=100 + wfmt + T)
    row = wfmt in (O.W_I8, O.W_I4, O.W_I2)
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16,
                          mpp41.MLP_ROW_SCALES if row else 0)
    dv = {k: to_dev(d[k]) for k in ("x", "wg", "wu", "wd", "sg", "su", "sd")}
    out, scr = empty_dev(T * H * 2), empty_dev(mpp41.scratch_bytes(desc))
    for _ in range(2):   # counters and workspace reused
        ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], scr, out)
    ctx.synchronize()
    assert ctx.mlp_last_kernel() == "small"
    got = from_dev(out, np.float16, (T, H))
    _, ref = O.mlp(0, wfmt, 4, 1, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"], row_scales=row)
    assert np.isfinite(got).all()
    assert rel_fro(got, ref) <= TOL
    print(f"wfmt {wfmt} T {T}: vs oracle {rel_fro(got, ref):.2e}, "
          f"quantized layer vs fp32 layer {rel_fro(got, fp32_layer(d['x'], d['f32'])):.3e}")


@pytest.mark.parametrize("wfmt", [O.W_I8, O.W_I2, O.W_E4M3, O.W_E5M2])
def test_unscaled_8bit_and_2bit_rows_take_the_small_kernel(ctx, wfmt):
    """The reference's unscaled INT8 / INT2 / FP8 rows at the config-2 shape run
    on the small-layer kernel too (reference seeds, half SwiGLU, fp32 out)."""
    from gpu_data import activations, weights
    T, H, I = 128, 1024, 4096
    x = activations(T, H)
    wg, _ = weights(wfmt, I, H, 0xABCD1357)
    wu, _ = weights(wfmt, I, H, 0x2468BDF0)
    wd, _ = weights(wfmt, H, I, 0x0BADCAFE)
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_HALF, mpp41.F32)
    out, scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, to_dev(x), to_dev(wg), to_dev(wu), to_dev(wd), None, None, None, scr, out)
    ctx.synchronize()
    assert ctx.mlp_last_kernel() == "small"
    _, ref = O.mlp(0, wfmt, 1, 0, T, H, I, x.view(np.uint16), wg, wu, wd)
    got = from_dev(out, np.float32, (T, H))
    fin = np.isfinite(ref)
    assert rel_fro(got[fin], ref[fin]) <= TOL


def test_scaled_rows_reject_shapes_outside_the_small_kernel(ctx):
    buf = empty_dev(16)
    desc = mpp41.mlp_desc(256, 1024, 4096, O.W_E4M3_MX, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    with pytest.raises(mpp41.MPP41Error) as e:
        ctx.mlp(desc, buf, buf, buf, buf, buf, buf, buf, buf, buf)
    assert e.value.status == mpp41.ERR_UNSUPPORTED_SHAPE
    desc = mpp41.mlp_desc(128, 1024, 4096, O.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16,
                          mpp41.MLP_ROW_SCALES)
    with pytest.raises(mpp41.MPP41Error) as e:
        ctx.mlp(desc, buf, buf, buf, buf, buf, buf, buf, buf, buf)
    assert e.value.status == mpp41.ERR_INVALID_ARGUMENT
