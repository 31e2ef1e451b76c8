"""The weight-major layer kernel in its CTA-pair form (tcgen05 cta_group::2:
two CTAs of a cluster run one M = 256 MMA, each holding 128 weight rows and
half of the token tile): chosen for MXFP4 layers with full 128-token tiles
when MPP41_FUSED_PAIR=1. The output must match the FP64 oracle like every
other layer kernel (relative Frobenius <= 1e-3) and the single-CTA form of
the same kernel to within fp32 summation order (a one-ulp move of some fp16
values)."""
import os

import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import rel_fro

pytestmark = pytest.mark.gpu


def layer(ctx, out_f16, T, H, I, pair):
    wfmt = mpp41.W_MXFP4
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16 if out_f16 else mpp41.F32)
    d = O.baseline_mlp_inputs(T, H, I, seed=T + H)   # x ~ N(0,1), W ~ N(0,0.02) quantized MXFP4
    x, wg, wu, wd, sg, su, sd = (d[k] for k in ("x", "wg", "wu", "wd", "sg", "su", "sd"))
    out_dt = np.float16 if out_f16 else np.float32
    d_out = empty_dev(T * H * np.dtype(out_dt).itemsize)
    d_scr = empty_dev(mpp41.scratch_bytes(desc))
    dv = [to_dev(a) for a in (x, wg, wu, wd, sg, su, sd)]
    old = os.environ.get("MPP41_FUSED_PAIR")
    os.environ["MPP41_FUSED_PAIR"] = "1" if pair else "0"
    try:
        for _ in range(2):   # a second call reuses the self-resetting counters
            ctx.mlp(desc, *dv, d_scr, d_out)
        ctx.synchronize()
    finally:
        if old is None:
            os.environ.pop("MPP41_FUSED_PAIR", None)
        else:
            os.environ["MPP41_FUSED_PAIR"] = old
    kernel = ctx.mlp_last_kernel()
    got = from_dev(d_out, out_dt, (T, H)).astype(np.float32)
    # epilogue 4: SwiGLU on the fp32 sums, fp16 mid (MPP41_SWIGLU_FP32)
    _, ref = O.mlp(0, O.W_MXFP4, 4, 1 if out_f16 else 0, T, H, I,
                   x.view(np.uint16), wg, wu, wd, sg, su, sd)
    return kernel, got, ref


@pytest.mark.parametrize("out_f16", [True, False])
@pytest.mark.parametrize("T,H,I", [(256, 1024, 4096), (300, 512, 2048), (1024, 2048, 1024)])
def test_pair_matches_oracle_and_single(ctx, out_f16, T, H, I):
    k1, one, ref = layer(ctx, out_f16, T, H, I, pair=False)
    k2, two, _ = layer(ctx, out_f16, T, H, I, pair=True)
    assert k1 == k2 == "weight_major"
    assert np.isfinite(ref).all()
    assert rel_fro(two, ref) <= 1e-3
    # same products; the M = 256 MMA may order the fp32 sums differently, which
    # can move an fp16 mid or output value by one ulp
    assert rel_fro(two, one) <= 2e-4
