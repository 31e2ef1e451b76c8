"""The fused MLP hot path, down(swiglu(gate(x), up(x))), through mpp41_mlp
against the oracle.

Pins: the reference's published MXFP4 checksum 403573 at tokens=128,
hidden=1024, intermediate=4096 (README.md:292-295) in reference-seeded mode;
relative Frobenius error against the FP64 oracle <= 1e-3 for every row (the
north_star bound is 1e-2). The SwiGLU is evaluated with expf on the GPU and a
double exp on the CPU, so a few fp16 mid values may differ by one ulp."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import activations, rel_fro, weights

pytestmark = pytest.mark.gpu

TOL = 1e-3


def run_mlp(ctx, gate_kernel, T, H, I, wide=False, seeds=(0xABCD1357, 0x2468BDF0, 0x0BADCAFE)):
    desc = mpp41.describe(gate_kernel, T, H, I)
    x = activations(T, H)
    wg, sg = weights(desc.wfmt, I, H, seeds[0], wide)
    wu, su = weights(desc.wfmt, I, H, seeds[1], wide)
    wd, sd = weights(desc.wfmt, H, I, seeds[2], wide)
    out_dt = {mpp41.F32: np.float32, mpp41.F16: np.float16}[desc.out_dtype]
    d_out = empty_dev(T * H * np.dtype(out_dt).itemsize)
    d_scr = empty_dev(mpp41.scratch_bytes(desc))
    dv = [to_dev(a) if a is not None else None for a in (x, wg, wu, wd, sg, su, sd)]
    ctx.mlp(desc, *dv, d_scr, d_out)
    ctx.synchronize()
    got = from_dev(d_out, out_dt, (T, H))
    mid_ref, ref = O.mlp(0, desc.wfmt, desc.epilogue, {np.float32: 0, np.float16: 1}[out_dt], T, H, I,
                         x.view(np.uint16), wg, wu, wd, sg, su, sd)
    mid = from_dev(d_scr, mid_ref.dtype, (T, I))
    return got, ref, mid, mid_ref


def test_mxfp4_reference_checksum_403573(ctx, golden):
    g = golden["mxfp4_mlp_checksum"]
    T, H, I = g["tokens"], g["hidden"], g["intermediate"]
    d = O.reference_mlp_inputs(T, H, I)
    desc = mpp41.describe("mxfp4_native_sp_h_f_n64", T, H, I)
    d_out, d_scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, to_dev(d["x"]), to_dev(d["wg"]), to_dev(d["wu"]), to_dev(d["wd"]), to_dev(d["sg"]),
            to_dev(d["su"]), to_dev(d["sd"]), d_scr, d_out)
    ctx.synchronize()
    got = from_dev(d_out, np.float32, (T, H))
    assert O.float_checksum(got) == g["value"]
    _, ref = O.mlp(0, O.W_MXFP4, 1, 0, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"])
    assert rel_fro(got, ref) <= TOL


@pytest.mark.parametrize("gate_kernel", [
    "mxfp4_native_sp_h_f_n64", "mpp_mlp_h_i4_f_n128", "mpp_mlp_h_fp4_f_n128", "mpp_mlp_h_i2_f_n128",
    "mpp_mlp_h_fp8e4m3_f_n128", "mpp_mlp_h_fp8e5m2_f_n128", "mpp_mlp_h_fp8e4m3_h_n128",
])
@pytest.mark.parametrize("T,H,I", [(128, 1024, 4096), (64, 256, 512), (1, 512, 1024), (200, 256, 768)])
def test_mlp_rows(ctx, gate_kernel, T, H, I):
    got, ref, mid, mid_ref = run_mlp(ctx, gate_kernel, T, H, I)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    assert rel_fro(got[fin], ref[fin]) <= TOL, gate_kernel
    # the fused SwiGLU mid: identical except for rare one-ulp exp differences
    diff = mid.astype(np.float64) != mid_ref.astype(np.float64)
    assert diff.mean() < 1e-3


def test_mxfp4_wide_scales(ctx):
    got, ref, _, _ = run_mlp(ctx, "mxfp4_native_sp_h_f_n64", 128, 512, 1024, wide=True)
    fin = np.isfinite(ref)
    assert rel_fro(got[fin], ref[fin]) <= TOL


@pytest.mark.parametrize("T", [16, 129, 512])
def test_mxfp4_token_counts(ctx, T):
    got, ref, _, _ = run_mlp(ctx, "mxfp4_native_sp_h_f_n64", T, 1024, 4096)
    assert rel_fro(got, ref) <= TOL


def test_benchmark_entry_point(ctx):
    T, H, I = 128, 1024, 4096
    d = O.reference_mlp_inputs(T, H, I)
    desc = mpp41.describe("mxfp4_native_sp_h_f_n64", T, H, I)
    d_out, d_scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    secs = ctx.mlp_benchmark(desc, to_dev(d["x"]), to_dev(d["wg"]), to_dev(d["wu"]), to_dev(d["wd"]),
                             to_dev(d["sg"]), to_dev(d["su"]), to_dev(d["sd"]), d_scr, d_out, 20)
    assert 0 < secs < 1.0
    assert O.float_checksum(from_dev(d_out, np.float32, (T, H))) == "403573 over 32 samples"
