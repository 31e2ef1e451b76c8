"""Weight handles (mpp41_weight_create, mpp41_mlp_weights, mpp41_gemm_weight):
the counterpart of the reference's host-built multi-plane MTLTensor over a
weight's packed values and scale plane (main.swift:2172-2212, 2254-2262). A
call through handles runs the same kernels on the same planes as the plain
entry point, so the outputs must be identical bit for bit; the handle's tensor
maps are encoded by the first call and reused by every later one."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import activations, rel_fro, weights

pytestmark = pytest.mark.gpu


def make_layer(ctx, wfmt, T, H, I, seed, row_scales=False):
    x = activations(T, H)
    if row_scales:
        rng = np.random.default_rng(seed)
        planes = {}
        for name, (r, c) in (("g", (I, H)), ("u", (I, H)), ("d", (H, I))):
            w = (rng.standard_normal((r, c), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            planes["w" + name], planes["s" + name] = O.quantize_int_rowscale(w, wfmt)
    else:
        planes = {}
        for name, (r, c), sd in (("g", (I, H), 1), ("u", (I, H), 2), ("d", (H, I), 3)):
            planes["w" + name], planes["s" + name] = weights(wfmt, r, c, seed + sd)
    dv = {k: (to_dev(v) if v is not None else None) for k, v in planes.items()}
    dv["x"] = to_dev(x)
    return dv


@pytest.mark.parametrize("T,H,I,kernel", [(128, 1024, 4096, "small"), (1, 4096, 2048, "gemv"),
                                          (256, 1024, 4096, "weight_major"), (20, 1024, 2048, "gemv_regs")])
def test_mlp_through_handles_matches_plain_call(ctx, T, H, I, kernel):
    wfmt = mpp41.W_MXFP4
    dv = make_layer(ctx, wfmt, T, H, I, seed=7)
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    nbytes = mpp41.scratch_bytes(desc)
    out_a, scr_a = empty_dev(T * H * 2), empty_dev(nbytes)
    ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], scr_a, out_a)
    ctx.synchronize()
    assert ctx.mlp_last_kernel() == kernel
    ref = from_dev(out_a, np.float16, (T, H))

    hg = ctx.weight(wfmt, dv["wg"], dv["sg"], H, I)
    hu = ctx.weight(wfmt, dv["wu"], dv["su"], H, I)
    hd = ctx.weight(wfmt, dv["wd"], dv["sd"], I, H)
    out_b, scr_b = empty_dev(T * H * 2), empty_dev(nbytes)
    ctx.mlp_weights(desc, dv["x"], hg, hu, hd, scr_b, out_b)
    ctx.synchronize()
    assert ctx.mlp_last_kernel() == kernel
    assert np.array_equal(from_dev(out_b, np.float16, (T, H)).view(np.uint16), ref.view(np.uint16))
    first = [h.map_counts() for h in (hg, hu, hd)]
    if kernel == "gemv_regs":                    # reads the weights with plain loads: no descriptors
        assert all(e == 0 for e, _ in first)
    else:
        assert all(e > 0 for e, _ in first)      # the launch encoded each plane's maps once

    for _ in range(2):
        ctx.mlp_weights(desc, dv["x"], hg, hu, hd, scr_b, out_b)
    ctx.synchronize()
    assert np.array_equal(from_dev(out_b, np.float16, (T, H)).view(np.uint16), ref.view(np.uint16))
    later = [h.map_counts() for h in (hg, hu, hd)]
    for (e0, r0), (e1, r1) in zip(first, later):
        assert e1 == e0 and r1 >= r0 + 2 * e0     # nothing re-encoded: every map reused
    for h in (hg, hu, hd):
        h.close()


def test_row_scaled_layer_through_handles(ctx):
    """BASELINE config 2 INT4 rows: the handle's scale plane is the fp16 row scales."""
    T, H, I, wfmt = 128, 1024, 4096, mpp41.W_I4
    dv = make_layer(ctx, wfmt, T, H, I, seed=21, row_scales=True)
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16, mpp41.MLP_ROW_SCALES)
    nbytes = mpp41.scratch_bytes(desc)
    out_a, out_b = empty_dev(T * H * 2), empty_dev(T * H * 2)
    ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], empty_dev(nbytes), out_a)
    hs = [ctx.weight(wfmt, dv["w" + n], dv["s" + n], k, r) for n, k, r in (("g", H, I), ("u", H, I), ("d", I, H))]
    ctx.mlp_weights(desc, dv["x"], *hs, empty_dev(nbytes), out_b)
    ctx.synchronize()
    assert np.array_equal(from_dev(out_a, np.uint16, (T, H)), from_dev(out_b, np.uint16, (T, H)))


def test_gemm_through_handle(ctx):
    """The handle row of the reference (mxfp4_native_sph_h_f_n64) through a handle."""
    M, N, K = 96, 512, 1024
    wfmt = mpp41.W_MXFP4
    a = to_dev(activations(M, K))
    wb, sb = weights(wfmt, N, K, 99)
    dw, ds = to_dev(wb), to_dev(sb)
    c_a, c_b = empty_dev(M * N * 4), empty_dev(M * N * 4)
    ctx.gemm("mxfp4_native_sph_h_f_n64", a, dw, c_a, M, N, K, ds)
    h = ctx.weight(wfmt, dw, ds, K, N)
    for _ in range(2):
        ctx.gemm_weight("mxfp4_native_sph_h_f_n64", a, h, c_b, M)
    ctx.synchronize()
    # split-K partial sums meet through float atomics, whose order varies between launches
    assert rel_fro(from_dev(c_b, np.float32, (M, N)), from_dev(c_a, np.float32, (M, N))) <= 1e-6
    e, r = h.map_counts()
    assert e >= 1 and r >= e


def test_handle_mismatches_are_rejected(ctx):
    T, H, I, wfmt = 4, 1024, 2048, mpp41.W_MXFP4
    dv = make_layer(ctx, wfmt, T, H, I, seed=5)
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    hg = ctx.weight(wfmt, dv["wg"], dv["sg"], H, I)
    hu = ctx.weight(wfmt, dv["wu"], dv["su"], H, I)
    wrong = ctx.weight(wfmt, dv["wd"], dv["sd"], H, I)       # down needs k = I, n = H
    with pytest.raises(mpp41.MPP41Error):
        ctx.mlp_weights(desc, dv["x"], hg, hu, wrong, empty_dev(mpp41.scratch_bytes(desc)), empty_dev(T * H * 2))
    with pytest.raises(mpp41.MPP41Error):                    # block-scaled format without its scale plane
        ctx.weight(wfmt, dv["wg"], None, H, I)
    fp4 = mpp41.mlp_desc(T, H, I, mpp41.W_FP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    hd = ctx.weight(wfmt, dv["wd"], dv["sd"], I, H)
    with pytest.raises(mpp41.MPP41Error):                    # handle format differs from the call's
        ctx.mlp_weights(fp4, dv["x"], hg, hu, hd, empty_dev(mpp41.scratch_bytes(fp4)), empty_dev(T * H * 2))
