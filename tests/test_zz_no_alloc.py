"""mpp41_mlp_noalloc: one MLP layer for callers that may not allocate GPU
memory (a host framework that owns every device allocation, a plugin running
while the process's allocator is locked). It takes no context and no scratch
buffer; its scratch is the library's fixed static device array.

Checked through the C ABI on two calls in a row against the FP64 oracle and
against mpp41_mlp (the entry point with a caller-allocated scratch buffer),
within the MLP row tolerance, on shapes that reach each kernel route the
static scratch serves: the cluster kernel, the decode-size
GEMV kernels, and the weight-major kernel with its split-K workspace. After
each call mpp41_mlp_noalloc_status must report no device-side error. This file
is named to be collected last."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import activations, rel_fro, weights

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _inputs(T, H, I, wfmt, seed):
    if wfmt == O.W_MXFP4:
        d = O.baseline_mlp_inputs(T, H, I, seed=seed)
        return d, mpp41.SWIGLU_FP32
    x = activations(T, H)
    wg, sg = weights(wfmt, I, H, seed)
    wu, su = weights(wfmt, I, H, seed + 1)
    wd, sd = weights(wfmt, H, I, seed + 2)
    return dict(x=x, wg=wg, wu=wu, wd=wd, sg=sg, su=su, sd=sd), mpp41.SWIGLU_HALF


@pytest.mark.parametrize("T,H,I,wfmt,out_dtype", [
    (128, 1024, 4096, O.W_MXFP4, mpp41.F16),   # cluster kernel
    (128, 1024, 4096, O.W_MXFP4, mpp41.F32),
    (16, 1024, 4096, O.W_MXFP4, mpp41.F16),    # GEMV decode kernels
    (256, 1024, 2048, O.W_MXFP4, mpp41.F16),   # weight-major kernel, split-K workspace
    (128, 1024, 2048, O.W_E4M3, mpp41.F32),    # FP8 weights
])
def test_noalloc_matches_oracle_and_mlp_twice(ctx, T, H, I, wfmt, out_dtype):
    d, epi = _inputs(T, H, I, wfmt, seed=77)
    dv = {k: (to_dev(v) if v is not None else None) for k, v in d.items()}
    desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, epi, out_dtype)
    assert mpp41.lib().mpp41_mlp_noalloc_scratch_bytes(desc) <= mpp41.NOALLOC_SCRATCH_BYTES
    dt = np.float16 if out_dtype == mpp41.F16 else np.float32
    _, oracle_out = O.mlp(0, wfmt, desc.epilogue, 1 if out_dtype == mpp41.F16 else 0, T, H, I,
                          d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"], d["sg"], d["su"], d["sd"])
    ref_out, scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], scr, ref_out)
    ctx.synchronize()
    ref = from_dev(ref_out, dt, (T, H))
    assert rel_fro(ref, oracle_out) <= TOL
    out = empty_dev(T * H * 4)
    for _ in range(2):                       # the second call reuses the static scratch
        out.zero_()
        mpp41.mlp_noalloc(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], out)
        mpp41.mlp_noalloc_status()           # raises on a recorded device-side error
        got = from_dev(out, dt, (T, H))
        assert np.isfinite(got).all()
        assert rel_fro(got, oracle_out) <= TOL
        assert rel_fro(got, ref) <= TOL


def test_noalloc_rejects_layers_beyond_its_scratch(ctx):
    T, H, I = 4096, 1024, 4096               # mid alone is 32 MiB > the static array
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    buf = empty_dev(16)
    with pytest.raises(mpp41.MPP41Error) as e:
        mpp41.mlp_noalloc(desc, buf, buf, buf, buf, buf, buf, buf, buf)
    assert e.value.status == mpp41.ERR_UNSUPPORTED_SHAPE
    assert "static scratch" in str(e.value)
    mpp41.mlp_noalloc_status()               # a rejected call records nothing
