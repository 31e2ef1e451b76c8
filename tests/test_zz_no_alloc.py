"""mpp41_mlp_noalloc: one MLP layer for callers that may not allocate GPU
memory (a host framework that owns every device allocation, a plugin running
while the process's allocator is locked). It takes no context and no scratch
buffer; its scratch is the library's fixed static device array.

Checked through the C ABI against mpp41_mlp (the existing entry point with a
caller-allocated scratch buffer) on two calls in a row, within the MLP row
tolerance. This file is named to be collected last."""
import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("out_dtype", [mpp41.F16, mpp41.F32])
def test_noalloc_matches_mlp_twice(ctx, out_dtype):
    T, H, I = 128, 1024, 4096
    d = O.baseline_mlp_inputs(T, H, I, seed=77)
    dv = {k: to_dev(v) for k, v in d.items()}
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, out_dtype)
    assert mpp41.lib().mpp41_mlp_noalloc_scratch_bytes(desc) <= mpp41.NOALLOC_SCRATCH_BYTES
    dt = np.float16 if out_dtype == mpp41.F16 else np.float32
    ref_out, scr = empty_dev(T * H * 4), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], scr, ref_out)
    ctx.synchronize()
    ref = from_dev(ref_out, dt, (T, H))
    out = empty_dev(T * H * 4)
    for _ in range(2):                       # the second call reuses the static scratch
        out.zero_()
        mpp41.mlp_noalloc(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], out)
        got = from_dev(out, dt, (T, H))
        assert np.isfinite(got).all()
        assert rel_fro(got, ref) <= TOL


def test_noalloc_rejects_layers_beyond_its_scratch(ctx):
    T, H, I = 4096, 1024, 4096               # mid alone is 32 MiB > the static array
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    buf = empty_dev(16)
    with pytest.raises(mpp41.MPP41Error) as e:
        mpp41.mlp_noalloc(desc, buf, buf, buf, buf, buf, buf, buf, buf)
    assert e.value.status == mpp41.ERR_UNSUPPORTED_SHAPE
    assert "static scratch" in str(e.value)
