"""The failure path of the bounded device waits, on one GPU without a fault.

Every spin-wait of the layer kernels (mbarriers, grid-wide counters) gives up
after a wall-clock limit, records MPP41_ERR_TIMEOUT and a site code in the
context's device error word and returns, so the host reports an error instead
of the GPU hanging (the counterpart of the reference's command-buffer error
check, main.swift:251-256). mpp41_wait_probe runs the counter wait the layer
kernels use with a short limit; a flag that nothing sets makes it run out."""
import time

import numpy as np
import pytest

import mpp41
import oracle as O
from conftest import empty_dev, from_dev, to_dev
from gpu_data import rel_fro

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout(ctx):
    flag = empty_dev(4)
    flag.zero_()
    t0 = time.perf_counter()
    ctx.wait_probe(flag, 1, 10_000_000)          # 10 ms; nothing sets the flag
    with pytest.raises(mpp41.MPP41Error) as e:
        ctx.synchronize()
    assert e.value.status == mpp41.ERR_TIMEOUT
    assert "site 0xf01" in str(e.value)
    assert time.perf_counter() - t0 < 5.0        # the limit, not the 2 s default, ended it


def test_wait_that_is_satisfied_reports_ok(ctx):
    flag = to_dev(np.array([3], np.uint32))
    ctx.wait_probe(flag, 3, 10_000_000)
    ctx.synchronize()


def test_context_usable_after_timeout(ctx):
    """After a reported timeout the error word and counters are cleared and the
    next layer runs normally."""
    flag = empty_dev(4)
    flag.zero_()
    ctx.wait_probe(flag, 1, 5_000_000)
    with pytest.raises(mpp41.MPP41Error):
        ctx.synchronize()
    T, H, I = 128, 1024, 4096
    d = O.baseline_mlp_inputs(T, H, I, seed=5)
    dv = {k: to_dev(v) for k, v in d.items()}
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    out, scr = empty_dev(T * H * 2), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, dv["x"], dv["wg"], dv["wu"], dv["wd"], dv["sg"], dv["su"], dv["sd"], scr, out)
    ctx.synchronize()
    _, ref = O.mlp(0, O.W_MXFP4, 4, 1, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"])
    assert rel_fro(from_dev(out, np.float16, (T, H)), ref) <= 1e-3


def test_wait_probe_rejects_bad_limits(ctx):
    flag = empty_dev(4)
    for bad in (0, 20_000_000_000):
        with pytest.raises(mpp41.MPP41Error) as e:
            ctx.wait_probe(flag, 1, bad)
        assert e.value.status == mpp41.ERR_INVALID_ARGUMENT
