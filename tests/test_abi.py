"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/mpp41.h declares, knows the reference kernel names, and fails with a
status (not a crash) when no device is present."""
import ctypes as C
import os

import pytest

import mpp41


def test_library_exports_every_declared_symbol():
    L = mpp41.lib()
    declared = mpp41.declared_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(L, s)]
    assert missing == []


@pytest.mark.parametrize("name", [
    "fp4_e2m1_roundtrip", "fp8_e4m3_roundtrip", "fp8_e5m2_roundtrip",
    "mxfp4_dequant_native_half", "mxfp4_dequant_lut_half",
    "mxfp4_native_sp_h_f_n64", "mxfp4_native_sp_h_f_n128", "mxfp4_native_sph_h_f_n64",
    "mxfp4_fused_h_f_n64", "mxfp4_fused_ci_h_f_sg_k32",
    "mpp_mlp_h_h_f_n128", "mpp_mlp_h_i4_f_n128", "mpp_mlp_h_fp4_f_n128", "mpp_mlp_h_i2_f_n128",
    "mpp_mlp_h_fp8e4m3_f_n128", "mpp_mlp_h_fp8e4m3_h_n128", "mpp_mlp_h_fp8e5m2_f_n128", "mpp_mlp_h_i8_f_n128",
    "mpp_mlp_swiglu_half", "mpp_mlp_swiglu_i8",
    "fp4_e2m1_matmul_benchmark", "int4_int8_matmul_benchmark", "half_fp4_mlp_gate_up_benchmark",
])
def test_registry_knows_reference_kernels(name):
    assert mpp41.has_kernel(name)


def test_registry_rejects_probe_only_kernels():
    # --mxfp4-decompose probes compute wrong math on purpose; they are out of scope
    for name in ["mxfp4_probe_coopstore_h_f_n64", "mxfp4_probe_noscale_h_f_n64", "no_such_kernel"]:
        assert not mpp41.has_kernel(name)


def test_describe_matches_reference_pairings():
    d = mpp41.describe("mxfp4_native_sp_h_f_n64", 128, 1024, 4096)
    assert (d.wfmt, d.epilogue, d.out_dtype) == (mpp41.W_MXFP4, mpp41.SWIGLU_HALF, mpp41.F32)
    d = mpp41.describe("mpp_mlp_h_fp8e4m3_h_n128", 128, 1024, 4096)
    assert (d.wfmt, d.epilogue, d.out_dtype) == (mpp41.W_E4M3, mpp41.SWIGLU_HALF_FROM_HALF, mpp41.F16)
    d = mpp41.describe("mpp_mlp_h_h_f_n128", 128, 1024, 4096)
    assert d.epilogue == mpp41.SWIGLU_FLOAT
    # the small-layer kernel: fp16 mid, then its 8 K-split partial tiles (fp32 T x H each)
    assert mpp41.scratch_bytes(mpp41.describe("mpp_mlp_h_i4_f_n128", 128, 1024, 4096)) == 128 * 4096 * 2 + 8 * 128 * 1024 * 4
    # the weight-major kernel: fp16 mid, then one fp32 T x H partial per K split (4 here)
    d = mpp41.mlp_desc(256, 1024, 2048, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F32)
    assert mpp41.scratch_bytes(d) == 256 * 2048 * 2 + 4 * 256 * 1024 * 4
    with pytest.raises(mpp41.MPP41Error) as e:
        mpp41.describe("not_a_kernel", 1, 64, 64)
    assert e.value.status == mpp41.ERR_MISSING_KERNEL


def test_status_strings():
    L = mpp41.lib()
    assert L.mpp41_status_string(mpp41.ERR_TIMEOUT) == b"device wait timed out"
    assert L.mpp41_status_string(mpp41.OK) == b"ok"


def test_null_context_is_an_error_not_a_crash():
    L = mpp41.lib()
    assert L.mpp41_synchronize(None) == mpp41.ERR_INVALID_ARGUMENT
    assert L.mpp41_mlp(None, None, *([None] * 9)) == mpp41.ERR_INVALID_ARGUMENT


def test_create_without_device_reports_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mpp41.MPP41Error) as e:
        mpp41.Context(0)
    assert e.value.status in (mpp41.ERR_NO_DEVICE, mpp41.ERR_CUDA)


def test_probe_cli_builds_and_fails_cleanly_without_a_device():
    import subprocess
    probe = os.path.join(os.path.dirname(mpp41.PKG) if False else mpp41.PKG, "bin", "mpp41probe")
    assert os.access(probe, os.X_OK)
    # unknown flags are ignored, as the reference's command line does; with no
    # device the probe exits 1 with the library's error
    r = subprocess.run([probe, "--no-such-flag"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "ignoring argument --no-such-flag" in r.stderr and "no device" in r.stderr
    r = subprocess.run([probe, "--mode=fast"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "--mode takes ref or baseline" in r.stderr
