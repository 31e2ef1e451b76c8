"""GPU packed-format parity, through the C ABI: the reference's roundtrip
known-answer tests (main.swift:108-132), every E2M1/E4M3/E5M2 code, clipped
U(-600,600) inputs (bit-exact against the oracle), and the two MXFP4
dequant kernels (MXFP4Kernels.metal:509-564) against the oracle."""
import numpy as np
import pytest

import oracle as O
from conftest import empty_dev, from_dev, to_dev

pytestmark = pytest.mark.gpu
FMT = {"fp4_e2m1_roundtrip": 0, "fp8_e4m3_roundtrip": 1, "fp8_e5m2_roundtrip": 2}


def test_roundtrip_kats(ctx, golden):
    tol = golden["roundtrip_tolerance"]
    for case in golden["roundtrip_cases"]:
        x = np.array(case["inputs"], np.float32)
        d_in, d_packed, d_out = to_dev(x), empty_dev(case["packed_bytes"]), empty_dev(4 * x.size)
        ctx.roundtrip(case["kernel"], d_in, d_packed, d_out)
        ctx.synchronize()
        got = from_dev(d_out, np.float32, x.shape)
        assert np.all(np.abs(got - np.array(case["expected"], np.float32)) <= tol), case["name"]
        packed = from_dev(d_packed, np.uint8, (case["packed_bytes"],))
        assert np.array_equal(packed, O.pack(FMT[case["kernel"]], x)), case["name"]


@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_all_codes_decode_and_reencode(ctx, fmt):
    codes = np.arange(256, dtype=np.uint8)
    n = 512 if fmt == 0 else 256
    d_codes, d_f = to_dev(codes), empty_dev(4 * n)
    ctx.unpack(fmt, d_codes, n, d_f)
    got = from_dev(d_f, np.float32, (n,))
    ref = O.unpack(fmt, codes, n)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))   # incl. signed zeros
    # every finite value re-encodes to its own code
    finite = np.isfinite(ref)
    vals = ref.copy()
    vals[~finite] = 0
    d_packed = empty_dev(n if fmt else n // 2)
    ctx.pack(fmt, to_dev(vals), n, d_packed)
    packed = from_dev(d_packed, np.uint8, (n if fmt else n // 2,))
    assert np.array_equal(packed, O.pack(fmt, vals))


@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_pack_uniform_600_bit_exact(ctx, fmt):
    rng = np.random.default_rng(100 + fmt)
    n = 1 << 24
    x = rng.uniform(-600, 600, n).astype(np.float32)
    x[:1000] = rng.uniform(-1, 1, 1000).astype(np.float32)        # values near zero and ties
    x[1000:1016] = [0.25, -0.25, 0.75, 2.5, 5.0, -5.0, 3.5, 1.25, 448, 464, -480, 57344, 61440, 1e9, -1e9, 0.0]
    nb = n // 2 if fmt == 0 else n
    d_packed = empty_dev(nb)
    ctx.pack(fmt, to_dev(x), n, d_packed)
    got = from_dev(d_packed, np.uint8, (nb,))
    assert np.array_equal(got, O.pack(fmt, x))
    # unpack round trip equals the oracle's decode
    d_f = empty_dev(4 * n)
    ctx.unpack(fmt, d_packed, n, d_f)
    assert np.array_equal(from_dev(d_f, np.float32, (n,)).view(np.uint32), O.unpack(fmt, got, n).view(np.uint32))


@pytest.mark.parametrize("n", [1, 7, 9, 33, 1000])
def test_pack_ragged_lengths(ctx, n):
    rng = np.random.default_rng(n)
    x = rng.uniform(-10, 10, n).astype(np.float32)
    for fmt in (0, 1, 2):
        nb = (n + 1) // 2 if fmt == 0 else n
        d_packed = empty_dev(nb + 16)
        ctx.pack(fmt, to_dev(x), n, d_packed)
        assert np.array_equal(from_dev(d_packed, np.uint8, (nb + 16,))[:nb], O.pack(fmt, x))


@pytest.mark.parametrize("kernel", ["mxfp4_dequant_native_half", "mxfp4_dequant_lut_half"])
@pytest.mark.parametrize("rows,depth", [(4096, 1024), (37, 96)])
def test_mxfp4_dequant_bit_exact(ctx, kernel, rows, depth):
    packed = O.packed_bytes(rows * depth // 2, 0xABCD1357)
    scales = O.pattern_bytes(rows * depth // 32, 0x7777DDDD, bytes(range(96, 150)) + bytes([0, 1, 127, 200, 250]))
    d_out = empty_dev(rows * depth * 2)
    ctx.dequant(kernel, to_dev(packed), to_dev(scales), d_out, rows, depth)
    got = from_dev(d_out, np.uint16, (rows, depth))
    ref = O.mxfp4_dequant_half(packed, scales, rows, depth).view(np.uint16)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("kind,name", [(0, "mpp_mlp_swiglu_float"), (1, "mpp_mlp_swiglu_half"),
                                       (2, "mpp_mlp_swiglu_half_from_half"), (3, "mpp_mlp_swiglu_i8")])
def test_swiglu_kernels_bit_exact(ctx, kind, name):
    rng = np.random.default_rng(3 + kind)
    T, I = 64, 512
    if kind == 3:
        g = rng.integers(-200000, 200000, (T, I)).astype(np.int32)
        u = rng.integers(-200000, 200000, (T, I)).astype(np.int32)
    else:
        g = (rng.standard_normal((T, I)) * 40).astype(np.float32)
        u = (rng.standard_normal((T, I)) * 40).astype(np.float32)
        if kind == 2:
            g, u = g.astype(np.float16), u.astype(np.float16)
    ref = O.swiglu(kind, g, u)
    d_mid = empty_dev(ref.nbytes)
    ctx.swiglu(name, to_dev(g), to_dev(u), d_mid, T, 1, I)
    got = from_dev(d_mid, ref.dtype, ref.shape)
    assert np.array_equal(got.view(np.uint8), ref.view(np.uint8))
