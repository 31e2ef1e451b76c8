"""CPU oracle pinned against the reference's golden values (no GPU).

Pins: the roundtrip known-answer vectors of main.swift:108-132 and the
published MXFP4 MLP checksum 403573 (README.md:292-295), both extracted
into tests/golden/reference_kats.json by tests/golden/make_golden.py.
"""
import numpy as np
import pytest

import oracle as O

FMT = {"fp4_e2m1_roundtrip": 0, "fp8_e4m3_roundtrip": 1, "fp8_e5m2_roundtrip": 2}


def test_roundtrip_kats(golden):
    tol = golden["roundtrip_tolerance"]
    for case in golden["roundtrip_cases"]:
        fmt = FMT[case["kernel"]]
        x = np.array(case["inputs"], np.float32)
        packed = O.pack(fmt, x)
        assert packed.size == case["packed_bytes"]
        got = O.unpack(fmt, packed, x.size)
        assert np.all(np.abs(got - np.array(case["expected"], np.float32)) <= tol), case["name"]


def test_mxfp4_mlp_checksum_403573(golden):
    g = golden["mxfp4_mlp_checksum"]
    T, H, I = g["tokens"], g["hidden"], g["intermediate"]
    d = O.reference_mlp_inputs(T, H, I)
    _, out = O.mlp(0, O.W_MXFP4, 1, 0, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"])
    assert O.float_checksum(out) == g["value"]


def test_e2m1_all_codes_roundtrip():
    vals = O.unpack(0, np.arange(256, dtype=np.uint8), 512)
    assert np.array_equal(O.pack(0, vals), np.arange(256, dtype=np.uint8))


@pytest.mark.parametrize("fmt,dtype", [(1, "float8_e4m3fn"), (2, "float8_e5m2")])
def test_fp8_codes_match_ml_dtypes(fmt, dtype):
    ml = pytest.importorskip("ml_dtypes")
    codes = np.arange(256, dtype=np.uint8)
    ours = O.unpack(fmt, codes, 256)
    theirs = codes.view(getattr(ml, dtype)).astype(np.float32)
    both_nan = np.isnan(ours) & np.isnan(theirs)
    assert np.all(both_nan | (ours == theirs))
    finite = np.isfinite(ours)
    # every finite code re-encodes to itself (incl. signed zero)
    assert np.array_equal(O.pack(fmt, ours[finite]), codes[finite])


@pytest.mark.parametrize("fmt,dtype,mx", [(0, "float4_e2m1fn", 6.0), (1, "float8_e4m3fn", 448.0),
                                          (2, "float8_e5m2", 57344.0)])
def test_encode_rne_matches_ml_dtypes_after_clamp(fmt, dtype, mx):
    """Round-to-nearest-even on U(-600, 600); ml_dtypes overflows to NaN/inf,
    the reference saturates, so compare after clamping to the finite range."""
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(7)
    x = rng.uniform(-600, 600, 200_000).astype(np.float32)
    x = np.concatenate([x, rng.uniform(-8, 8, 100_000).astype(np.float32)])
    ours = O.unpack(fmt, O.pack(fmt, x), x.size)
    theirs = np.clip(x, -mx, mx).astype(getattr(ml, dtype)).astype(np.float32)
    assert np.array_equal(ours, theirs)


def test_e8m0_edge_codes():
    L = O.lib()
    assert L.orc_e8m0_decode(127) == 1.0
    assert L.orc_e8m0_decode(0) == 0.0          # bit trick, not OCP 2^-127
    assert L.orc_e8m0_decode(255) == float("inf")  # bit trick, not OCP NaN
    assert L.orc_e8m0_decode(130) == 8.0


def test_int_decoders():
    w = np.arange(256, dtype=np.uint8)
    i4 = O.decode_weights(O.W_I4, w, None, 1, 512).ravel()
    assert set(i4.astype(int)) == set(range(-8, 8))
    assert i4[0] == 0 and i4[1] == 0 and i4[2] == 1 and i4[16 * 2 + 1] == 1  # low nibble = even k
    i2 = O.decode_weights(O.W_I2, w, None, 1, 1024).ravel()
    assert set(i2.astype(int)) == {-2, -1, 0, 1}
    assert list(i2[4 * 0x1B:4 * 0x1B + 4]) == [-1, -2, 1, 0]  # 0b00011011: pairs 3,2,1,0 LSB first; ((b&3)^2)-2


def test_half_fma_single_rounding():
    L = O.lib()
    h = lambda v: int(np.float16(v).view(np.uint16))
    # 2049 is not representable; a double-rounding fma would give 2048 or 2050 inconsistently
    assert L.orc_half_fma(h(2048), h(1), h(1)) == h(2048)  # tie -> even
    assert L.orc_half_fma(h(2048), h(1), h(3)) == h(2052)  # 2051 -> 2052 (even)
    # product 1+2^-11 exact in fp32 math; sum with 2048 ties broken by the low part
    a = h(1 + 2 ** -10)
    assert L.orc_half_fma(a, h(1 + 2 ** -10), h(2048)) == h(2050)


def test_swiglu_i8_monotone_and_clamped():
    L = O.lib()
    assert L.orc_swiglu_i8(0, 123456) == 0
    assert L.orc_swiglu_i8(10 ** 8, 10 ** 8) == 127
    assert L.orc_swiglu_i8(10 ** 8, -(10 ** 8)) == -128


def test_generators_shapes_and_ranges():
    x = O.half_values(4096, 0x11112222, 0.125).astype(np.float32)
    assert set(np.unique(x * 8).astype(int)) <= set(range(-8, 8))
    i8 = O.int8_values(4096, 0x22223333)
    assert i8.min() >= -8 and i8.max() <= 7
    s = O.pattern_bytes(4096, 0x7777DDDD, O.MXFP4_SCALE_PATTERN)
    assert set(np.unique(s)) <= set(O.MXFP4_SCALE_PATTERN)


def test_cpu_baseline_close_to_oracle():
    T, H, I = 64, 256, 512
    d = O.reference_mlp_inputs(T, H, I)
    _, ref = O.mlp(0, O.W_MXFP4, 1, 0, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"])
    got, n = O.mlp_mxfp4_cpu(T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"], d["sg"], d["su"], d["sd"])
    assert n >= 1
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


def test_quantizer_matches_independent_numpy_restatement():
    """OCP-MX quantizer against a numpy + ml_dtypes restatement."""
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0                                 # all-zero block
    w[1, :32] *= 1e4                                # large block
    packed, scales = O.quantize_mxfp4(w)
    blocks = w.reshape(32, 16, 32).astype(np.float64)
    amax = np.abs(blocks).max(axis=2)
    e = np.where(amax > 0, np.floor(np.log2(np.where(amax > 0, amax, 1))) - 2, -127)
    code = np.clip(e + 127, 0, 254)
    assert np.array_equal(scales, np.where(amax > 0, code, 0).astype(np.uint8))
    q = (blocks / np.exp2(code - 127)[..., None]).astype(np.float32)
    q = np.clip(q, -6, 6).astype(ml.float4_e2m1fn).astype(np.float32)
    deq = O.decode_weights(O.W_MXFP4, packed, scales, 32, 512).reshape(32, 16, 32)
    want = q * np.exp2(code - 127)[..., None]
    want[amax == 0] = 0
    assert np.array_equal(deq, want)


def test_baseline_inputs_are_finite_and_scaled():
    d = O.baseline_mlp_inputs(8, 256, 512)
    assert d["x"].dtype == np.float16 and d["wg"].shape == (512, 128) and d["sg"].shape == (512, 8)
    assert 110 < int(np.median(d["sg"])) < 125   # amax of 32 N(0, 0.02) draws ~ 2^-4.5
