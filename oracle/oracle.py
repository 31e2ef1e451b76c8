"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this module; the product path never does. The arithmetic lives in
oracle/mpp41_oracle.c, a C restatement of the reference's Metal kernels and
Swift data generators (each C function cites its reference file:line).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# weight formats (match include/mpp41.h enum mpp41_wfmt)
W_F16, W_I8, W_I4, W_I2, W_FP4, W_E4M3, W_E5M2, W_MXFP4, W_E4M3_MX, W_E5M2_MX = range(10)

# reference seeds, main.swift:611-638 (MLP) and 409-413 (big matmul)
MLP_SEEDS = {
    "x_half": 0x11112222, "x_int8": 0x22223333,
    "wg_half": 0x55556666, "wu_half": 0x77778888, "wd_half": 0x9999AAAA,
    "wg_i8": 0x33334444, "wu_i8": 0x44445555, "wd_i8": 0x55557777,
    "wg_i4": 0x13572468, "wu_i4": 0xACE01357, "wd_i4": 0xC001D00D,
    "wg_i2": 0x24681357, "wu_i2": 0xBAD0CAFE, "wd_i2": 0xD00DC001,
    "wg_fp4": 0xABCD1357, "wu_fp4": 0x2468BDF0, "wd_fp4": 0x0BADCAFE,
    "wg_e4m3": 0x11117777, "wu_e4m3": 0x22228888, "wd_e4m3": 0x33339999,
    "wg_e5m2": 0x4444AAAA, "wu_e5m2": 0x5555BBBB, "wd_e5m2": 0x6666CCCC,
    "sg": 0x7777DDDD, "su": 0x8888EEEE, "sd": 0x9999FFFF,
}
MXFP4_SCALE_PATTERN = bytes([124, 125, 126, 127, 127, 128, 128, 129, 130])
MATMUL_SEEDS = {"a_packed": 0x12345678, "b_packed": 0x87654321, "a_half": 0x2468ACE0,
                "a_int8": 0x13579BDF, "b_half": 0xFDB97531}

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, u32, sz = C.c_void_p, C.c_uint32, C.c_size_t
        L.orc_make_packed_bytes.argtypes = [vp, sz, u32]
        L.orc_make_pattern_bytes.argtypes = [vp, sz, u32, vp, sz]
        L.orc_make_fp8_e4m3_bytes.argtypes = [vp, sz, u32]
        L.orc_make_fp8_e5m2_bytes.argtypes = [vp, sz, u32]
        L.orc_make_half_values.argtypes = [vp, sz, u32, C.c_float]
        L.orc_make_int8_values.argtypes = [vp, sz, u32]
        L.orc_pack.argtypes = [C.c_int, vp, sz, vp]
        L.orc_unpack.argtypes = [C.c_int, vp, sz, vp]
        L.orc_decode_weights.argtypes = [C.c_int, vp, vp, u32, u32, vp]
        L.orc_mxfp4_dequant_half.argtypes = [vp, vp, vp, u32, u32]
        L.orc_gemm_f64.argtypes = [vp, vp, vp, u32, u32, u32]
        L.orc_mlp.argtypes = [C.c_int] * 4 + [u32] * 3 + [vp] * 9
        L.orc_mlp_row_scaled.argtypes = [C.c_int] * 3 + [u32] * 3 + [vp] * 9
        L.orc_mlp_mxfp4_cpu.argtypes = [u32] * 3 + [vp] * 8 + [C.c_int, u32, u32, C.c_int]
        L.orc_quantize_mxfp4.argtypes = [vp, u32, u32, vp, vp]
        L.orc_quantize_nvfp4.argtypes = [vp, u32, u32, vp, vp, vp]
        L.orc_decode_nvfp4.argtypes = [vp, vp, C.c_float, u32, u32, vp]
        L.orc_mlp_mxfp4_cpu.restype = C.c_int
        L.orc_scalar_mlp_gate_up.argtypes = [C.c_int, u32, u32, u32, vp, vp, vp, vp]
        L.orc_scalar_mlp_down.argtypes = [C.c_int, u32, u32, u32, vp, vp, vp]
        L.orc_scalar_matmul.argtypes = [C.c_int, u32, u32, u32, vp, vp, vp]
        L.orc_half_fma.argtypes = [C.c_uint16] * 3
        L.orc_half_fma.restype = C.c_uint16
        L.orc_swiglu_array.argtypes = [C.c_int, vp, vp, vp, sz]
        L.orc_swiglu_i8.argtypes = [C.c_int32, C.c_int32]
        L.orc_swiglu_i8.restype = C.c_int8
        L.orc_e2m1_encode.argtypes = [C.c_float]
        L.orc_e2m1_encode.restype = C.c_uint8
        L.orc_e8m0_decode.argtypes = [C.c_uint8]
        L.orc_e8m0_decode.restype = C.c_float
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- generators
def packed_bytes(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().orc_make_packed_bytes(_p(out), n, seed)
    return out


def pattern_bytes(n: int, seed: int, pattern: bytes) -> np.ndarray:
    out = np.empty(n, np.uint8)
    pat = np.frombuffer(pattern, np.uint8).copy()
    lib().orc_make_pattern_bytes(_p(out), n, seed, _p(pat), len(pat))
    return out


def fp8_bytes(n: int, seed: int, e5m2: bool) -> np.ndarray:
    out = np.empty(n, np.uint8)
    (lib().orc_make_fp8_e5m2_bytes if e5m2 else lib().orc_make_fp8_e4m3_bytes)(_p(out), n, seed)
    return out


def half_values(n: int, seed: int, scale: float = 0.25) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_make_half_values(_p(out), n, seed, scale)
    return out.view(np.float16)


def int8_values(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_make_int8_values(_p(out), n, seed)
    return out


# ---------------------------------------------------------------- codecs
def pack(fmt: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    out = np.zeros((n + 1) // 2 if fmt == 0 else n, np.uint8)
    lib().orc_pack(fmt, _p(x), n, _p(out))
    return out


def unpack(fmt: int, packed: np.ndarray, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.empty(n, np.float32)
    lib().orc_unpack(fmt, _p(packed), n, _p(out))
    return out


def decode_weights(wfmt: int, w: np.ndarray, scales, rows: int, depth: int) -> np.ndarray:
    out = np.empty((rows, depth), np.float64)
    s = _p(scales) if scales is not None else None
    lib().orc_decode_weights(wfmt, _p(np.ascontiguousarray(w)), s, rows, depth, _p(out))
    return out


def mxfp4_dequant_half(packed, scales, rows, depth) -> np.ndarray:
    out = np.empty((rows, depth), np.uint16)
    lib().orc_mxfp4_dequant_half(_p(packed), _p(scales), _p(out), rows, depth)
    return out.view(np.float16)


def mlp(act, wfmt, epi, out_kind, T, H, I, x, wg, wu, wd, sg=None, su=None, sd=None, row_scales=False):
    """Returns (mid, out) of one MLP row, fp64-exact GEMMs (see mpp41_oracle.h).
    row_scales: sg / su / sd are fp16 per-output-channel scales (INT weights)."""
    mid_dt = {0: np.float32, 1: np.float16, 2: np.float16, 3: np.int8, 4: np.float16}[epi]
    out_dt = {0: np.float32, 1: np.float16, 2: np.int32}[out_kind]
    mid = np.empty((T, I), mid_dt)
    out = np.empty((T, H), out_dt)
    ps = [(_p(np.ascontiguousarray(a)) if a is not None else None) for a in (sg, su, sd)]
    args = (T, H, I, _p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(wg)), _p(np.ascontiguousarray(wu)),
            _p(np.ascontiguousarray(wd)), *ps, _p(mid), _p(out))
    if row_scales:
        lib().orc_mlp_row_scaled(wfmt, epi, out_kind, *args)
    else:
        lib().orc_mlp(act, wfmt, epi, out_kind, *args)
    return mid, out


INT_QMAX = {W_I8: 127, W_I4: 7, W_I2: 1}


def quantize_int_rowscale(w: np.ndarray, wfmt: int):
    """Per-output-row symmetric integer weights with an fp16 scale (BASELINE
    config 2's INT rows): s = half(amax / qmax) (1 for an all-zero row),
    q = clip(rint(w / s), -qmax - 1, qmax), packed in the reference layouts
    (INT8 bytes; INT4 low nibble = even k; INT2 LSB pair first). Returns
    (packed, fp16 scales)."""
    w = np.asarray(w, np.float32)
    qmax = INT_QMAX[wfmt]
    s = (np.abs(w).max(axis=1) / qmax).astype(np.float16)
    s[s == 0] = np.float16(1.0)
    q = np.clip(np.rint(w / s.astype(np.float32)[:, None]), -qmax - 1, qmax).astype(np.int32)
    if wfmt == W_I8:
        return q.astype(np.int8), s
    if wfmt == W_I4:
        n = (q & 0xF).astype(np.uint8)
        return (n[:, 0::2] | (n[:, 1::2] << 4)).astype(np.uint8), s
    n = (q & 0x3).astype(np.uint8)
    return (n[:, 0::4] | (n[:, 1::4] << 2) | (n[:, 2::4] << 4) | (n[:, 3::4] << 6)).astype(np.uint8), s


def quantize_mxfp8(w: np.ndarray, e5m2: bool = False):
    """OCP-MX style FP8 with an E8M0 scale per 32 along K (BASELINE config 2's
    FP8 rows): e = floor(log2(block amax)) - emax (8 for E4M3, 15 for E5M2),
    elements = RNE-saturated encode(w / 2^e). Returns (bytes [rows][depth],
    scales [rows][depth/32])."""
    w = np.asarray(w, np.float32)
    rows, depth = w.shape
    blk = w.reshape(rows, depth // 32, 32)
    amax = np.abs(blk).max(axis=2)
    e = np.where(amax > 0, np.floor(np.log2(np.where(amax > 0, amax, 1.0))) - (15 if e5m2 else 8), -127)
    e = np.clip(e, -127, 127).astype(np.int32)
    scaled = (blk / np.exp2(e.astype(np.float64))[:, :, None]).astype(np.float32).reshape(-1)
    packed = pack(2 if e5m2 else 1, scaled).reshape(rows, depth)
    return packed, (e + 127).astype(np.uint8)


def swiglu(kind: int, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """Standalone SwiGLU kernels (MPPMLPKernels.metal:186-257), elementwise."""
    gate, up = np.ascontiguousarray(gate), np.ascontiguousarray(up)
    out = np.empty(gate.shape, {0: np.float32, 1: np.float16, 2: np.float16, 3: np.int8}[kind])
    lib().orc_swiglu_array(kind, _p(gate), _p(up), _p(out), gate.size)
    return out


def mlp_mxfp4_cpu(T, H, I, x, wg, wu, wd, sg, su, sd, nthreads=0, t0=0, t1=None, plain=False):
    out = np.zeros((T, H), np.float32)
    t1 = T if t1 is None else t1
    n = lib().orc_mlp_mxfp4_cpu(T, H, I, _p(x), _p(wg), _p(wu), _p(wd), _p(sg), _p(su), _p(sd),
                                _p(out), nthreads, t0, t1, int(plain))
    return out, n


def quantize_mxfp4(w: np.ndarray):
    """OCP-MX fp32 [rows][depth] -> (packed [rows][depth/2], scales [rows][depth/32])."""
    w = np.ascontiguousarray(w, np.float32)
    rows, depth = w.shape
    packed = np.empty((rows, depth // 2), np.uint8)
    scales = np.empty((rows, depth // 32), np.uint8)
    lib().orc_quantize_mxfp4(_p(w), rows, depth, _p(packed), _p(scales))
    return packed, scales


def quantize_nvfp4(w: np.ndarray):
    """NVFP4 fp32 [rows][depth] -> (packed [rows][depth/2], scales [rows][depth/16], tensor scale)."""
    w = np.ascontiguousarray(w, np.float32)
    rows, depth = w.shape
    packed = np.empty((rows, depth // 2), np.uint8)
    scales = np.empty((rows, depth // 16), np.uint8)
    ts = np.zeros(1, np.float32)
    lib().orc_quantize_nvfp4(_p(w), rows, depth, _p(packed), _p(scales), _p(ts))
    return packed, scales, float(ts[0])


def decode_nvfp4(packed, scales, tensor_scale, rows, depth) -> np.ndarray:
    out = np.empty((rows, depth), np.float64)
    lib().orc_decode_nvfp4(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)),
                           C.c_float(tensor_scale), rows, depth, _p(out))
    return out


def nvfp4_mlp(x, wg, sg, tg, wu, su, tu, wd, sd, td):
    """NVFP4 W4A4 layer restated: x quantized (NVFP4 recipe), exact gate/up
    products, mid = silu(g) * u in fp64 rounded to fp16 (the layer's stored
    mid), quantized again, exact down product. Returns (xq, xs, tx, mid16, out)."""
    T, H = x.shape
    I = wg.shape[0]
    xq, xs, tx = quantize_nvfp4(np.asarray(x, np.float32))
    xd = decode_nvfp4(xq, xs, tx, T, H)
    g = xd @ decode_nvfp4(wg, sg, tg, I, H).T
    u = xd @ decode_nvfp4(wu, su, tu, I, H).T
    mid = (g / (1.0 + np.exp(-g)) * u).astype(np.float16)
    mq, ms, tm = quantize_nvfp4(mid.astype(np.float32))
    out = decode_nvfp4(mq, ms, tm, T, I) @ decode_nvfp4(wd, sd, td, H, I).T
    return xq, xs, tx, mid, out


def w4a4_mlp(x, wg, sg, wu, su, wd, sd):
    """W4A4 layer restated (no reference counterpart; its MXFP4 decode is
    MXFP4Kernels.metal:26-29 and docs/MXFP4-MPP41-GUIDE.md:43-55): x is
    quantized with the OCP-MX rule, gate/up products are exact (fp64),
    mid = silu(g) * u in fp64 rounded to fp32, then quantized with the same
    rule; the down product is exact on the decoded quantized mid.
    Returns (xq, xs, mq, ms, out) with out fp64 [T][H]."""
    T, H = x.shape
    I = wg.shape[0]
    xq, xs = quantize_mxfp4(np.asarray(x, np.float32))
    xd = decode_weights(W_MXFP4, xq, xs, T, H)
    g = xd @ decode_weights(W_MXFP4, wg, sg, I, H).T
    u = xd @ decode_weights(W_MXFP4, wu, su, I, H).T
    mid = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
    mq, ms = quantize_mxfp4(mid)
    out = decode_weights(W_MXFP4, mq, ms, T, I) @ decode_weights(W_MXFP4, wd, sd, H, I).T
    return xq, xs, mq, ms, out


def moe_route(logits: np.ndarray, k: int):
    """Top-k by descending logit, ties to the lower expert id; weights =
    softmax over the chosen logits (fp64)."""
    order = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    chosen = np.take_along_axis(logits, order, axis=1).astype(np.float64)
    e = np.exp(chosen - chosen[:, :1])
    return order.astype(np.int32), e / e.sum(axis=1, keepdims=True)


def moe_permutation(ids: np.ndarray, E: int):
    """Rows grouped by expert, assignment order within an expert: perm[r] = assignment."""
    flat = ids.reshape(-1)
    perm = np.argsort(flat, kind="stable").astype(np.uint32)
    counts = np.bincount(flat, minlength=E).astype(np.uint32)
    return perm, counts


def moe_w4a4(x, logits, k, wg, sg, wu, su, wd, sd, shared=None):
    """W4A4 MoE restated: returns (ids, weights, perm, mq, ms, y, out) with y and
    out fp64; each expert row follows w4a4_mlp's rules (x quantized once)."""
    T, H = x.shape
    E, I = wg.shape[0], wg.shape[1]
    ids, w = moe_route(logits, k)
    perm, counts = moe_permutation(ids, E)
    xq, xs = quantize_mxfp4(np.asarray(x, np.float32))
    xd = decode_weights(W_MXFP4, xq, xs, T, H)
    R = T * k
    mq = np.zeros((R, I // 2), np.uint8)
    ms = np.zeros((R, I // 32), np.uint8)
    y = np.zeros((R, H))
    r0 = 0
    for e in range(E):
        rows = perm[r0:r0 + counts[e]]
        if len(rows):
            xr = xd[rows // k]
            g = xr @ decode_weights(W_MXFP4, wg[e], sg[e], I, H).T
            u = xr @ decode_weights(W_MXFP4, wu[e], su[e], I, H).T
            q, qs = quantize_mxfp4((g / (1.0 + np.exp(-g)) * u).astype(np.float32))
            mq[r0:r0 + len(rows)], ms[r0:r0 + len(rows)] = q, qs
            y[r0:r0 + len(rows)] = decode_weights(W_MXFP4, q, qs, len(rows), I) @ decode_weights(W_MXFP4, wd[e], sd[e], H, I).T
        r0 += counts[e]
    inv = np.empty(R, np.int64)
    inv[perm] = np.arange(R)
    out = (w[:, :, None] * y[inv].reshape(T, k, H)).sum(axis=1)
    if shared is not None:
        out = out + w4a4_mlp(x, *shared)[-1]
    return ids, w, perm, mq, ms, y, out


def quantize_int_rows(w: np.ndarray, bits: int):
    """Per-row symmetric integer weights (no reference counterpart; its int rows
    carry no scales): scale = amax/qmax (fp32; 1 for a zero row), q =
    rint(w/scale) clamped to +-qmax, packed like PackedNumericKernels.metal:25-33
    (INT4 low nibble = even k, INT2 LSB pair first). Returns (packed, scales)."""
    w = np.ascontiguousarray(w, np.float32)
    qmax = np.float32({8: 127, 4: 7, 2: 1}[bits])
    amax = np.abs(w).max(axis=1)
    scale = np.where(amax > 0, amax / qmax, np.float32(1)).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -qmax, qmax).astype(np.int64)
    per = 8 // bits
    q = (q & ((1 << bits) - 1)).reshape(w.shape[0], -1, per)
    packed = np.zeros(q.shape[:2], np.int64)
    for j in range(per):
        packed |= q[:, :, j] << (bits * j)
    return packed.astype(np.uint8), scale


def quantize_act_s8(x: np.ndarray):
    """Per-token int8 (the rule of mpp41_quantize_act_s8): inv = 127/amax,
    q = rint(clip(x*inv, +-127)), scale = amax/127, all fp32."""
    xf = np.asarray(x, np.float32)
    amax = np.abs(xf).max(axis=1)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    q = np.rint(np.clip(xf * inv[:, None], -127, 127)).astype(np.int8)
    return q, (amax / np.float32(127)).astype(np.float32)


def baseline_mlp_inputs(T=128, H=1024, I=4096, seed=0):
    """x ~ N(0,1) fp16, weights ~ N(0,0.02) fp32 quantized OCP-MX."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    out = {"x": x}
    for name, (r, c) in (("g", (I, H)), ("u", (I, H)), ("d", (H, I))):
        w = (rng.standard_normal((r, c), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        out["w" + name], out["s" + name] = quantize_mxfp4(w)
    return out


def scalar_mlp(wfmt, T, H, I, x, wg, wu, wd):
    mid = np.empty((T, I), np.uint16)
    out = np.empty((T, H), np.uint16)
    lib().orc_scalar_mlp_gate_up(wfmt, T, H, I, _p(x), _p(wg), _p(wu), _p(mid))
    lib().orc_scalar_mlp_down(wfmt, T, H, I, _p(mid), _p(wd), _p(out))
    return mid.view(np.float16), out.view(np.float16)


def scalar_matmul(kind, M, N, K, a, b):
    dt = {0: np.float32, 4: np.int32}.get(kind, np.uint16)
    out = np.empty((M, N), dt)
    lib().orc_scalar_matmul(kind, M, N, K, _p(np.ascontiguousarray(a)), _p(np.ascontiguousarray(b)), _p(out))
    return out.view(np.float16) if dt is np.uint16 else out


# ---------------------------------------------------------------- checksums
def sample_indices(count: int) -> np.ndarray:
    step = max(1, count // 32)
    return np.arange(0, count, step)


def float_checksum(a: np.ndarray) -> str:
    flat = np.ascontiguousarray(a, np.float32).ravel()
    idx = sample_indices(flat.size)
    s = float(np.sum(flat[idx].astype(np.float64)))
    return f"{s:.6g} over {idx.size} samples"


def int_checksum(a: np.ndarray) -> str:
    flat = np.ascontiguousarray(a, np.int32).ravel()
    idx = sample_indices(flat.size)
    return f"{int(np.sum(flat[idx].astype(np.int64)))} over {idx.size} samples"


def half_raw_checksum(a: np.ndarray) -> str:
    flat = np.ascontiguousarray(a).view(np.uint16).ravel()
    idx = sample_indices(flat.size)
    return f"raw16 sum {int(np.sum(flat[idx].astype(np.uint64)))} over {idx.size} samples"


# ---------------------------------------------------------------- mode-R data
def reference_mlp_inputs(T=128, H=1024, I=4096):
    """The MXFP4 MLP inputs of runMLPBenchmark (main.swift:611-638)."""
    s = MLP_SEEDS
    return {
        "x": half_values(T * H, s["x_half"], 0.125).reshape(T, H),
        "wg": packed_bytes(I * H // 2, s["wg_fp4"]).reshape(I, H // 2),
        "wu": packed_bytes(I * H // 2, s["wu_fp4"]).reshape(I, H // 2),
        "wd": packed_bytes(H * I // 2, s["wd_fp4"]).reshape(H, I // 2),
        "sg": pattern_bytes(I * (H // 32), s["sg"], MXFP4_SCALE_PATTERN).reshape(I, H // 32),
        "su": pattern_bytes(I * (H // 32), s["su"], MXFP4_SCALE_PATTERN).reshape(I, H // 32),
        "sd": pattern_bytes(H * (I // 32), s["sd"], MXFP4_SCALE_PATTERN).reshape(H, I // 32),
    }
