"""Python binding of libmpp41 (the C ABI in include/mpp41.h).

A thin ctypes layer that mirrors the reference probe's kernel interface:
kernels are addressed by the reference's own names ("mxfp4_native_sp_h_f_n64",
"mpp_mlp_h_i4_f_n128", "fp4_e2m1_roundtrip", ...), buffers are device
pointers, and every failing call raises MPP41Error carrying the status code
(the analogue of the reference's ProbeError, main.swift:5-38).

Device memory is any object with a ``data_ptr()`` (a torch CUDA tensor) or an
integer address. There is no CPU fallback: without the built library or a
B200 every call fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB_PATH = os.environ.get("MPP41_LIB") or os.path.join(PKG, "lib", "libmpp41.so")
HEADER = os.path.join(ROOT, "include", "mpp41.h")

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED_SHAPE, ERR_NO_DEVICE, ERR_MISSING_KERNEL, ERR_OUT_OF_MEMORY, \
    ERR_CUDA, ERR_TIMEOUT, ERR_BOUNDS, ERR_COMM = range(10)
W_F16, W_I8, W_I4, W_I2, W_FP4, W_E4M3, W_E5M2, W_MXFP4, W_E4M3_MX, W_E5M2_MX = range(10)
A_F16, A_S8 = 0, 1
SWIGLU_FLOAT, SWIGLU_HALF, SWIGLU_HALF_FROM_HALF, SWIGLU_I8, SWIGLU_FP32 = range(5)
F32, F16, S32, S8 = range(4)
MLP_UNFUSED = 0x1
MLP_ROW_SCALES = 0x2
FMT_E2M1, FMT_E4M3, FMT_E5M2 = 0, 1, 2


class MPP41Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"mpp41 status {status}: {message}")
        self.status = status


class MatmulConfig(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("depth", C.c_uint32),
                ("packed_depth_bytes", C.c_uint32)]


class MLPConfig(C.Structure):
    _fields_ = [("tokens", C.c_uint32), ("hidden", C.c_uint32), ("intermediate", C.c_uint32)]


class MLPDesc(C.Structure):
    _fields_ = [("tokens", C.c_uint32), ("hidden", C.c_uint32), ("intermediate", C.c_uint32),
                ("wfmt", C.c_int32), ("afmt", C.c_int32), ("epilogue", C.c_int32), ("out_dtype", C.c_int32),
                ("flags", C.c_uint32)]


class MoEDesc(C.Structure):
    _fields_ = [("tokens", C.c_uint32), ("hidden", C.c_uint32), ("intermediate", C.c_uint32),
                ("experts", C.c_uint32), ("top_k", C.c_uint32), ("shared_intermediate", C.c_uint32),
                ("out_f16", C.c_int32)]


MOE_PARTS = ("xq", "xs", "ids", "weights", "counts", "offsets", "n_tiles", "tiles", "perm", "inv", "pq", "ps",
             "mq", "ms", "y", "smq", "sms", "sy")


_lib = None


def build() -> str:
    """Compile libmpp41.so in-tree (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-C", PKG, "-j8"], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise MPP41Error(ERR_MISSING_KERNEL, f"{LIB_PATH} is not built; run make -C {PKG}")
    L = C.CDLL(LIB_PATH)
    vp, u32, st, sz = C.c_void_p, C.c_uint32, C.c_int, C.c_size_t
    sigs = {
        "mpp41_create": ([C.c_int, C.POINTER(vp)], st),
        "mpp41_destroy": ([vp], None),
        "mpp41_last_error": ([], C.c_char_p),
        "mpp41_status_string": ([st], C.c_char_p),
        "mpp41_device_name": ([vp, C.c_char_p, sz], st),
        "mpp41_set_stream": ([vp, vp], st),
        "mpp41_get_stream": ([vp], vp),
        "mpp41_synchronize": ([vp], st),
        "mpp41_device_error_word": ([vp], vp),
        "mpp41_set_trace": ([vp, vp, sz], st),
        "mpp41_alloc": ([vp, sz, C.POINTER(vp)], st),
        "mpp41_free": ([vp, vp], st),
        "mpp41_upload": ([vp, vp, vp, sz], st),
        "mpp41_download": ([vp, vp, vp, sz], st),
        "mpp41_memset": ([vp, vp, C.c_int, sz], st),
        "mpp41_has_kernel": ([C.c_char_p], C.c_int),
        "mpp41_roundtrip": ([vp, C.c_char_p, vp, vp, vp], st),
        "mpp41_pack": ([vp, C.c_int, vp, sz, vp], st),
        "mpp41_unpack": ([vp, C.c_int, vp, sz, vp], st),
        "mpp41_dequant": ([vp, C.c_char_p, vp, vp, vp, u32, u32], st),
        "mpp41_gemm": ([vp, C.c_char_p, vp, vp, vp, u32, u32, u32, vp], st),
        "mpp41_swiglu": ([vp, C.c_char_p, vp, vp, vp, C.POINTER(MLPConfig)], st),
        "mpp41_matmul_scalar": ([vp, C.c_char_p, vp, vp, vp, C.POINTER(MatmulConfig)], st),
        "mpp41_matmul_workspace_bytes": ([C.c_char_p, C.POINTER(MatmulConfig)], sz),
        "mpp41_matmul": ([vp, C.c_char_p, vp, vp, vp, C.POINTER(MatmulConfig), vp], st),
        "mpp41_mlp_scalar": ([vp, C.c_char_p, C.c_char_p, vp, vp, vp, vp, vp, vp, C.POINTER(MLPConfig)], st),
        "mpp41_mlp_scratch_bytes": ([C.POINTER(MLPDesc)], sz),
        "mpp41_mlp": ([vp, C.POINTER(MLPDesc)] + [vp] * 9, st),
        "mpp41_weight_create": ([vp, C.c_int32, vp, vp, u32, u32, C.POINTER(vp)], st),
        "mpp41_weight_destroy": ([vp], None),
        "mpp41_weight_map_counts": ([vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)], st),
        "mpp41_gemm_weight": ([vp, C.c_char_p, vp, vp, vp, u32], st),
        "mpp41_mlp_weights": ([vp, C.POINTER(MLPDesc), vp, vp, vp, vp, vp, vp], st),
        "mpp41_mlp_gate_up": ([vp, C.POINTER(MLPDesc)] + [vp] * 7, st),
        "mpp41_mlp_down": ([vp, C.POINTER(MLPDesc), vp, vp, vp, vp, C.c_int], st),
        "mpp41_quantize_mxfp4": ([vp, vp, u32, u32, vp, vp], st),
        "mpp41_quantize_act_mxfp4": ([vp, vp, u32, u32, vp, vp], st),
        "mpp41_quantize_act_s8": ([vp, vp, u32, u32, vp, vp], st),
        "mpp41_matmul_mxf4": ([vp] * 6 + [u32, u32, u32, C.c_int], st),
        "mpp41_mlp_w4a4_scratch_bytes": ([u32, u32, u32], sz),
        "mpp41_mlp_w4a4": ([vp, u32, u32, u32] + [vp] * 8 + [C.c_int, vp], st),
        "mpp41_quantize_nvfp4": ([vp, vp, u32, u32, vp, vp, vp], st),
        "mpp41_quantize_act_nvfp4": ([vp, vp, u32, u32, vp, vp, vp], st),
        "mpp41_matmul_nvf4": ([vp] * 8 + [u32, u32, u32, C.c_int], st),
        "mpp41_mlp_nvfp4_scratch_bytes": ([u32, u32, u32], sz),
        "mpp41_moe_scratch_layout": ([C.POINTER(MoEDesc), vp], sz),
        "mpp41_quantize_weights_int": ([vp, vp, u32, u32, C.c_int, vp, vp], st),
        "mpp41_mlp_w8a8_scratch_bytes": ([u32, u32, u32], sz),
        "mpp41_mlp_w8a8": ([vp, C.c_int, u32, u32, u32] + [vp] * 9, st),
        "mpp41_moe_route": ([vp, vp, u32, u32, u32, vp, vp], st),
        "mpp41_moe_w4a4": ([vp, C.POINTER(MoEDesc)] + [vp] * 16, st),
        "mpp41_moe_ep_scratch_layout": ([C.POINTER(MoEDesc), C.c_int, u32, vp], sz),
        "mpp41_moe_ep": ([vp, C.POINTER(MoEDesc), u32] + [vp] * 16, st),
        "mpp41_mlp_nvfp4": ([vp, u32, u32, u32] + [vp] * 11 + [C.c_int, vp], st),
        "mpp41_mlp_noalloc_scratch_bytes": ([C.POINTER(MLPDesc)], sz),
        "mpp41_mlp_noalloc": ([C.POINTER(MLPDesc)] + [vp] * 9, st),
        "mpp41_mlp_noalloc_status": ([vp], st),
        "mpp41_mlp_last_kernel": ([vp], C.c_char_p),
        "mpp41_wait_probe": ([vp, vp, C.c_uint32, C.c_uint64], st),
        "mpp41_mlp_describe": ([C.c_char_p, u32, u32, u32, C.POINTER(MLPDesc)], st),
        "mpp41_mlp_benchmark": ([vp, C.POINTER(MLPDesc)] + [vp] * 9 + [C.c_int, C.POINTER(C.c_double)], st),
        "mpp41_comm_unique_id": ([vp], st),
        "mpp41_comm_init": ([vp, C.c_int, C.c_int, vp], st),
        "mpp41_comm_destroy": ([vp], None),
        "mpp41_mlp_tp_scratch_bytes": ([C.POINTER(MLPDesc), C.c_int], sz),
        "mpp41_mlp_tp": ([vp, C.POINTER(MLPDesc)] + [vp] * 9, st),
    }
    for name, (args, res) in sigs.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def declared_symbols() -> list[str]:
    """Every function the public header declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mpp41_[a-z0-9_]+)\s*\(", text)))


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _check(status: int):
    if status != OK:
        msg = lib().mpp41_last_error()
        raise MPP41Error(status, msg.decode() if msg else "")


def w4a4_scratch_bytes(tokens: int, hidden: int, intermediate: int) -> int:
    return lib().mpp41_mlp_w4a4_scratch_bytes(tokens, hidden, intermediate)


def w4a4_scratch_layout(tokens: int, hidden: int, intermediate: int):
    """Byte offsets of (packed x, x scales, packed mid, mid scales) in the W4A4 scratch."""
    up = lambda n: (n + 255) & ~255
    o0 = 0
    o1 = o0 + up(tokens * hidden // 2)
    o2 = o1 + up(tokens * hidden // 32)
    o3 = o2 + up(tokens * intermediate // 2)
    return o0, o1, o2, o3


def nvfp4_scratch_bytes(tokens: int, hidden: int, intermediate: int) -> int:
    return lib().mpp41_mlp_nvfp4_scratch_bytes(tokens, hidden, intermediate)


def nvfp4_scratch_layout(tokens: int, hidden: int, intermediate: int):
    """Byte offsets of (packed x, x scales, fp16 mid, packed mid, mid scales, tensor scales) in the NVFP4 scratch."""
    up = lambda n: (n + 255) & ~255
    sizes = [tokens * hidden // 2, tokens * hidden // 16, tokens * intermediate * 2, tokens * intermediate // 2,
             tokens * intermediate // 16]
    offs, o = [], 0
    for n in sizes:
        offs.append(o)
        o += up(n)
    offs.append(o)
    return tuple(offs)


def moe_desc(tokens, hidden, intermediate, experts, top_k, shared_intermediate=0, out_f16=False) -> MoEDesc:
    return MoEDesc(tokens, hidden, intermediate, experts, top_k, shared_intermediate, int(out_f16))


def moe_scratch_layout(desc: MoEDesc):
    """(total bytes, {part name: byte offset}) of the MoE scratch."""
    offs = (C.c_size_t * len(MOE_PARTS))()
    total = lib().mpp41_moe_scratch_layout(C.byref(desc), offs)
    return total, dict(zip(MOE_PARTS, list(offs)))


def moe_ep_scratch_bytes(desc: MoEDesc, nranks: int, capacity: int) -> int:
    return lib().mpp41_moe_ep_scratch_layout(C.byref(desc), nranks, capacity, None)


def w8a8_scratch_bytes(tokens: int, hidden: int, intermediate: int) -> int:
    return lib().mpp41_mlp_w8a8_scratch_bytes(tokens, hidden, intermediate)


def w8a8_scratch_layout(tokens: int, hidden: int, intermediate: int):
    """Byte offsets of (int8 x, x scales, fp16 mid, int8 mid, mid scales) in the W8A8 scratch."""
    up = lambda n: (n + 255) & ~255
    offs, o = [], 0
    for n in (tokens * hidden, tokens * 4, tokens * intermediate * 2, tokens * intermediate, tokens * 4):
        offs.append(o)
        o += up(n)
    return tuple(offs)


def has_kernel(name: str) -> bool:
    return bool(lib().mpp41_has_kernel(name.encode()))


def describe(gate_kernel: str, tokens: int, hidden: int, intermediate: int) -> MLPDesc:
    d = MLPDesc()
    _check(lib().mpp41_mlp_describe(gate_kernel.encode(), tokens, hidden, intermediate, C.byref(d)))
    return d


def mlp_desc(tokens, hidden, intermediate, wfmt=W_MXFP4, afmt=A_F16, epilogue=SWIGLU_HALF, out_dtype=F32,
             flags=0) -> MLPDesc:
    return MLPDesc(tokens, hidden, intermediate, wfmt, afmt, epilogue, out_dtype, flags)


NOALLOC_SCRATCH_BYTES = 8 << 20
COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (rank 0 creates it and shares it)."""
    buf = (C.c_uint8 * COMM_ID_BYTES)()
    _check(lib().mpp41_comm_unique_id(buf))
    return bytes(buf)


def tp_scratch_bytes(desc: "MLPDesc", nranks: int) -> int:
    return lib().mpp41_mlp_tp_scratch_bytes(C.byref(desc), nranks)


def mlp_noalloc(desc: MLPDesc, x, wg, wu, wd, sg, su, sd, out, stream_handle=None):
    """One MLP layer with no device allocation and no context (mpp41_mlp_noalloc):
    for callers that may not allocate GPU memory. Uses the library's fixed static
    scratch; overlapping calls race."""
    _check(lib().mpp41_mlp_noalloc(C.byref(desc), _ptr(x), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su),
                                   _ptr(sd), _ptr(out), stream_handle))


def mlp_noalloc_status(stream_handle=None):
    """Waits for the stream, then raises MPP41Error if a no-alloc call recorded a
    device-side error (bounded wait ran out, bounds check); clears it."""
    _check(lib().mpp41_mlp_noalloc_status(stream_handle))


def scratch_bytes(desc: MLPDesc) -> int:
    return lib().mpp41_mlp_scratch_bytes(C.byref(desc))


class Weight:
    """Handle over a weight's device planes (mpp41_weight); keeps the planes
    referenced while it lives."""

    def __init__(self, h, planes):
        self.h = h
        self._planes = planes

    def map_counts(self):
        """(descriptors encoded, launches that reused one)."""
        e, r = C.c_uint64(), C.c_uint64()
        _check(lib().mpp41_weight_map_counts(self.h, C.byref(e), C.byref(r)))
        return e.value, r.value

    def close(self):
        if self.h:
            lib().mpp41_weight_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """One libmpp41 context (device + stream + device error word)."""

    def __init__(self, device: int = 0):
        L = lib()
        h = C.c_void_p()
        _check(L.mpp41_create(device, C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().mpp41_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- plumbing
    def device_name(self) -> str:
        buf = C.create_string_buffer(256)
        _check(lib().mpp41_device_name(self.h, buf, 256))
        return buf.value.decode()

    def set_stream(self, stream_handle: int | None):
        _check(lib().mpp41_set_stream(self.h, stream_handle))

    def synchronize(self):
        _check(lib().mpp41_synchronize(self.h))

    def set_trace(self, buf):
        """Per-CTA counters of the fused MLP kernel into `buf` (zeroed int64 CUDA tensor); None disables."""
        _check(lib().mpp41_set_trace(self.h, _ptr(buf), buf.numel() if buf is not None else 0))

    def error_word_ptr(self) -> int:
        return lib().mpp41_device_error_word(self.h)

    # -- kernels
    def roundtrip(self, kernel: str, inp, packed, out):
        _check(lib().mpp41_roundtrip(self.h, kernel.encode(), _ptr(inp), _ptr(packed), _ptr(out)))

    def pack(self, fmt: int, inp, n: int, packed):
        _check(lib().mpp41_pack(self.h, fmt, _ptr(inp), n, _ptr(packed)))

    def unpack(self, fmt: int, packed, n: int, out):
        _check(lib().mpp41_unpack(self.h, fmt, _ptr(packed), n, _ptr(out)))

    def dequant(self, kernel: str, packed, scales, out, rows: int, depth: int):
        _check(lib().mpp41_dequant(self.h, kernel.encode(), _ptr(packed), _ptr(scales), _ptr(out), rows, depth))

    def gemm(self, kernel: str, a, b, c, m: int, n: int, k: int, scales=None):
        _check(lib().mpp41_gemm(self.h, kernel.encode(), _ptr(a), _ptr(b), _ptr(c), m, n, k, _ptr(scales)))

    @staticmethod
    def matmul_workspace_bytes(kernel: str, rows: int, columns: int, depth: int) -> int:
        cfg = MatmulConfig(rows, columns, depth, 0)
        return lib().mpp41_matmul_workspace_bytes(kernel.encode(), C.byref(cfg))

    def matmul(self, kernel: str, a, b, c, rows: int, columns: int, depth: int, workspace=None):
        """Tensor-core big-matmul row (mpp41_matmul)."""
        cfg = MatmulConfig(rows, columns, depth, 0)
        _check(lib().mpp41_matmul(self.h, kernel.encode(), _ptr(a), _ptr(b), _ptr(c), C.byref(cfg), _ptr(workspace)))

    def swiglu(self, kernel: str, gate, up, mid, tokens: int, hidden: int, intermediate: int):
        cfg = MLPConfig(tokens, hidden, intermediate)
        _check(lib().mpp41_swiglu(self.h, kernel.encode(), _ptr(gate), _ptr(up), _ptr(mid), C.byref(cfg)))

    def matmul_scalar(self, kernel: str, a, b, c, rows: int, columns: int, depth: int):
        cfg = MatmulConfig(rows, columns, depth, depth // 2)
        _check(lib().mpp41_matmul_scalar(self.h, kernel.encode(), _ptr(a), _ptr(b), _ptr(c), C.byref(cfg)))

    def mlp_scalar(self, gate_kernel: str, down_kernel: str, x, wg, wu, mid, wd, out, tokens, hidden, intermediate):
        cfg = MLPConfig(tokens, hidden, intermediate)
        _check(lib().mpp41_mlp_scalar(self.h, gate_kernel.encode(), down_kernel.encode(), _ptr(x), _ptr(wg),
                                      _ptr(wu), _ptr(mid), _ptr(wd), _ptr(out), C.byref(cfg)))

    def mlp(self, desc: MLPDesc, x, wg, wu, wd, sg, su, sd, scratch, out):
        _check(lib().mpp41_mlp(self.h, C.byref(desc), _ptr(x), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su),
                               _ptr(sd), _ptr(scratch), _ptr(out)))

    def weight(self, wfmt: int, data, scales, k: int, n: int) -> "Weight":
        """A weight handle (mpp41_weight_create) over device planes data [n][k]
        and scales; the planes must outlive it."""
        h = C.c_void_p()
        _check(lib().mpp41_weight_create(self.h, wfmt, _ptr(data), _ptr(scales), k, n, C.byref(h)))
        return Weight(h, (data, scales))

    def gemm_weight(self, kernel: str, a, w: "Weight", c, m: int):
        _check(lib().mpp41_gemm_weight(self.h, kernel.encode(), _ptr(a), w.h, _ptr(c), m))

    def mlp_weights(self, desc: MLPDesc, x, wg: "Weight", wu: "Weight", wd: "Weight", scratch, out):
        _check(lib().mpp41_mlp_weights(self.h, C.byref(desc), _ptr(x), wg.h, wu.h, wd.h, _ptr(scratch), _ptr(out)))

    def wait_probe(self, flag, target: int, limit_ns: int):
        """Enqueue a bounded wait until *flag >= target (mpp41_wait_probe)."""
        _check(lib().mpp41_wait_probe(self.h, _ptr(flag), target, limit_ns))

    def mlp_last_kernel(self) -> str:
        """Kernel family the last mlp() call launched ("cluster", "gemv", ...)."""
        return lib().mpp41_mlp_last_kernel(self.h).decode()

    def mlp_gate_up(self, desc: MLPDesc, x, wg, wu, sg, su, scratch, out=None):
        _check(lib().mpp41_mlp_gate_up(self.h, C.byref(desc), _ptr(x), _ptr(wg), _ptr(wu), _ptr(sg), _ptr(su),
                                       _ptr(scratch), _ptr(out)))

    def mlp_down(self, desc: MLPDesc, scratch, wd, sd, out, prepared=False):
        _check(lib().mpp41_mlp_down(self.h, C.byref(desc), _ptr(scratch), _ptr(wd), _ptr(sd), _ptr(out),
                                    int(bool(prepared))))

    # ---- tensor parallelism (mpp41_comm_*, mpp41_mlp_tp)
    def comm_init(self, nranks: int, rank: int, unique_id: bytes):
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(unique_id)
        _check(lib().mpp41_comm_init(self.h, nranks, rank, buf))

    def comm_destroy(self):
        lib().mpp41_comm_destroy(self.h)

    def mlp_tp(self, desc: MLPDesc, x, wg, wu, wd, sg, su, sd, scratch, out):
        _check(lib().mpp41_mlp_tp(self.h, C.byref(desc), _ptr(x), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su),
                                  _ptr(sd), _ptr(scratch), _ptr(out)))

    def quantize_mxfp4(self, w, rows: int, depth: int, packed, scales):
        _check(lib().mpp41_quantize_mxfp4(self.h, _ptr(w), rows, depth, _ptr(packed), _ptr(scales)))

    def quantize_act_mxfp4(self, x, tokens: int, hidden: int, packed, scales):
        _check(lib().mpp41_quantize_act_mxfp4(self.h, _ptr(x), tokens, hidden, _ptr(packed), _ptr(scales)))

    def quantize_act_s8(self, x, tokens: int, hidden: int, q, scale):
        _check(lib().mpp41_quantize_act_s8(self.h, _ptr(x), tokens, hidden, _ptr(q), _ptr(scale)))

    def matmul_mxf4(self, a, sa, b, sb, c, M: int, N: int, K: int, c_f16: bool = False):
        """W4A4 GEMM: C[M][N] = A[M][K] B[N][K]^T, both MXFP4 (mpp41_matmul_mxf4)."""
        _check(lib().mpp41_matmul_mxf4(self.h, _ptr(a), _ptr(sa), _ptr(b), _ptr(sb), _ptr(c), M, N, K, int(c_f16)))

    def quantize_nvfp4(self, w, rows: int, depth: int, packed, scales, tensor_scale):
        """fp32 weights -> NVFP4 (mpp41_quantize_nvfp4); tensor_scale is a device float."""
        _check(lib().mpp41_quantize_nvfp4(self.h, _ptr(w), rows, depth, _ptr(packed), _ptr(scales), _ptr(tensor_scale)))

    def quantize_act_nvfp4(self, x, tokens: int, hidden: int, packed, scales, tensor_scale):
        _check(lib().mpp41_quantize_act_nvfp4(self.h, _ptr(x), tokens, hidden, _ptr(packed), _ptr(scales),
                                              _ptr(tensor_scale)))

    def matmul_nvf4(self, a, sa, ta, b, sb, tb, c, M: int, N: int, K: int, c_f16: bool = False):
        _check(lib().mpp41_matmul_nvf4(self.h, _ptr(a), _ptr(sa), _ptr(ta), _ptr(b), _ptr(sb), _ptr(tb), _ptr(c),
                                       M, N, K, int(c_f16)))

    def mlp_nvfp4(self, tokens: int, hidden: int, intermediate: int, x, wg, sg, tg, wu, su, tu, wd, sd, td, out,
                  scratch, out_f16: bool = False):
        """One NVFP4 W4A4 layer (mpp41_mlp_nvfp4); scratch of nvfp4_scratch_bytes()."""
        _check(lib().mpp41_mlp_nvfp4(self.h, tokens, hidden, intermediate, _ptr(x), _ptr(wg), _ptr(sg), _ptr(tg),
                                     _ptr(wu), _ptr(su), _ptr(tu), _ptr(wd), _ptr(sd), _ptr(td), _ptr(out),
                                     int(out_f16), _ptr(scratch)))

    def moe_route(self, logits, tokens: int, experts: int, top_k: int, ids, weights):
        _check(lib().mpp41_moe_route(self.h, _ptr(logits), tokens, experts, top_k, _ptr(ids), _ptr(weights)))

    def moe_w4a4(self, desc: "MoEDesc", x, logits, wg, sg, wu, su, wd, sd, out, scratch, shared=None):
        """One W4A4 mixture-of-experts layer (mpp41_moe_w4a4); shared = (wg, sg, wu, su, wd, sd) or None."""
        sh = [_ptr(v) for v in shared] if shared is not None else [None] * 6
        _check(lib().mpp41_moe_w4a4(self.h, C.byref(desc), _ptr(x), _ptr(logits), _ptr(wg), _ptr(sg), _ptr(wu),
                                    _ptr(su), _ptr(wd), _ptr(sd), *sh, _ptr(out), _ptr(scratch)))

    def moe_ep(self, desc: "MoEDesc", capacity: int, x, logits, wg, sg, wu, su, wd, sd, out, scratch, shared=None):
        """Expert-parallel MoE layer (mpp41_moe_ep) over this context's communicator; w* hold this rank's experts."""
        sh = [_ptr(v) for v in shared] if shared is not None else [None] * 6
        _check(lib().mpp41_moe_ep(self.h, C.byref(desc), capacity, _ptr(x), _ptr(logits), _ptr(wg), _ptr(sg),
                                  _ptr(wu), _ptr(su), _ptr(wd), _ptr(sd), *sh, _ptr(out), _ptr(scratch)))

    def quantize_weights_int(self, w, rows: int, depth: int, bits: int, packed, scales):
        """fp32 weights -> per-row symmetric INT8/INT4/INT2 + fp32 row scales (mpp41_quantize_weights_int)."""
        _check(lib().mpp41_quantize_weights_int(self.h, _ptr(w), rows, depth, bits, _ptr(packed), _ptr(scales)))

    def mlp_w8a8(self, wfmt: int, tokens: int, hidden: int, intermediate: int, x, wg, sg, wu, su, wd, sd, out, scratch):
        """Scaled W8A8 / W4A8 / W2A8 layer (mpp41_mlp_w8a8); scratch of w8a8_scratch_bytes()."""
        _check(lib().mpp41_mlp_w8a8(self.h, wfmt, tokens, hidden, intermediate, _ptr(x), _ptr(wg), _ptr(sg), _ptr(wu),
                                    _ptr(su), _ptr(wd), _ptr(sd), _ptr(out), _ptr(scratch)))

    def mlp_w4a4(self, tokens: int, hidden: int, intermediate: int, x, wg, sg, wu, su, wd, sd, out, scratch,
                 out_f16: bool = False):
        """One W4A4 MLP layer (mpp41_mlp_w4a4); scratch of w4a4_scratch_bytes()."""
        _check(lib().mpp41_mlp_w4a4(self.h, tokens, hidden, intermediate, _ptr(x), _ptr(wg), _ptr(sg), _ptr(wu),
                                    _ptr(su), _ptr(wd), _ptr(sd), _ptr(out), int(out_f16), _ptr(scratch)))

    def mlp_benchmark(self, desc: MLPDesc, x, wg, wu, wd, sg, su, sd, scratch, out, iterations: int) -> float:
        secs = C.c_double()
        _check(lib().mpp41_mlp_benchmark(self.h, C.byref(desc), _ptr(x), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg),
                                         _ptr(su), _ptr(sd), _ptr(scratch), _ptr(out), iterations,
                                         C.byref(secs)))
        return secs.value
