/*
 * libmpp41 -- C ABI of the B200 (sm_100a) quantized-weight MLP hot path.
 *
 * Drop-in boundary for the reference probe's Metal kernel ABI
 * (Sources/MetalFP41Probe/main.swift). The reference binds kernels by name
 * (library.makeFunction(name:), main.swift:208-212, 1730-1733, 1981-1989),
 * binds buffers by index (a=0, b=1, c=2, m=3, n=4, k=5, scales=6 for the
 * matmul2d kernels, main.swift:2151-2161 and 2734-2743) and runs every
 * iteration of a row in one command buffer (main.swift:2062-2121). Each entry
 * point below names the reference interface it replaces.
 *
 * Plain C: pointers and sizes only, no exceptions across the ABI. Device
 * pointers are CUDA global-memory addresses owned by the caller. Launches are
 * asynchronous on the context's stream; mpp41_synchronize() waits and turns
 * a device-side error word (bounded-wait timeout, bounds check) into a status.
 * Threading: one context per host thread (or per stream).
 */
#ifndef MPP41_H
#define MPP41_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MPP41_ABI_VERSION 1

/* Replaces the ProbeError cases of main.swift:5-38. */
typedef enum mpp41_status {
    MPP41_OK = 0,
    MPP41_ERR_INVALID_ARGUMENT = 1,  /* .invalidArgument */
    MPP41_ERR_UNSUPPORTED_SHAPE = 2, /* size gates of main.swift:390-392, 595-597, 946, 1043 */
    MPP41_ERR_NO_DEVICE = 3,         /* .missingDevice */
    MPP41_ERR_MISSING_KERNEL = 4,    /* .missingFunction: makeFunction(name:) == nil */
    MPP41_ERR_OUT_OF_MEMORY = 5,     /* .missingBuffer */
    MPP41_ERR_CUDA = 6,              /* .gpuExecutionFailed */
    MPP41_ERR_TIMEOUT = 7,           /* a bounded device-side wait ran out */
    MPP41_ERR_BOUNDS = 8,            /* device-side bounds check tripped */
    MPP41_ERR_COMM = 9               /* multi-GPU communication failure */
} mpp41_status;

/* Weight formats (the B operand of the reference's kernels). */
typedef enum mpp41_wfmt {
    MPP41_W_F16 = 0,    /* half [n][k] */
    MPP41_W_I8 = 1,     /* int8 [n][k] */
    MPP41_W_I4 = 2,     /* int4 [n][k/2], low nibble = even k, (n^8)-8 */
    MPP41_W_I2 = 3,     /* int2 [n][k/4], LSB pair first, ((b&3)^2)-2 */
    MPP41_W_FP4 = 4,    /* E2M1 [n][k/2], unscaled */
    MPP41_W_E4M3 = 5,   /* FP8 E4M3 [n][k] */
    MPP41_W_E5M2 = 6,   /* FP8 E5M2 [n][k] */
    MPP41_W_MXFP4 = 7,  /* E2M1 [n][k/2] + E8M0 scales [n][k/32] */
    MPP41_W_E4M3_MX = 8,/* FP8 E4M3 [n][k] + E8M0 scales [n][k/32] (MXFP8, BASELINE config 2; the
                           reference has unscaled FP8 rows only): each weight is
                           half(value * 2^(scale - 127)) */
    MPP41_W_E5M2_MX = 9 /* FP8 E5M2 [n][k] + E8M0 scales [n][k/32], as MPP41_W_E4M3_MX */
} mpp41_wfmt;

/* Activation (A operand) formats. */
typedef enum mpp41_afmt { MPP41_A_F16 = 0, MPP41_A_S8 = 1 } mpp41_afmt;

/* SwiGLU variants, MPPMLPKernels.metal:186-257. */
typedef enum mpp41_epilogue {
    MPP41_SWIGLU_FLOAT = 0,          /* mpp_mlp_swiglu_float: fp32 mid */
    MPP41_SWIGLU_HALF = 1,           /* mpp_mlp_swiglu_half: /16, clamp 20, fp16 mid */
    MPP41_SWIGLU_HALF_FROM_HALF = 2, /* mpp_mlp_swiglu_half_from_half: fp16 gate/up */
    MPP41_SWIGLU_I8 = 3,             /* mpp_mlp_swiglu_i8: int8 mid */
    MPP41_SWIGLU_FP32 = 4            /* silu(g) * u in fp32 without the /16 prescale, fp16 mid
                                        (no reference kernel) */
} mpp41_epilogue;

typedef enum mpp41_dtype { MPP41_F32 = 0, MPP41_F16 = 1, MPP41_S32 = 2, MPP41_S8 = 3 } mpp41_dtype;

/* MatmulConfig, main.swift:55-60 (PackedNumericKernels.metal:6-11). */
typedef struct mpp41_matmul_config {
    uint32_t rows, columns, depth, packed_depth_bytes;
} mpp41_matmul_config;

/* MLPConfig, main.swift:62-66 (PackedNumericKernels.metal:13-17). */
typedef struct mpp41_mlp_config {
    uint32_t tokens, hidden, intermediate;
} mpp41_mlp_config;

/* One MLP row: down(swiglu(gate(x), up(x))). */
typedef struct mpp41_mlp_desc {
    uint32_t tokens, hidden, intermediate;
    int32_t wfmt;      /* mpp41_wfmt of gate, up and down weights */
    int32_t afmt;      /* mpp41_afmt of x */
    int32_t epilogue;  /* mpp41_epilogue */
    int32_t out_dtype; /* mpp41_dtype of out: F32, F16 or S32 */
    uint32_t flags;    /* MPP41_MLP_* below */
} mpp41_mlp_desc;

/* Run the reference's four-dispatch structure (gate GEMM, up GEMM, SwiGLU
 * kernel, down GEMM) instead of the fused path; scratch then also holds
 * gate and up. */
#define MPP41_MLP_UNFUSED 0x1u
/* Per-output-channel fp16 scales (no reference counterpart):
 * with INT8 / INT4 / INT2 weights, sg, su and sd point to fp16 scales of the
 * gate rows [intermediate], up rows [intermediate] and down rows [hidden]; each
 * fp32 gate / up / down sum is multiplied by its row's scale before the SwiGLU
 * (gate, up) or the output (down). Runs on the fused kernels for fp16
 * activations and fp16-mid SwiGLU variants. */
#define MPP41_MLP_ROW_SCALES 0x2u

typedef struct mpp41_ctx mpp41_ctx;

/* ---- context: replaces MTLCreateSystemDefaultDevice + makeLibrary +
 *      makeCommandQueue (main.swift:90-105, 164-200) ---- */
mpp41_status mpp41_create(int device, mpp41_ctx **out);
void mpp41_destroy(mpp41_ctx *ctx);
/* Message of the last failing call on this host thread. */
const char *mpp41_last_error(void);
const char *mpp41_status_string(mpp41_status s);
/* "Device:" line of main.swift:95. */
mpp41_status mpp41_device_name(mpp41_ctx *ctx, char *buf, size_t len);
/* Launch on this cudaStream_t from now on. NULL selects the CUDA legacy
 * default stream; a new context starts on its own non-blocking stream. */
mpp41_status mpp41_set_stream(mpp41_ctx *ctx, void *cuda_stream);
void *mpp41_get_stream(mpp41_ctx *ctx);
/* Waits for the stream, then reports CUDA and device-side errors. */
mpp41_status mpp41_synchronize(mpp41_ctx *ctx);
/* Failure-path check of the bounded device waits (the counterpart of the
 * reference's command-buffer error check, main.swift:251-256): enqueues one
 * thread that waits, bounded by limit_ns (at most 10 s), until *flag >= target
 * -- the wait the layer kernels use for their grid-wide counters. If nothing
 * sets the flag in time the wait gives up, the kernel returns and the next
 * mpp41_synchronize reports MPP41_ERR_TIMEOUT; the context stays usable. */
mpp41_status mpp41_wait_probe(mpp41_ctx *ctx, const uint32_t *flag, uint32_t target, uint64_t limit_ns);
/* Device address of the context's 32-bit device error word. */
uint32_t *mpp41_device_error_word(mpp41_ctx *ctx);

/* Profiling aid with no reference counterpart: when `dev` is non-NULL, later
 * fused MLP launches of this context write 256 counters per CTA into it
 * (phase timestamps in ns, per-role wait/work SM cycles and per-stage SM
 * clock stamps, slots as enum TraceSlot in csrc/mpp41_mlp_fused.cuh; zero the
 * buffer first, sums accumulate). `words` >= 256 * number of SMs. NULL
 * disables. */
mpp41_status mpp41_set_trace(mpp41_ctx *ctx, unsigned long long *dev, size_t words);

/* ---- buffers: replace device.makeBuffer / contents() ---- */
mpp41_status mpp41_alloc(mpp41_ctx *ctx, size_t bytes, void **dev);
mpp41_status mpp41_free(mpp41_ctx *ctx, void *dev);
mpp41_status mpp41_upload(mpp41_ctx *ctx, void *dev, const void *host, size_t bytes);
mpp41_status mpp41_download(mpp41_ctx *ctx, void *host, const void *dev, size_t bytes);
mpp41_status mpp41_memset(mpp41_ctx *ctx, void *dev, int value, size_t bytes);

/* ---- kernel registry: makeFunction(name:) != nil (main.swift:949-950).
 *      Returns 1 if `name` (a reference kernel name) is implemented. ---- */
int mpp41_has_kernel(const char *name);

/* ---- packed formats: fp4_e2m1_roundtrip / fp8_e4m3_roundtrip /
 *      fp8_e5m2_roundtrip (PackedNumericKernels.metal:35-96; host driver
 *      run(testCase:) main.swift:202-262). in: 16 (E2M1) or 8 (FP8) floats;
 *      packed: 8 bytes; out: unpacked floats. ---- */
mpp41_status mpp41_roundtrip(mpp41_ctx *ctx, const char *kernel_name, const float *in, uint8_t *packed, float *out);
/* Bulk pack / unpack. fmt: 0 = E2M1 (2 per byte, low nibble first),
 * 1 = E4M3, 2 = E5M2. Round to nearest even, saturating. */
mpp41_status mpp41_pack(mpp41_ctx *ctx, int fmt, const float *in, size_t n, uint8_t *packed);
mpp41_status mpp41_unpack(mpp41_ctx *ctx, int fmt, const uint8_t *packed, size_t n, float *out);

/* ---- MXFP4 dequant: mxfp4_dequant_native_half / mxfp4_dequant_lut_half
 *      (MXFP4Kernels.metal:509-564; encodeMXFP4DequantMLP main.swift:2426-2469).
 *      out: fp16 [rows][depth]. ---- */
mpp41_status mpp41_dequant(mpp41_ctx *ctx, const char *kernel_name, const uint8_t *packed, const uint8_t *scales,
                           void *out_half, uint32_t rows, uint32_t depth);

/* ---- GEMM by reference kernel name: the matmul2d kernels of
 *      MPPMLPKernels.metal:39-184 and MXFP4Kernels.metal:108-296 with the
 *      encodeMPPMatmulDispatch / encodeMXFP4MatmulDispatch binding
 *      (main.swift:2137-2170, 2724-2752): c[m][n] = a[m][k] * b[n][k]^T.
 *      scales: [n][k/32] E8M0 for MXFP4 kernels, else NULL. ---- */
mpp41_status mpp41_gemm(mpp41_ctx *ctx, const char *kernel_name, const void *a, const void *b, void *c, uint32_t m,
                        uint32_t n, uint32_t k, const uint8_t *scales);

/* ---- Weight handles: replace the host-built multi-plane MTLTensor over a
 *      weight's packed values and scale plane (main.swift:2172-2212 builds it,
 *      2254-2262 binds it; MXFP4Kernels.metal:180-226 reads through it, the
 *      mxfp4_native_sph_* rows). A handle names the planes once -- format
 *      (mpp41_wfmt), packed data [n][k], scales (E8M0 [n][k/32] for block-scaled
 *      formats, fp16 [n] for MPP41_MLP_ROW_SCALES layers, else NULL) -- and keeps
 *      the TMA descriptors the kernels encode for them: a kernel's first launch
 *      through the handle encodes its box, later launches reuse it. The caller
 *      keeps ownership of the planes and must not free them before the handle;
 *      a handle belongs to the context's device. Calls through the same handle
 *      from several host threads are safe. ---- */
typedef struct mpp41_weight mpp41_weight;
mpp41_status mpp41_weight_create(mpp41_ctx *ctx, int32_t wfmt, const void *data, const uint8_t *scales, uint32_t k,
                                 uint32_t n, mpp41_weight **out);
void mpp41_weight_destroy(mpp41_weight *w);
/* Descriptors encoded for this handle so far, and launches that reused one. */
mpp41_status mpp41_weight_map_counts(const mpp41_weight *w, uint64_t *encoded, uint64_t *reused);
/* mpp41_gemm through a handle: c[m][n] = a[m][k] * w^T, kernel_name as for
 * mpp41_gemm (its weight format must be the handle's). */
mpp41_status mpp41_gemm_weight(mpp41_ctx *ctx, const char *kernel_name, const void *a, const mpp41_weight *w, void *c,
                               uint32_t m);
/* mpp41_mlp through handles: gate and up [intermediate][hidden], down
 * [hidden][intermediate], all of desc->wfmt; same kernels, results and scratch. */
mpp41_status mpp41_mlp_weights(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x, const mpp41_weight *wg,
                               const mpp41_weight *wu, const mpp41_weight *wd, void *scratch, void *out);

/* ---- OCP-MX quantizer (no reference counterpart: the reference draws random
 *      packed bytes, main.swift:2785-2793): fp32 w [rows][depth] ->
 *      E2M1 packed [rows][depth/2] + E8M0 scales [rows][depth/32], shared
 *      exponent floor(log2(amax)) - 2, elements round-to-nearest-even with
 *      saturation. depth % 32 == 0; w 16-byte aligned. ---- */
mpp41_status mpp41_quantize_mxfp4(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, uint8_t *packed,
                                  uint8_t *scales);

/* ---- SwiGLU by reference kernel name (mpp_mlp_swiglu_*,
 *      MPPMLPKernels.metal:186-257; encoder main.swift:2092-2100). ---- */
mpp41_status mpp41_swiglu(mpp41_ctx *ctx, const char *kernel_name, const void *gate, const void *up, void *mid,
                          const mpp41_mlp_config *cfg);

/* ---- scalar rows of PackedNumericKernels.metal (half serial accumulate):
 *      big matmul (runMatmulBenchmarkKernel main.swift:1715-1793) and the
 *      scalar MLP (encodeMLP main.swift:2575-2634). ---- */
mpp41_status mpp41_matmul_scalar(mpp41_ctx *ctx, const char *kernel_name, const void *a, const void *b, void *c,
                                 const mpp41_matmul_config *cfg);
/* Tensor-core formulation of the same big-matmul rows (kernel names of
 * mpp41_matmul_scalar, 2048^3 in BASELINE config 1): fp32 / int32 accumulation
 * in tensor memory and one final rounding for half outputs.
 * fp4_e2m1_matmul[_g8] (FP4 x FP4 -> fp32) and int4_int8_matmul (INT4 x INT4 ->
 * int32) are exact, hence equal to the reference; the half-output rows are the
 * exactly rounded sum, not the reference's serial-half-accumulate result.
 * `workspace` (mpp41_matmul_workspace_bytes) holds A widened to the MMA's
 * operand type for the rows whose A is FP4, INT4 or int8 (NULL when 0). */
size_t mpp41_matmul_workspace_bytes(const char *kernel_name, const mpp41_matmul_config *cfg);
mpp41_status mpp41_matmul(mpp41_ctx *ctx, const char *kernel_name, const void *a, const void *b, void *c,
                          const mpp41_matmul_config *cfg, void *workspace);

mpp41_status mpp41_mlp_scalar(mpp41_ctx *ctx, const char *gate_kernel_name, const char *down_kernel_name,
                              const void *x, const void *wg, const void *wu, void *mid, const void *wd, void *out,
                              const mpp41_mlp_config *cfg);

/* ---- the hot path: one MLP layer down(swiglu(gate(x), up(x))).
 *      Replaces encodeMPPMLP (main.swift:2636-2722) and encodeMXFP4FusedMLP
 *      (main.swift:2033-2135). Weights use the reference layouts ([n][k],
 *      scales [n][k/32]); sg/su/sd are only read for MXFP4. scratch must hold
 *      mpp41_mlp_scratch_bytes(desc) bytes: the fp16/fp32/int8 mid, then for
 *      fp16 output the split-K fp32 workspace and tile counters. Kernels by
 *      shape: up to 16 tokens with MXFP4/FP4/INT4 weights, hidden and
 *      intermediate multiples of 256 and at least 8M weights per matrix, one
 *      persistent weight-streaming kernel ("gemv"); other layers up to 32 tokens
 *      with those weights, two register-fed GEMV kernels ("gemv_regs"); 33..128 tokens of a small layer with 4-bit
 *      weights (hidden <= 1024), the small-layer kernel
 *      (one G and one D tile per CTA); otherwise one persistent tcgen05 kernel per layer
 *      (token-major for 65..128 tokens of a small layer, weight-major else).
 *      mpp41_mlp_last_kernel names the family the last mpp41_mlp call on the
 *      context launched: "gemv", "gemv_regs", "small", "token_major", "weight_major",
 *      "unfused" (two GEMM kernels) or "i8"; "" before the first call.
 *      MPP41_FUSED_PAIR=1 (read at each call) runs MXFP4 weight-major layers
 *      with full 128-token tiles as CTA pairs (tcgen05 cta_group::2, M = 256):
 *      same results within fp32 summation order, no faster on B200 so far. ---- */
const char *mpp41_mlp_last_kernel(const mpp41_ctx *ctx);
size_t mpp41_mlp_scratch_bytes(const mpp41_mlp_desc *desc);
mpp41_status mpp41_mlp(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x, const void *wg, const void *wu,
                       const void *wd, const uint8_t *sg, const uint8_t *su, const uint8_t *sd, void *scratch,
                       void *out);
/* The two stages of mpp41_mlp, for callers that place their own work (or a
 * collective) between them. mpp41_mlp_gate_up writes mid = swiglu(x Wg^T,
 * x Wu^T) to the start of `scratch` and clears what the split-K down
 * projection accumulates into (`out` for fp32 output, may be NULL otherwise).
 * mpp41_mlp_down computes out = mid Wd^T from the same scratch; pass
 * prepared = 1 when mpp41_mlp_gate_up ran before it on the same stream. */
mpp41_status mpp41_mlp_gate_up(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x, const void *wg,
                               const void *wu, const uint8_t *sg, const uint8_t *su, void *scratch, void *out);
mpp41_status mpp41_mlp_down(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, void *scratch, const void *wd,
                            const uint8_t *sd, void *out, int prepared);
/* Fill a descriptor from a reference gate/up kernel name (e.g.
 * "mxfp4_native_sp_h_f_n64", "mpp_mlp_h_i4_f_n128", "mpp_mlp_i8_i8_i32_n128")
 * with the SwiGLU and output type the reference pairs with it in
 * runMLPBenchmark (main.swift:945-1416). */
mpp41_status mpp41_mlp_describe(const char *gate_kernel_name, uint32_t tokens, uint32_t hidden,
                                uint32_t intermediate, mpp41_mlp_desc *desc);

/* Timed run: `iterations` back-to-back layers captured in one CUDA graph
 * (the analogue of one command buffer, main.swift:2062-2134); writes the GPU
 * seconds of the timed replay (CUDA events) after one untimed warm-up. */
mpp41_status mpp41_mlp_benchmark(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x, const void *wg,
                                 const void *wu, const void *wd, const uint8_t *sg, const uint8_t *su,
                                 const uint8_t *sd, void *scratch, void *out, int iterations, double *gpu_seconds);

/* ---- one MLP layer without any device allocation. No counterpart in the
 *      reference. For callers that may not call cudaMalloc (a host framework
 *      that owns every device allocation through its own pool, a plugin
 *      running while the process's allocator is locked): it needs no context
 *      and no scratch argument. Its scratch -- the fp16 mid, the fp32 split-K
 *      workspace, the kernel's counters -- is a fixed static device array of
 *      MPP41_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps
 *      until exit; layers needing more (mpp41_mlp_noalloc_scratch_bytes)
 *      are rejected with MPP41_ERR_UNSUPPORTED_SHAPE. Same math as mpp41_mlp
 *      for fp16 activations, packed weights (not MPP41_W_F16), fp16-mid SwiGLU
 *      variants and F32/F16 output. Launches on `cuda_stream` (NULL = legacy
 *      default stream) on the current device. The first call on a device looks
 *      up the static array's device address (cudaGetSymbolAddress); make that
 *      first call before any stream capture. All calls share the one array:
 *      calls that overlap on the GPU (other streams, other host threads) race
 *      and give wrong results -- serialise them. ---- */
#define MPP41_NOALLOC_SCRATCH_BYTES (8u << 20)
size_t mpp41_mlp_noalloc_scratch_bytes(const mpp41_mlp_desc *desc);
mpp41_status mpp41_mlp_noalloc(const mpp41_mlp_desc *desc, const void *x, const void *wg, const void *wu,
                               const void *wd, const uint8_t *sg, const uint8_t *su, const uint8_t *sd, void *out,
                               void *cuda_stream);
/* Device-side status of the no-alloc calls. The kernels record the first
 * bounded wait that ran out (MPP41_ERR_TIMEOUT) or bounds check that tripped
 * (MPP41_ERR_BOUNDS) in a static device word shared by all calls on the device;
 * mpp41_mlp_noalloc returns MPP41_OK once it has launched. This call waits for
 * `cuda_stream`, returns that recorded status (MPP41_OK when none) and clears
 * it. Allocates nothing. The cached device addresses stay valid for the life
 * of the CUDA context: do not use the no-alloc calls across cudaDeviceReset. */
mpp41_status mpp41_mlp_noalloc_status(void *cuda_stream);

/* ---- activation quantization (the epilogue after the layer, feeding the next
 *      layer's low-precision GEMM; no reference counterpart). fp16 x [tokens]
 *      [hidden]:
 *      - mpp41_quantize_act_mxfp4: OCP-MX MXFP4 per 32-wide block along hidden,
 *        same rule as mpp41_quantize_mxfp4 (W4A4 activations);
 *      - mpp41_quantize_act_s8: per-token symmetric int8 (W8A8 activations),
 *        scale[t] = absmax / 127, q = rint(x * 127 / absmax). ---- */
mpp41_status mpp41_quantize_act_mxfp4(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden, uint8_t *packed,
                                      uint8_t *scales);
mpp41_status mpp41_quantize_act_s8(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden, int8_t *q,
                                   float *scale);

/* ---- scaled integer layers W8A8 / W4A8 / W2A8 (the serving form of the
 *      reference's int8-activation rows, whose scales it leaves out):
 *      - mpp41_quantize_weights_int: fp32 [rows][depth] -> INT8/INT4/INT2 in the
 *        reference's packed layouts, per-row symmetric: scale = amax/qmax
 *        (qmax 127/7/1; 1 for a zero row), q = rint(w/scale) clamped to ±qmax;
 *      - mpp41_mlp_w8a8: x fp16 -> per-token int8 (mpp41_quantize_act_s8 rule),
 *        gate/up on kind::i8 (exact int32), dequant ((float)acc*sx[t])*sw[n],
 *        silu(g)*u -> fp16 mid, per-token int8 mid, down GEMM, dequant -> fp16
 *        out [T][H]. wfmt MPP41_W_I8/I4/I2; H, I % 128 == 0. scratch
 *        (mpp41_mlp_w8a8_scratch_bytes), 256-byte aligned sections: int8 x
 *        [T][H], x scales [T] fp32, fp16 mid [T][I], int8 mid [T][I], mid
 *        scales [T]. ---- */
mpp41_status mpp41_quantize_weights_int(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, int bits,
                                        void *packed, float *scales);
size_t mpp41_mlp_w8a8_scratch_bytes(uint32_t tokens, uint32_t hidden, uint32_t intermediate);
mpp41_status mpp41_mlp_w8a8(mpp41_ctx *ctx, int wfmt, uint32_t tokens, uint32_t hidden, uint32_t intermediate,
                            const void *x, const void *wg, const float *sg, const void *wu, const float *su,
                            const void *wd, const float *sd, void *out, void *scratch);

/* ---- device-time measurement on the context's stream (CUDA events):
 *      mpp41_timer_start records the start; mpp41_timer_stop records the end,
 *      waits for it and returns the seconds in between. ---- */
mpp41_status mpp41_timer_start(mpp41_ctx *ctx);
mpp41_status mpp41_timer_stop(mpp41_ctx *ctx, double *seconds);

/* ---- W4A4: activations as well as weights in MXFP4, multiplied on the FP4
 *      tensor cores with the E8M0 block scales applied inside the MMA (no
 *      reference counterpart: its FP4 rows keep fp16 activations; the weight
 *      layout is the reference's, docs/MXFP4-MPP41-GUIDE.md:43-55).
 *      - mpp41_matmul_mxf4: C[M][N] = A[M][K] B[N][K]^T, A and B packed E2M1
 *        [rows][K/2] with E8M0 scales [rows][K/32]; C fp32 (c_f16 = 0) or fp16.
 *        K % 512 == 0, N % 32 == 0, 16-byte aligned buffers.
 *      - mpp41_mlp_w4a4: one MLP layer. x (fp16 [T][H]) is quantized with the
 *        mpp41_quantize_act_mxfp4 rule; the gate/up GEMM's epilogue forms
 *        silu(g) * u in fp32 and quantizes it with the same rule; the down
 *        GEMM writes out [T][H] (fp32, or fp16 when out_f16). H % 512 == 0,
 *        I % 512 == 0. scratch (mpp41_mlp_w4a4_scratch_bytes) holds, each
 *        section 256-byte aligned: packed x [T][H/2], x scales [T][H/32],
 *        packed mid [T][I/2], mid scales [T][I/32]. ---- */
mpp41_status mpp41_matmul_mxf4(mpp41_ctx *ctx, const uint8_t *a, const uint8_t *sa, const uint8_t *b,
                               const uint8_t *sb, void *c, uint32_t M, uint32_t N, uint32_t K, int c_f16);
size_t mpp41_mlp_w4a4_scratch_bytes(uint32_t tokens, uint32_t hidden, uint32_t intermediate);
mpp41_status mpp41_mlp_w4a4(mpp41_ctx *ctx, uint32_t tokens, uint32_t hidden, uint32_t intermediate, const void *x,
                            const uint8_t *wg, const uint8_t *sg, const uint8_t *wu, const uint8_t *su,
                            const uint8_t *wd, const uint8_t *sd, void *out, int out_f16, void *scratch);

/* ---- NVFP4 (the reference emulates it, README.md:383-389): E2M1 elements,
 *      one UE4M3 scale per 16 along K, one fp32 tensor scale per tensor; on
 *      the FP4 tensor cores through kind::mxf4nvf4 (block16). Quantization
 *      (IEEE fp32, round to nearest even): g = amax(tensor) / 2688 (1 if
 *      zero); s = UE4M3((amax(block16) / 6) / g), saturating; element =
 *      E2M1(v * (1 / (decode(s) * g))) with one correctly rounded reciprocal
 *      per block; value = element * decode(s) * g.
 *      - mpp41_quantize_nvfp4 (fp32 weights) / mpp41_quantize_act_nvfp4 (fp16
 *        activations): packed [rows][depth/2], scales [rows][depth/16],
 *        *tensor_scale (device float) = g.
 *      - mpp41_matmul_nvf4: C = (A B^T) * ta * tb; K % 256, N % 32.
 *      - mpp41_mlp_nvfp4: one W4A4 layer with NVFP4 activations and weights
 *        (gate/up GEMM -> fp16 silu(g)*u -> NVFP4 -> down GEMM). H % 256,
 *        I % 256. scratch (mpp41_mlp_nvfp4_scratch_bytes), sections 256-byte
 *        aligned: packed x [T][H/2], x scales [T][H/16], fp16 mid [T][I],
 *        packed mid [T][I/2], mid scales [T][I/16], tensor scales {x, mid}. ---- */
mpp41_status mpp41_quantize_nvfp4(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, uint8_t *packed,
                                  uint8_t *scales, float *tensor_scale);
mpp41_status mpp41_quantize_act_nvfp4(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden,
                                      uint8_t *packed, uint8_t *scales, float *tensor_scale);
mpp41_status mpp41_matmul_nvf4(mpp41_ctx *ctx, const uint8_t *a, const uint8_t *sa, const float *ta,
                               const uint8_t *b, const uint8_t *sb, const float *tb, void *c, uint32_t M, uint32_t N,
                               uint32_t K, int c_f16);
size_t mpp41_mlp_nvfp4_scratch_bytes(uint32_t tokens, uint32_t hidden, uint32_t intermediate);
mpp41_status mpp41_mlp_nvfp4(mpp41_ctx *ctx, uint32_t tokens, uint32_t hidden, uint32_t intermediate, const void *x,
                             const uint8_t *wg, const uint8_t *sg, const float *tg, const uint8_t *wu,
                             const uint8_t *su, const float *tu, const uint8_t *wd, const uint8_t *sd,
                             const float *td, void *out, int out_f16, void *scratch);

/* ---- mixture of experts (no reference counterpart: the
 *      reference has one dense MLP). W4A4 experts on the FP4 tensor cores:
 *      route: logits [T][E] fp32 -> top_k expert ids (descending logit, ties to
 *        the lower id) and weights = softmax over the chosen logits (the full
 *        softmax renormalised over the top k);
 *      then x is quantized to MXFP4 once, its rows are grouped by expert
 *      (within an expert in token order), the grouped gate/up GEMM applies
 *      SwiGLU and re-quantizes the mid to MXFP4, the grouped down GEMM writes
 *      fp32 rows, and out[t] = shared_expert(x[t]) + sum_j w[t][j] * row(t, j),
 *      summed in slot order. Expert weights are stacked: wg/wu [E][I][H/2]
 *      (scales [E][I][H/32]), wd [E][H][I/2] (scales [E][H][I/32]); the
 *      optional shared expert (shared_intermediate > 0) uses one MLP's
 *      layout. H, I and shared_intermediate % 512 == 0; E % 32 == 0, E <= 512;
 *      1 <= top_k <= min(16, E). ---- */
typedef struct {
    uint32_t tokens, hidden, intermediate;
    uint32_t experts, top_k;
    uint32_t shared_intermediate;
    int32_t out_f16;
} mpp41_moe_desc;
enum {
    MPP41_MOE_XQ, MPP41_MOE_XS, MPP41_MOE_IDS, MPP41_MOE_WEIGHTS, MPP41_MOE_COUNTS, MPP41_MOE_OFFSETS,
    MPP41_MOE_NTILES, MPP41_MOE_TILES, MPP41_MOE_PERM, MPP41_MOE_INV, MPP41_MOE_PQ, MPP41_MOE_PS, MPP41_MOE_MQ,
    MPP41_MOE_MS, MPP41_MOE_Y, MPP41_MOE_SMQ, MPP41_MOE_SMS, MPP41_MOE_SY, MPP41_MOE_PARTS
};
/* Byte offsets of each scratch part (256-byte aligned) into offsets[MPP41_MOE_PARTS]
 * (may be NULL); returns the total scratch size. */
size_t mpp41_moe_scratch_layout(const mpp41_moe_desc *desc, size_t *offsets);
mpp41_status mpp41_moe_route(mpp41_ctx *ctx, const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                             int32_t *ids, float *weights);
mpp41_status mpp41_moe_w4a4(mpp41_ctx *ctx, const mpp41_moe_desc *desc, const void *x, const float *logits,
                            const uint8_t *wg, const uint8_t *sg, const uint8_t *wu, const uint8_t *su,
                            const uint8_t *wd, const uint8_t *sd, const uint8_t *shared_wg, const uint8_t *shared_sg,
                            const uint8_t *shared_wu, const uint8_t *shared_su, const uint8_t *shared_wd,
                            const uint8_t *shared_sd, void *out, void *scratch);

/* ---- expert parallelism: the same layer with the E experts split over the
 *      communicator's P ranks (mpp41_comm_init), rank r holding experts
 *      [r E/P, (r+1) E/P) (wg/wu/wd and scales stacked over those only) and
 *      its own `tokens` tokens. Each rank routes and groups its assignments,
 *      the per-expert counts are all-gathered (one host synchronisation
 *      sizes the exchanges), the quantized rows and scales go to the owning
 *      ranks (NCCL send/recv), the experts run on the rows received
 *      (regrouped expert-major), the fp32 rows come back the same way and
 *      each rank combines its own tokens. Every per-row computation and the
 *      combine order match mpp41_moe_w4a4, so the result is identical to it.
 *      capacity bounds the rows one rank may receive (P * tokens * top_k
 *      always suffices); scratch: mpp41_moe_ep_scratch_layout. ---- */
enum {
    MPP41_MOE_EP_ALLC, MPP41_MOE_EP_SEGS, MPP41_MOE_EP_TILES, MPP41_MOE_EP_NTILES, MPP41_MOE_EP_RQ,
    MPP41_MOE_EP_RS, MPP41_MOE_EP_GQ, MPP41_MOE_EP_GS, MPP41_MOE_EP_GMQ, MPP41_MOE_EP_GMS, MPP41_MOE_EP_GY,
    MPP41_MOE_EP_RY, MPP41_MOE_EP_PARTS
};
size_t mpp41_moe_ep_scratch_layout(const mpp41_moe_desc *desc, int nranks, uint32_t capacity, size_t *offsets);
mpp41_status mpp41_moe_ep(mpp41_ctx *ctx, const mpp41_moe_desc *desc, uint32_t capacity, const void *x,
                          const float *logits, const uint8_t *wg, const uint8_t *sg, const uint8_t *wu,
                          const uint8_t *su, const uint8_t *wd, const uint8_t *sd, const uint8_t *shared_wg,
                          const uint8_t *shared_sg, const uint8_t *shared_wu, const uint8_t *shared_su,
                          const uint8_t *shared_wd, const uint8_t *shared_sd, void *out, void *scratch);

/* ---- tensor parallelism (no counterpart in the
 *      single-GPU reference). Rank r of P holds rows [i0, i1) of the gate and
 *      up weights (and their scale rows) and the same columns of the down
 *      weights, repacked contiguous [H][i1-i0] (scales [H][(i1-i0)/32]). The
 *      slices: when I is a multiple of 512 with at least P units of 512, the
 *      units are dealt in order, the first I/512 mod P ranks taking one more
 *      (rank r starts at 512*(r*floor(I/512/P) + min(r, I/512 mod P))), so every
 *      slice keeps the 16-byte-aligned scale rows the fused kernels need;
 *      otherwise [r*I/P, (r+1)*I/P), which needs I a multiple of 32*P. Each
 *      rank computes its partial output with the fused layer kernel in fp32,
 *      then the partials are summed across ranks on the context's stream
 *      into `out` on every rank: for fp16 output of at least 2^20 elements an
 *      NCCL reduce-scatter of the fp32 partials, each rank's share rounded to
 *      fp16 and an fp16 all-gather (MPP41_TP_REDUCE=allreduce asks for the
 *      other form), otherwise an NCCL all-reduce. NCCL is loaded at run time
 *      (libnccl.so.2); without it mpp41_comm_init fails with MPP41_ERR_COMM. ---- */
#define MPP41_COMM_ID_BYTES 128
/* Rank 0 creates the id and shares it with the other ranks (any channel). */
mpp41_status mpp41_comm_unique_id(uint8_t id[MPP41_COMM_ID_BYTES]);
/* Collective over all ranks; binds the communicator to the context's device. */
/* Before mpp41_comm_destroy, destroy any CUDA graph that captured
 * mpp41_mlp_tp or mpp41_moe_ep calls: NCCL keeps resources for captured
 * operations until their graph is destroyed. mpp41_mlp_tp sums the partials
 * with NCCL; MPP41_TP_ALLREDUCE=oneshot selects a one-shot all-reduce over
 * CUDA-IPC-mapped peer buffers (bounded waits, same sum order on every rank)
 * for partials up to 2 MiB. */
mpp41_status mpp41_comm_init(mpp41_ctx *ctx, int nranks, int rank, const uint8_t id[MPP41_COMM_ID_BYTES]);
void mpp41_comm_destroy(mpp41_ctx *ctx);
/* Scratch of one rank for the global layer `desc` split over `nranks`. */
size_t mpp41_mlp_tp_scratch_bytes(const mpp41_mlp_desc *desc, int nranks);
/* `desc` describes the global layer; weights are this rank's shards. */
mpp41_status mpp41_mlp_tp(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x, const void *wg_shard,
                          const void *wu_shard, const void *wd_shard, const uint8_t *sg_shard,
                          const uint8_t *su_shard, const uint8_t *sd_shard, void *scratch, void *out);

#ifdef __cplusplus
}
#endif
#endif /* MPP41_H */
