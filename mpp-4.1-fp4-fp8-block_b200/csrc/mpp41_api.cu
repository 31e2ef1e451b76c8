// C ABI of libmpp41 (include/mpp41.h): context, buffers, the kernel registry
// keyed by the reference's kernel names, and the MLP orchestration.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>
#include <string>

#include "../../include/mpp41.h"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"


namespace {

thread_local std::string g_last_error;

mpp41_status fail(mpp41_status s, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

mpp41_status cuda_fail(cudaError_t e, const char *what)
{
    return fail(MPP41_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                                   \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

#define NEED(ctx)                                                              \
    do {                                                                       \
        if (!(ctx)) return fail(MPP41_ERR_INVALID_ARGUMENT, "null context");   \
    } while (0)

// ---------------------------------------------------------------- registry
enum Kind { K_ROUNDTRIP, K_DEQUANT, K_GEMM, K_SWIGLU, K_SCALAR_MM, K_SCALAR_GU, K_SCALAR_DOWN };

struct KernelInfo {
    const char *name;
    Kind kind;
    int arg0;   // roundtrip fmt / dequant lut / gemm wfmt / swiglu kind / scalar kind or wfmt
    int arg1;   // gemm: output epilogue (EPI_STORE_F32 / EPI_STORE_F16)
    int afmt;   // gemm: activation format (0 fp16, 1 int8, 2 fp32)
};

using namespace mpp41;

const KernelInfo kKernels[] = {
    // PackedNumericKernels.metal:35-96
    {"fp4_e2m1_roundtrip", K_ROUNDTRIP, 0, 0, 0},
    {"fp8_e4m3_roundtrip", K_ROUNDTRIP, 1, 0, 0},
    {"fp8_e5m2_roundtrip", K_ROUNDTRIP, 2, 0, 0},
    // MXFP4Kernels.metal:509-564
    {"mxfp4_dequant_native_half", K_DEQUANT, 0, 0, 0},
    {"mxfp4_dequant_lut_half", K_DEQUANT, 1, 0, 0},
    // MPPMLPKernels.metal:39-161 (fp16 activations)
    {"mpp_mlp_h_h_f_n128", K_GEMM, W_F16, EPI_STORE_F32, 0},
    {"mpp_mlp_h_i8_f_n128", K_GEMM, W_I8, EPI_STORE_F32, 0},
    {"mpp_mlp_h_i4_f_n128", K_GEMM, W_I4, EPI_STORE_F32, 0},
    {"mpp_mlp_h_fp4_f_n128", K_GEMM, W_FP4, EPI_STORE_F32, 0},
    {"mpp_mlp_h_fp8e4m3_f_n128", K_GEMM, W_E4M3, EPI_STORE_F32, 0},
    {"mpp_mlp_h_fp8e4m3_h_n128", K_GEMM, W_E4M3, EPI_STORE_F16, 0},
    {"mpp_mlp_h_fp8e5m2_f_n128", K_GEMM, W_E5M2, EPI_STORE_F32, 0},
    {"mpp_mlp_h_i2_f_n128", K_GEMM, W_I2, EPI_STORE_F32, 0},
    // int8 activations, exact int32 accumulate (MPPMLPKernels.metal:61, 140, 152)
    {"mpp_mlp_i8_i8_i32_n128", K_GEMM, W_I8, 0, 1},
    {"mpp_mlp_i8_i4_i32_n128", K_GEMM, W_I4, 0, 1},
    {"mpp_mlp_i8_i2_i32_n128", K_GEMM, W_I2, 0, 1},
    // fp32 activations (the swiglu_float mid) x half / INT8 weights (MPPMLPKernels.metal:164, 175)
    {"mpp_mlp_f_h_f_n128", K_GEMM, W_F16, EPI_STORE_F32, 2},
    {"mpp_mlp_f_i8_f_n128", K_GEMM, W_I8, EPI_STORE_F32, 2},
    // MXFP4Kernels.metal:108-296, 361-383: one B200 kernel serves every
    // strategy the reference compares (the math is identical)
    {"mxfp4_fused_h_f_n128", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_fused_h_f_n64", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_native_sp_h_f_n128", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_native_sp_h_f_n64", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_native_sph_h_f_n64", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_fused_ci_h_f_sg_k64", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    {"mxfp4_fused_ci_h_f_sg_k32", K_GEMM, W_MXFP4, EPI_STORE_F32, 0},
    // MPPMLPKernels.metal:186-257
    {"mpp_mlp_swiglu_float", K_SWIGLU, 0, 0, 0},
    {"mpp_mlp_swiglu_half", K_SWIGLU, 1, 0, 0},
    {"mpp_mlp_swiglu_half_from_half", K_SWIGLU, 2, 0, 0},
    {"mpp_mlp_swiglu_i8", K_SWIGLU, 3, 0, 0},
    // PackedNumericKernels.metal:98-423 (big matmul scalar rows)
    {"fp4_e2m1_matmul_benchmark", K_SCALAR_MM, 0, 0, 0},
    {"fp4_e2m1_matmul_g8_benchmark", K_SCALAR_MM, 0, 0, 0},
    {"half_fp4_matmul_half_benchmark", K_SCALAR_MM, 1, 0, 0},
    {"half_fp4_matmul_half_g8_benchmark", K_SCALAR_MM, 1, 0, 0},
    {"half_int4_matmul_half_benchmark", K_SCALAR_MM, 2, 0, 0},
    {"int8_half_matmul_half_benchmark", K_SCALAR_MM, 3, 0, 0},
    {"int4_int8_matmul_benchmark", K_SCALAR_MM, 4, 0, 0},
    // PackedNumericKernels.metal:425-832 (scalar MLP rows)
    {"half_mlp_gate_up_benchmark", K_SCALAR_GU, W_F16, 0, 0},
    {"half_int8_mlp_gate_up_benchmark", K_SCALAR_GU, W_I8, 0, 0},
    {"half_int4_mlp_gate_up_benchmark", K_SCALAR_GU, W_I4, 0, 0},
    {"half_int2_mlp_gate_up_benchmark", K_SCALAR_GU, W_I2, 0, 0},
    {"half_fp4_mlp_gate_up_benchmark", K_SCALAR_GU, W_FP4, 0, 0},
    {"half_fp4_mlp_gate_up_g8_benchmark", K_SCALAR_GU, W_FP4, 0, 0},
    {"half_mlp_down_benchmark", K_SCALAR_DOWN, W_F16, 0, 0},
    {"half_int8_mlp_down_benchmark", K_SCALAR_DOWN, W_I8, 0, 0},
    {"half_int4_mlp_down_benchmark", K_SCALAR_DOWN, W_I4, 0, 0},
    {"half_int2_mlp_down_benchmark", K_SCALAR_DOWN, W_I2, 0, 0},
    {"half_fp4_mlp_down_benchmark", K_SCALAR_DOWN, W_FP4, 0, 0},
    {"half_fp4_mlp_down_g8_benchmark", K_SCALAR_DOWN, W_FP4, 0, 0},
};

const KernelInfo *find_kernel(const char *name)
{
    if (!name) return nullptr;
    for (const KernelInfo &k : kKernels)
        if (strcmp(k.name, name) == 0) return &k;
    return nullptr;
}

mpp41_status missing(const char *name)
{
    return fail(MPP41_ERR_MISSING_KERNEL, "libmpp41 does not contain kernel %s", name ? name : "(null)");
}

uint32_t pick_splits(uint32_t tiles, uint32_t K)
{
    // enough CTAs to cover the 148 SMs; each split keeps >= 256 of K
    uint32_t s = 1;
    while (tiles * s * 2 <= 160 && (K % (64 * s * 2)) == 0 && K / (s * 2) >= 256) s *= 2;
    return s;
}

int mid_bytes_per_elem(int epilogue)
{
    return epilogue == MPP41_SWIGLU_FLOAT ? 4 : (epilogue == MPP41_SWIGLU_I8 ? 1 : 2);
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// split-K factor of the down projection (1 = plain store)
uint32_t down_splits(const mpp41_mlp_desc *d)
{
    return pick_splits((d->hidden / 64) * ((d->tokens + 127) / 128), d->intermediate);
}

LayerPlan desc_plan(const mpp41_mlp_desc *d)
{
    return plan_layer(d->tokens, d->hidden, d->intermediate, d->out_dtype == MPP41_F16, d->wfmt);
}

// Scratch layout: [mid][fp32 workspace T x H][tile counters] for the
// two-kernel path (the last two only for fp16 output). The fused kernel uses
// [mid][splits x T x H fp32 partials] over the same bytes; the total covers
// both.
struct ScratchLayout {
    size_t mid_bytes, ws_off, ws_bytes, cnt_off, cnt_bytes, total;
};

ScratchLayout scratch_layout(const mpp41_mlp_desc *d)
{
    ScratchLayout L{};
    L.mid_bytes = (size_t)d->tokens * d->intermediate * mid_bytes_per_elem(d->epilogue);
    L.ws_off = align256(L.mid_bytes);
    if (d->out_dtype == MPP41_F16) {
        L.ws_bytes = (size_t)d->tokens * d->hidden * 4;
        L.cnt_off = L.ws_off + L.ws_bytes;
        L.cnt_bytes = ((size_t)(d->hidden / 64) * ((d->tokens + 127) / 128) * 4 + 15) & ~size_t(15);
    } else {
        L.cnt_off = L.ws_off;
    }
    L.total = L.cnt_off + L.cnt_bytes;
    const size_t fused = L.ws_off + desc_plan(d).ws_bytes;
    if (fused > L.total) L.total = fused;
    return L;
}

mpp41_status check_mlp_desc(const mpp41_mlp_desc *d)
{
    if (!d) return fail(MPP41_ERR_INVALID_ARGUMENT, "null descriptor");
    if (!d->tokens || !d->hidden || !d->intermediate)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "MLP sizes must be positive");
    if (d->hidden % 64 || d->intermediate % 64)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden and intermediate must be multiples of 64 (got %u, %u)",
                    d->hidden, d->intermediate);
    if (d->wfmt < 0 || d->wfmt > MPP41_W_E5M2_MX) return fail(MPP41_ERR_INVALID_ARGUMENT, "bad weight format %d", d->wfmt);
    return MPP41_OK;
}

mpp41_status check_fp16_row(const mpp41_mlp_desc *d)
{
    if (d->afmt != MPP41_A_F16)
        return fail(MPP41_ERR_MISSING_KERNEL, "int8-activation MLP rows are not available in this build");
    if (d->epilogue == MPP41_SWIGLU_I8)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "swiglu_i8 needs int8 activations");
    if (d->epilogue == MPP41_SWIGLU_FLOAT && ((d->wfmt != MPP41_W_F16 && d->wfmt != MPP41_W_I8) || d->out_dtype != MPP41_F32))
        return fail(MPP41_ERR_MISSING_KERNEL,
                    "the fp32-mid rows (swiglu_float, then mpp_mlp_f_*_f) take half or INT8 weights and fp32 output");
    if (d->epilogue < 0 || d->epilogue > MPP41_SWIGLU_FP32)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "bad epilogue %d", d->epilogue);
    if (d->out_dtype != MPP41_F32 && d->out_dtype != MPP41_F16)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "output dtype %d not valid for fp16-activation rows", d->out_dtype);
    return MPP41_OK;
}

int gate_up_epi(int epilogue)
{
    switch (epilogue) {
    case MPP41_SWIGLU_HALF: return EPI_SWIGLU_HALF;
    case MPP41_SWIGLU_FP32: return EPI_SWIGLU_PLAIN;
    case MPP41_SWIGLU_FLOAT: return EPI_SWIGLU_FLOAT;
    default: return EPI_SWIGLU_HALF_H;
    }
}

// Split-K factor of the int8 GEMM: enough 128x128 tiles to cover the SMs, each
// split keeping >= 256 of K.
uint32_t i8_splits(uint32_t m, uint32_t n, uint32_t k)
{
    const uint32_t tiles = ((n + 127) / 128) * ((m + 127) / 128);
    uint32_t s = 1;
    while (tiles * s * 2 <= 160 && k % (128 * s * 2) == 0 && k / (s * 2) >= 256) s *= 2;
    return s;
}

// C int32 [m][n] = A int8 [m][k] x W[n][k] on `st` (clears C first when split).
mpp41_status enqueue_i8_gemm(mpp41_ctx *ctx, int wfmt, const void *a, const void *w, void *c, uint32_t m,
                             uint32_t n, uint32_t k, cudaStream_t st, const char *what)
{
    I8Launch L{};
    L.wfmt = wfmt;
    L.a = a; L.b0 = w; L.out = c;
    L.M = m; L.N = n; L.K = k; L.ldc = n;
    L.err = ctx->err;
    L.splits = i8_splits(m, n, k);
    L.epi = L.splits > 1 ? 1 : 0;
    if (L.splits > 1) CK(cudaMemsetAsync(c, 0, (size_t)m * n * 4, st), "zero output");
    const char *why = "";
    const int rc = launch_i8_gemm(L, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "%s: %s", what, why);
    return MPP41_OK;
}

// C fp32 [m][n] = A fp32 [m][k] x W[n][k] (half or INT8) on `st`; clears C
// first when split.
mpp41_status enqueue_f32_gemm(mpp41_ctx *ctx, int wfmt, const void *a, const void *w, void *c, uint32_t m,
                              uint32_t n, uint32_t k, cudaStream_t st, const char *what)
{
    F32Launch L{};
    L.wfmt = wfmt;
    L.a = static_cast<const float *>(a); L.b = w; L.out = static_cast<float *>(c);
    L.M = m; L.N = n; L.K = k; L.ldc = n;
    L.err = ctx->err;
    const uint32_t tiles = ((n + 127) / 128) * ((m + 127) / 128);
    L.splits = 1;
    while (tiles * L.splits * 2 <= 160 && k % (32 * L.splits * 2) == 0 && k / (L.splits * 2) >= 256) L.splits *= 2;
    if (L.splits > 1) CK(cudaMemsetAsync(c, 0, (size_t)m * n * 4, st), "zero output");
    const char *why = "";
    const int rc = launch_f32_gemm(L, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "%s: %s", what, why);
    return MPP41_OK;
}

// int8-activation rows (W8A8 / W4A8 / W2A8): the gate/up pair GEMM ends in
// mpp_mlp_swiglu_i8 (int8 mid in scratch), the down GEMM writes int32.
bool is_i8_row(const mpp41_mlp_desc *d) { return d->afmt == MPP41_A_S8; }

// MXFP8 weights or per-output-channel scales: only the
// small-layer kernel computes them.
bool is_scaled_row(const mpp41_mlp_desc *d)
{
    return d->wfmt == MPP41_W_E4M3_MX || d->wfmt == MPP41_W_E5M2_MX || (d->flags & MPP41_MLP_ROW_SCALES);
}

mpp41_status check_scaled_row(const mpp41_mlp_desc *d, const void *sg, const void *su, const void *sd)
{
    if (!is_scaled_row(d)) return MPP41_OK;
    if (d->flags & MPP41_MLP_ROW_SCALES) {
        if (d->wfmt != MPP41_W_I8 && d->wfmt != MPP41_W_I4 && d->wfmt != MPP41_W_I2)
            return fail(MPP41_ERR_INVALID_ARGUMENT, "MPP41_MLP_ROW_SCALES needs INT8, INT4 or INT2 weights");
    }
    if (!sg || !su || !sd) return fail(MPP41_ERR_INVALID_ARGUMENT, "scaled weights need gate, up and down scales");
    if (d->afmt != MPP41_A_F16 || d->epilogue == MPP41_SWIGLU_FLOAT || d->epilogue == MPP41_SWIGLU_I8 ||
        (d->flags & MPP41_MLP_UNFUSED))
        return fail(MPP41_ERR_MISSING_KERNEL,
                    "MXFP8 weights and per-row scales run on the fused small-layer kernel only (fp16 "
                    "activations, an fp16-mid SwiGLU)");
    if (d->tokens <= 32 || !sl::covers(d->tokens, d->hidden, d->intermediate, d->wfmt))
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE,
                    "MXFP8 weights and per-row scales run on the small-layer kernel: 33..128 tokens, hidden <= 1024 "
                    "(a multiple of the stage K), intermediate a multiple of 8 stages (MXFP8: hidden 1024, "
                    "intermediate 4096); got %u x %u x %u", d->tokens, d->hidden, d->intermediate);
    return MPP41_OK;
}

mpp41_status check_i8_row(const mpp41_mlp_desc *d)
{
    if (d->epilogue != MPP41_SWIGLU_I8 || d->out_dtype != MPP41_S32)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "int8-activation rows use the swiglu_i8 epilogue and int32 output");
    if (d->wfmt != MPP41_W_I8 && d->wfmt != MPP41_W_I4 && d->wfmt != MPP41_W_I2)
        return fail(MPP41_ERR_MISSING_KERNEL, "int8-activation rows take INT8, INT4 or INT2 weights");
    return MPP41_OK;
}

mpp41_status enqueue_i8_gate_up(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg,
                                const void *wu, void *scratch, cudaStream_t st)
{
    I8Launch L{};
    L.wfmt = d->wfmt;
    L.epi = 2;
    L.a = x; L.b0 = wg; L.b1 = wu; L.out = scratch;
    L.M = d->tokens; L.N = d->intermediate; L.K = d->hidden; L.ldc = d->intermediate;
    L.splits = 1;
    L.err = ctx->err;
    const char *why = "";
    const int rc = launch_i8_gemm(L, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "int8 gate/up GEMM: %s", why);
    return MPP41_OK;
}

// Stage 1: mid = swiglu(x Wg^T, x Wu^T) into scratch; clears the split-K
// accumulation target of stage 2 (out for fp32, the workspace for fp16).
mpp41_status enqueue_gate_up(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg, const void *wu,
                             const uint8_t *sg, const uint8_t *su, void *scratch, void *out, cudaStream_t st)
{
    if (is_i8_row(d)) {
        mpp41_status s = check_i8_row(d);
        return s ? s : enqueue_i8_gate_up(ctx, d, x, wg, wu, scratch, st);
    }
    mpp41_status s = check_fp16_row(d);
    if (s) return s;
    if (is_scaled_row(d))
        return fail(MPP41_ERR_MISSING_KERNEL, "MXFP8 weights and per-row scales run through mpp41_mlp only");
    if (d->wfmt == MPP41_W_MXFP4 && (!sg || !su))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "MXFP4 needs gate and up scales");
    const ScratchLayout SL = scratch_layout(d);
    WqLaunch g{};
    g.wfmt = d->wfmt;
    g.epi = gate_up_epi(d->epilogue);
    g.a = x; g.b0 = wg; g.b1 = wu; g.s0 = sg; g.s1 = su;
    g.out = scratch;
    g.M = d->tokens; g.N = d->intermediate; g.K = d->hidden; g.ldc = d->intermediate;
    g.err = ctx->err;
    if (down_splits(d) > 1 && d->epilogue != MPP41_SWIGLU_FLOAT) {   // the fp32-mid down GEMM clears its own output
        if (d->out_dtype == MPP41_F32 && out) {
            g.zero = out;
            g.zero_bytes = (size_t)d->tokens * d->hidden * 4;
        } else if (d->out_dtype == MPP41_F16) {
            g.zero = static_cast<uint8_t *>(scratch) + SL.ws_off;
            g.zero_bytes = SL.ws_bytes + SL.cnt_bytes;
        }
    }
    const char *why = "";
    const int rc = launch_wq_gemm(g, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "gate/up GEMM: %s", why);
    return MPP41_OK;
}

// Stage 2: out = mid Wd^T. Unless `prepared`, clears its split-K target first.
mpp41_status enqueue_down(mpp41_ctx *ctx, const mpp41_mlp_desc *d, void *scratch, const void *wd, const uint8_t *sd,
                          void *out, bool prepared, cudaStream_t st)
{
    if (is_i8_row(d)) {
        mpp41_status s = check_i8_row(d);
        return s ? s : enqueue_i8_gemm(ctx, d->wfmt, scratch, wd, out, d->tokens, d->hidden, d->intermediate, st,
                                       "int8 down GEMM");
    }
    mpp41_status s = check_fp16_row(d);
    if (s) return s;
    if (d->epilogue == MPP41_SWIGLU_FLOAT)   // fp32 mid: mpp_mlp_f_h_f_n128 / mpp_mlp_f_i8_f_n128
        return enqueue_f32_gemm(ctx, d->wfmt, scratch, wd, out, d->tokens, d->hidden, d->intermediate, st,
                                "fp32-mid down GEMM");
    if (is_scaled_row(d))
        return fail(MPP41_ERR_MISSING_KERNEL, "MXFP8 weights and per-row scales run through mpp41_mlp only");
    if (d->wfmt == MPP41_W_MXFP4 && !sd) return fail(MPP41_ERR_INVALID_ARGUMENT, "MXFP4 needs down scales");
    const ScratchLayout SL = scratch_layout(d);
    WqLaunch dn{};
    dn.wfmt = d->wfmt;
    dn.a = scratch; dn.b0 = wd; dn.s0 = sd;
    dn.out = out;
    dn.M = d->tokens; dn.N = d->hidden; dn.K = d->intermediate; dn.ldc = d->hidden;
    dn.err = ctx->err;
    dn.splits = down_splits(d);
    if (d->out_dtype == MPP41_F32) {
        dn.epi = dn.splits > 1 ? EPI_ATOMIC_F32 : EPI_STORE_F32;
        if (dn.splits > 1 && !prepared) CK(cudaMemsetAsync(out, 0, (size_t)d->tokens * d->hidden * 4, st), "clear");
    } else {
        dn.epi = dn.splits > 1 ? EPI_SPLITK_F16 : EPI_STORE_F16;
        if (dn.splits > 1) {
            dn.ws = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + SL.ws_off);
            dn.tile_count = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(scratch) + SL.cnt_off);
            if (!prepared) CK(cudaMemsetAsync(dn.ws, 0, SL.ws_bytes + SL.cnt_bytes, st), "clear workspace");
        }
    }
    const char *why = "";
    const int rc = launch_wq_gemm(dn, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "down GEMM: %s", why);
    return MPP41_OK;
}

// Enqueue one MLP layer on `st`. Preferred: the single persistent kernel
// (mpp41_mlp_fused.cuh). Otherwise, or with MPP41_MLP_UNFUSED: two kernels,
// the first also clearing what the split-K second one accumulates into.
mpp41_status enqueue_mlp(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg, const void *wu,
                         const void *wd, const uint8_t *sg, const uint8_t *su, const uint8_t *sd, void *scratch,
                         void *out, cudaStream_t st)
{
    if (is_i8_row(d)) {
        mpp41_status s = check_i8_row(d);
        if (!s) s = enqueue_i8_gate_up(ctx, d, x, wg, wu, scratch, st);
        if (!s) s = enqueue_i8_gemm(ctx, d->wfmt, scratch, wd, out, d->tokens, d->hidden, d->intermediate, st,
                                    "int8 down GEMM");
        if (!s) snprintf(ctx->last_mlp_kernel, sizeof(ctx->last_mlp_kernel), "i8");
        return s;
    }
    mpp41_status s = check_fp16_row(d);
    if (s) return s;
    if (d->wfmt == MPP41_W_MXFP4 && (!sg || !su || !sd))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "MXFP4 needs gate, up and down scales");
    s = check_scaled_row(d, sg, su, sd);
    if (s) return s;
    const bool scaled = is_scaled_row(d);
    const char *declined = nullptr, *declined_kernel = "";
    if (!(d->flags & MPP41_MLP_UNFUSED) && d->wfmt != MPP41_W_F16 && d->epilogue != MPP41_SWIGLU_FLOAT &&
        desc_plan(d).sync_words <= ctx->sync_words) {
        const ScratchLayout SL = scratch_layout(d);
        FusedLaunch L{};
        L.wfmt = d->wfmt;
        L.gate_epi = gate_up_epi(d->epilogue);
        L.out_f16 = d->out_dtype == MPP41_F16;
        L.x = x; L.wg = wg; L.wu = wu; L.wd = wd; L.sg = sg; L.su = su; L.sd = sd;
        L.mid = scratch;
        L.out = out;
        L.ws = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + SL.ws_off);
        L.sync = ctx->sync;
        L.err = ctx->err;
        L.T = d->tokens; L.H = d->hidden; L.I = d->intermediate;
        L.trace = ctx->trace;
        L.row_scales = (d->flags & MPP41_MLP_ROW_SCALES) != 0;
        const char *why = "";
        const LayerPlan plan = desc_plan(d);
        const int rc = launch_layer(plan, L, st, &why);
        if (rc == 0) {
            snprintf(ctx->last_mlp_kernel, sizeof(ctx->last_mlp_kernel), "%s",
                     layer_kernel_name(plan, L.T, L.H, L.I, L.wfmt));
            return MPP41_OK;
        }
        if (rc == 2) return fail(MPP41_ERR_CUDA, "fused MLP kernel: %s", why);
        if (scaled) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "small-layer kernel declined: %s", why);
        declined = why;
        declined_kernel = layer_kernel_name(plan, L.T, L.H, L.I, L.wfmt);
    }
    s = enqueue_gate_up(ctx, d, x, wg, wu, sg, su, scratch, out, st);
    if (s) return s;
    s = enqueue_down(ctx, d, scratch, wd, sd, out, true, st);
    if (!s) {
        if (declined)
            snprintf(ctx->last_mlp_kernel, sizeof(ctx->last_mlp_kernel), "unfused (%s kernel declined: %s)",
                     declined_kernel, declined);
        else
            snprintf(ctx->last_mlp_kernel, sizeof(ctx->last_mlp_kernel), "unfused");
    }
    return s;
}

}  // namespace

extern "C" {

const char *mpp41_last_error(void) { return g_last_error.c_str(); }

const char *mpp41_status_string(mpp41_status s)
{
    switch (s) {
    case MPP41_OK: return "ok";
    case MPP41_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MPP41_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case MPP41_ERR_NO_DEVICE: return "no device";
    case MPP41_ERR_MISSING_KERNEL: return "missing kernel";
    case MPP41_ERR_OUT_OF_MEMORY: return "out of memory";
    case MPP41_ERR_CUDA: return "CUDA error";
    case MPP41_ERR_TIMEOUT: return "device wait timed out";
    case MPP41_ERR_BOUNDS: return "device bounds check";
    case MPP41_ERR_COMM: return "communication error";
    }
    return "unknown status";
}

mpp41_status mpp41_create(int device, mpp41_ctx **out)
{
    if (!out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null output pointer");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(MPP41_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= n) return fail(MPP41_ERR_NO_DEVICE, "device %d out of range (%d devices)", device, n);
    CK(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(MPP41_ERR_NO_DEVICE, "libmpp41 is built for sm_100a (B200); device is sm_%d%d", prop.major,
                    prop.minor);
    mpp41_ctx *c = new mpp41_ctx();
    c->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->err, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&c->amax, sizeof(uint32_t));
    c->sync_words = 1u << 16;
    if (e == cudaSuccess) e = cudaMalloc(&c->sync, c->sync_words * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c->sync, 0, c->sync_words * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaEventCreate(&c->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&c->ev1);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "context setup");
    }
    c->stream = c->own_stream;
    *out = c;
    return MPP41_OK;
}

void mpp41_destroy(mpp41_ctx *ctx)
{
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->err);
    cudaFree(ctx->amax);
    cudaFree(ctx->sync);
    cudaEventDestroy(ctx->ev0);
    cudaEventDestroy(ctx->ev1);
    mpp41::comm_release(ctx);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
}

mpp41_status mpp41_device_name(mpp41_ctx *ctx, char *buf, size_t len)
{
    NEED(ctx);
    if (!buf || !len) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, ctx->device), "cudaGetDeviceProperties");
    snprintf(buf, len, "%s", prop.name);
    return MPP41_OK;
}

mpp41_status mpp41_set_stream(mpp41_ctx *ctx, void *s)
{
    NEED(ctx);
    ctx->stream = static_cast<cudaStream_t>(s);
    return MPP41_OK;
}

void *mpp41_get_stream(mpp41_ctx *ctx) { return ctx ? ctx->stream : nullptr; }

uint32_t *mpp41_device_error_word(mpp41_ctx *ctx) { return ctx ? ctx->err : nullptr; }

constexpr unsigned kTraceWords = 256;   // TraceSlot kTraceSlots of the fused kernel

mpp41_status mpp41_set_trace(mpp41_ctx *ctx, unsigned long long *dev, size_t words)
{
    NEED(ctx);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    if (dev && words < (size_t)kTraceWords * sms)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "trace buffer needs %u words per SM", kTraceWords);
    ctx->trace = dev;
    return MPP41_OK;
}

mpp41_status mpp41_wait_probe(mpp41_ctx *ctx, const uint32_t *flag, uint32_t target, uint64_t limit_ns)
{
    NEED(ctx);
    if (!flag) return fail(MPP41_ERR_INVALID_ARGUMENT, "null flag");
    if (limit_ns == 0 || limit_ns > 10000000000ull)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "limit must be in (0, 10 s]");
    CK(launch_wait_probe(flag, target, limit_ns, ctx->err, ctx->stream), "wait probe launch");
    return MPP41_OK;
}

const char *mpp41_mlp_last_kernel(const mpp41_ctx *ctx) { return ctx ? ctx->last_mlp_kernel : ""; }

mpp41_status mpp41_synchronize(mpp41_ctx *ctx)
{
    NEED(ctx);
    CK(cudaStreamSynchronize(ctx->stream), "stream synchronize");
    uint32_t w = 0;
    CK(cudaMemcpy(&w, ctx->err, sizeof(w), cudaMemcpyDeviceToHost), "read device error word");
    if (w) {
        cudaMemset(ctx->err, 0, sizeof(uint32_t));
        // a kernel that gave up may have left grid counters mid-count
        cudaMemset(ctx->sync, 0, ctx->sync_words * sizeof(uint32_t));
        const uint32_t code = w & 0xFFFFu, site = w >> 16;
        return fail(code == 7 ? MPP41_ERR_TIMEOUT : code == 8 ? MPP41_ERR_BOUNDS : MPP41_ERR_CUDA,
                    "device-side error code %u at site 0x%x", code, site);
    }
    return MPP41_OK;
}

mpp41_status mpp41_alloc(mpp41_ctx *ctx, size_t bytes, void **dev)
{
    NEED(ctx);
    if (!dev) return fail(MPP41_ERR_INVALID_ARGUMENT, "null output pointer");
    if (cudaMalloc(dev, bytes ? bytes : 1) != cudaSuccess) {
        cudaGetLastError();
        return fail(MPP41_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu) failed", bytes);
    }
    return MPP41_OK;
}

mpp41_status mpp41_free(mpp41_ctx *ctx, void *dev)
{
    NEED(ctx);
    CK(cudaFree(dev), "cudaFree");
    return MPP41_OK;
}

mpp41_status mpp41_upload(mpp41_ctx *ctx, void *dev, const void *host, size_t bytes)
{
    NEED(ctx);
    CK(cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, ctx->stream), "upload");
    CK(cudaStreamSynchronize(ctx->stream), "upload sync");
    return MPP41_OK;
}

mpp41_status mpp41_download(mpp41_ctx *ctx, void *host, const void *dev, size_t bytes)
{
    NEED(ctx);
    CK(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, ctx->stream), "download");
    CK(cudaStreamSynchronize(ctx->stream), "download sync");
    return MPP41_OK;
}

mpp41_status mpp41_memset(mpp41_ctx *ctx, void *dev, int value, size_t bytes)
{
    NEED(ctx);
    CK(cudaMemsetAsync(dev, value, bytes, ctx->stream), "memset");
    return MPP41_OK;
}

int mpp41_has_kernel(const char *name) { return find_kernel(name) ? 1 : 0; }

mpp41_status mpp41_roundtrip(mpp41_ctx *ctx, const char *name, const float *in, uint8_t *packed, float *out)
{
    NEED(ctx);
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_ROUNDTRIP) return missing(name);
    if (!in || !packed || !out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_roundtrip(k->arg0, in, packed, out, ctx->stream), name);
    return MPP41_OK;
}

mpp41_status mpp41_pack(mpp41_ctx *ctx, int fmt, const float *in, size_t n, uint8_t *packed)
{
    NEED(ctx);
    if (fmt < 0 || fmt > 2) return fail(MPP41_ERR_INVALID_ARGUMENT, "format %d", fmt);
    if (!n) return MPP41_OK;
    if (!in || !packed) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_pack(fmt, in, n, packed, ctx->stream), "pack");
    return MPP41_OK;
}

mpp41_status mpp41_unpack(mpp41_ctx *ctx, int fmt, const uint8_t *packed, size_t n, float *out)
{
    NEED(ctx);
    if (fmt < 0 || fmt > 2) return fail(MPP41_ERR_INVALID_ARGUMENT, "format %d", fmt);
    if (!n) return MPP41_OK;
    if (!packed || !out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_unpack(fmt, packed, n, out, ctx->stream), "unpack");
    return MPP41_OK;
}

mpp41_status mpp41_dequant(mpp41_ctx *ctx, const char *name, const uint8_t *packed, const uint8_t *scales,
                           void *out, uint32_t rows, uint32_t depth)
{
    NEED(ctx);
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_DEQUANT) return missing(name);
    if (depth % 32) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "depth must be a multiple of 32");
    if (!rows || !depth) return MPP41_OK;
    if (!packed || !scales || !out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if ((reinterpret_cast<uintptr_t>(packed) & 7u) || (reinterpret_cast<uintptr_t>(out) & 15u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "packed must be 8-byte and out 16-byte aligned");
    CK(launch_dequant(k->arg0, packed, scales, out, rows, depth, ctx->stream), name);
    return MPP41_OK;
}

mpp41_status mpp41_gemm(mpp41_ctx *ctx, const char *name, const void *a, const void *b, void *c, uint32_t m,
                        uint32_t n, uint32_t k, const uint8_t *scales)
{
    NEED(ctx);
    const KernelInfo *ki = find_kernel(name);
    if (!ki || ki->kind != K_GEMM) return missing(name);
    if (!a || !b || !c) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (ki->arg0 == W_MXFP4 && !scales) return fail(MPP41_ERR_INVALID_ARGUMENT, "MXFP4 kernel needs scales");
    if (!m || !n || !k) return MPP41_OK;
    if (ki->afmt == 1) return enqueue_i8_gemm(ctx, ki->arg0, a, b, c, m, n, k, ctx->stream, name);
    if (ki->afmt == 2) return enqueue_f32_gemm(ctx, ki->arg0, a, b, c, m, n, k, ctx->stream, name);
    if (k % 64 || n % 64) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "n and k must be multiples of 64");
    WqLaunch L{};
    L.wfmt = ki->arg0;
    L.a = a; L.b0 = b; L.s0 = scales; L.out = c;
    L.M = m; L.N = n; L.K = k; L.ldc = n;
    L.err = ctx->err;
    L.epi = ki->arg1;
    if (ki->arg1 == EPI_STORE_F32) {
        const uint32_t tiles = (n / 64) * ((m + 127) / 128);
        L.splits = pick_splits(tiles, k);
        if (L.splits > 1) {
            L.epi = EPI_ATOMIC_F32;
            CK(cudaMemsetAsync(c, 0, (size_t)m * n * 4, ctx->stream), "zero output");
        }
    }
    const char *why = "";
    const int rc = launch_wq_gemm(L, ctx->stream, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "%s: %s", name, why);
    return MPP41_OK;
}

size_t mpp41_matmul_workspace_bytes(const char *name, const mpp41_matmul_config *cfg)
{
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_SCALAR_MM || !cfg) return 0;
    const size_t mk = (size_t)cfg->rows * cfg->depth;
    switch (k->arg0) {
    case 0: case 3: return 2 * mk;   // A widened to fp16
    case 4: return mk;               // A widened to int8
    default: return 0;
    }
}

mpp41_status mpp41_matmul(mpp41_ctx *ctx, const char *name, const void *a, const void *b, void *c,
                          const mpp41_matmul_config *cfg, void *workspace)
{
    NEED(ctx);
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_SCALAR_MM) return missing(name);
    if (!cfg || !a || !b || !c) return fail(MPP41_ERR_INVALID_ARGUMENT, "null argument");
    const uint32_t m = cfg->rows, n = cfg->columns, kk = cfg->depth;
    if (!m || !n || !kk) return MPP41_OK;
    if (kk % 128 || n % 64) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "depth must be a multiple of 128, columns of 64");
    const size_t ws = mpp41_matmul_workspace_bytes(name, cfg);
    if (ws && !workspace) return fail(MPP41_ERR_INVALID_ARGUMENT, "%s needs a %zu-byte workspace", name, ws);
    cudaStream_t st = ctx->stream;
    const int kind = k->arg0;
    if (kind == 0 || kind == 3) CK(launch_widen(kind == 0 ? 0 : 1, a, (size_t)m * kk, workspace, st), "widen A");
    if (kind == 4) {
        CK(launch_widen(2, a, (size_t)m * kk, workspace, st), "widen A");
        return enqueue_i8_gemm(ctx, W_I4, workspace, b, c, m, n, kk, st, name);
    }
    const void *a16 = (kind == 0 || kind == 3) ? workspace : a;
    if (kind <= 2 && n % 128 == 0 && 2 + (size_t)(n / 128 + 1) * ((m + 127) / 128 + 1) <= ctx->sync_words) {
        // weight-major tensor-core path: the fused layer kernel's down tiles as a
        // plain GEMM (weights decoded into tensor memory, tokens as N)
        FusedLaunch F{};
        F.wfmt = kind == 2 ? W_I4 : W_FP4;
        F.gate_epi = EPI_SWIGLU_PLAIN;
        F.out_f16 = kind != 0;
        F.mid = const_cast<void *>(a16);
        F.wd = b; F.out = c;
        F.sync = ctx->sync; F.err = ctx->err; F.trace = nullptr;
        F.T = m; F.H = n; F.I = kk; F.splits = 1;
        F.gemm_only = true;
        const char *fwhy = "";
        const int frc = launch_mlp_fused(F, st, &fwhy);
        if (frc == 0) return MPP41_OK;
        if (frc == 2) return fail(MPP41_ERR_CUDA, "%s: %s", name, fwhy);
    }
    WqLaunch L{};
    L.a = a16;
    L.b0 = b; L.out = c;
    L.M = m; L.N = n; L.K = kk; L.ldc = n;
    L.err = ctx->err;
    L.wfmt = kind == 0 ? W_FP4 : kind == 1 ? W_FP4 : kind == 2 ? W_I4 : W_F16;
    L.epi = kind == 0 ? EPI_STORE_F32 : EPI_STORE_F16;
    const char *why = "";
    const int rc = launch_wq_gemm(L, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "%s: %s", name, why);
    return MPP41_OK;
}

mpp41_status mpp41_swiglu(mpp41_ctx *ctx, const char *name, const void *gate, const void *up, void *mid,
                          const mpp41_mlp_config *cfg)
{
    NEED(ctx);
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_SWIGLU) return missing(name);
    if (!cfg || !gate || !up || !mid) return fail(MPP41_ERR_INVALID_ARGUMENT, "null argument");
    const size_t n = (size_t)cfg->tokens * cfg->intermediate;
    if (!n) return MPP41_OK;
    CK(launch_swiglu(k->arg0, gate, up, mid, n, ctx->stream), name);
    return MPP41_OK;
}

mpp41_status mpp41_matmul_scalar(mpp41_ctx *ctx, const char *name, const void *a, const void *b, void *c,
                                 const mpp41_matmul_config *cfg)
{
    NEED(ctx);
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_SCALAR_MM) return missing(name);
    if (!cfg || !a || !b || !c) return fail(MPP41_ERR_INVALID_ARGUMENT, "null argument");
    if (cfg->depth % 16) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "Matmul K/depth must be a multiple of 16");
    CK(launch_scalar_matmul(k->arg0, cfg->rows, cfg->columns, cfg->depth, a, b, c, ctx->stream), name);
    return MPP41_OK;
}

mpp41_status mpp41_mlp_scalar(mpp41_ctx *ctx, const char *gate_name, const char *down_name, const void *x,
                              const void *wg, const void *wu, void *mid, const void *wd, void *out,
                              const mpp41_mlp_config *cfg)
{
    NEED(ctx);
    const KernelInfo *g = find_kernel(gate_name), *d = find_kernel(down_name);
    if (!g || g->kind != K_SCALAR_GU) return missing(gate_name);
    if (!d || d->kind != K_SCALAR_DOWN) return missing(down_name);
    if (g->arg0 != d->arg0) return fail(MPP41_ERR_INVALID_ARGUMENT, "gate and down kernels use different formats");
    if (!cfg) return fail(MPP41_ERR_INVALID_ARGUMENT, "null config");
    if (cfg->hidden % 16 || cfg->intermediate % 16)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE,
                    "MLP hidden and intermediate sizes must be multiples of 16 for packed FP4 weights.");
    CK(launch_scalar_mlp(g->arg0, cfg->tokens, cfg->hidden, cfg->intermediate, x, wg, wu, mid, wd, out, ctx->stream),
       gate_name);
    return MPP41_OK;
}

size_t mpp41_mlp_scratch_bytes(const mpp41_mlp_desc *d)
{
    if (!d || !d->tokens || !d->hidden || !d->intermediate) return 0;
    return scratch_layout(d).total;
}

mpp41_status mpp41_mlp_describe(const char *name, uint32_t T, uint32_t H, uint32_t I, mpp41_mlp_desc *d)
{
    if (!d) return fail(MPP41_ERR_INVALID_ARGUMENT, "null descriptor");
    const KernelInfo *k = find_kernel(name);
    if (!k || k->kind != K_GEMM) return missing(name);
    memset(d, 0, sizeof(*d));
    d->tokens = T; d->hidden = H; d->intermediate = I;
    d->wfmt = k->arg0;
    d->afmt = k->afmt == 1 ? MPP41_A_S8 : MPP41_A_F16;
    // runMLPBenchmark pairings (main.swift:945-1416): half and INT8 weights use
    // swiglu_float; the FP8 half-destination row uses swiglu_half_from_half and
    // a half output; int8 activations use swiglu_i8 and int32 output; the rest
    // use swiglu_half with fp32 output.
    if (k->afmt == 1) { d->epilogue = MPP41_SWIGLU_I8; d->out_dtype = MPP41_S32; }
    else if (k->arg1 == EPI_STORE_F16) { d->epilogue = MPP41_SWIGLU_HALF_FROM_HALF; d->out_dtype = MPP41_F16; }
    else if (k->arg0 == W_F16 || k->arg0 == W_I8) { d->epilogue = MPP41_SWIGLU_FLOAT; d->out_dtype = MPP41_F32; }
    else { d->epilogue = MPP41_SWIGLU_HALF; d->out_dtype = MPP41_F32; }
    return MPP41_OK;
}

mpp41_status mpp41_mlp(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg, const void *wu,
                       const void *wd, const uint8_t *sg, const uint8_t *su, const uint8_t *sd, void *scratch,
                       void *out)
{
    NEED(ctx);
    mpp41_status s = check_mlp_desc(d);
    if (s) return s;
    if (!x || !wg || !wu || !wd || !scratch || !out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    return enqueue_mlp(ctx, d, x, wg, wu, wd, sg, su, sd, scratch, out, ctx->stream);
}

mpp41_status mpp41_mlp_gate_up(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg,
                               const void *wu, const uint8_t *sg, const uint8_t *su, void *scratch, void *out)
{
    NEED(ctx);
    mpp41_status s = check_mlp_desc(d);
    if (s) return s;
    if (!x || !wg || !wu || !scratch) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    return enqueue_gate_up(ctx, d, x, wg, wu, sg, su, scratch, out, ctx->stream);
}

mpp41_status mpp41_mlp_down(mpp41_ctx *ctx, const mpp41_mlp_desc *d, void *scratch, const void *wd,
                            const uint8_t *sd, void *out, int prepared)
{
    NEED(ctx);
    mpp41_status s = check_mlp_desc(d);
    if (s) return s;
    if (!scratch || !wd || !out) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    return enqueue_down(ctx, d, scratch, wd, sd, out, prepared != 0, ctx->stream);
}

mpp41_status mpp41_quantize_mxfp4(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, uint8_t *packed,
                                  uint8_t *scales)
{
    NEED(ctx);
    if (depth % 32) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "depth must be a multiple of 32");
    if (!rows || !depth) return MPP41_OK;
    if (!w || !packed || !scales) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 15u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "w and packed must be 16-byte aligned");
    CK(launch_quantize_mxfp4(w, rows, depth, packed, scales, ctx->stream), "quantize");
    return MPP41_OK;
}

mpp41_status mpp41_quantize_act_mxfp4(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden, uint8_t *packed,
                                      uint8_t *scales)
{
    NEED(ctx);
    if (hidden % 32) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden must be a multiple of 32");
    if (!tokens || !hidden) return MPP41_OK;
    if (!x || !packed || !scales) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 15u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "x and packed must be 16-byte aligned");
    CK(launch_quantize_mxfp4_f16(x, tokens, hidden, packed, scales, ctx->stream), "quantize activations");
    return MPP41_OK;
}

mpp41_status mpp41_quantize_act_s8(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden, int8_t *q,
                                   float *scale)
{
    NEED(ctx);
    if (!tokens || !hidden) return MPP41_OK;
    if (!x || !q || !scale) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_quantize_act_s8(x, tokens, hidden, q, scale, ctx->stream), "quantize activations");
    return MPP41_OK;
}

// ------------------------------------------------------------------ timer
mpp41_status mpp41_timer_start(mpp41_ctx *ctx)
{
    NEED(ctx);
    CK(cudaEventRecord(ctx->ev0, ctx->stream), "timer start");
    return MPP41_OK;
}

mpp41_status mpp41_timer_stop(mpp41_ctx *ctx, double *seconds)
{
    NEED(ctx);
    if (!seconds) return fail(MPP41_ERR_INVALID_ARGUMENT, "null seconds");
    float ms = 0.0f;
    CK(cudaEventRecord(ctx->ev1, ctx->stream), "timer stop");
    CK(cudaEventSynchronize(ctx->ev1), "timer stop");
    CK(cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1), "timer stop");
    *seconds = ms * 1e-3;
    return MPP41_OK;
}

// ------------------------------------------------------------------ W4A4
static bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static size_t up256(size_t n) { return (n + 255) & ~size_t(255); }

static mpp41_status enqueue_mxf4(mpp41_ctx *ctx, const MxLaunch &L, const char *what)
{
    const char *why = "";
    const int rc = launch_mxf4_gemm(L, ctx->stream, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "%s: %s", what, why);
    return MPP41_OK;
}

mpp41_status mpp41_matmul_mxf4(mpp41_ctx *ctx, const uint8_t *a, const uint8_t *sa, const uint8_t *b,
                               const uint8_t *sb, void *c, uint32_t M, uint32_t N, uint32_t K, int c_f16)
{
    NEED(ctx);
    if (!M || !N || !K) return MPP41_OK;
    if (!a || !sa || !b || !sb || !c) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(a) || !al16(sa) || !al16(b) || !al16(sb) || !al16(c))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "buffers must be 16-byte aligned");
    MxLaunch L{};
    L.a = a; L.sa = sa;
    L.b0 = L.b1 = b; L.sb0 = L.sb1 = sb;
    L.b_rows = N;
    L.out = c; L.M = M; L.N = N; L.K = K; L.ldc = N;
    L.epi = c_f16 ? 1 : 0;
    L.err = ctx->err;
    return enqueue_mxf4(ctx, L, "mxf4 GEMM");
}

size_t mpp41_mlp_w4a4_scratch_bytes(uint32_t T, uint32_t H, uint32_t I)
{
    return up256((size_t)T * H / 2) + up256((size_t)T * H / 32) + up256((size_t)T * I / 2) + up256((size_t)T * I / 32);
}

mpp41_status mpp41_mlp_w4a4(mpp41_ctx *ctx, uint32_t T, uint32_t H, uint32_t I, const void *x, const uint8_t *wg,
                            const uint8_t *sg, const uint8_t *wu, const uint8_t *su, const uint8_t *wd,
                            const uint8_t *sd, void *out, int out_f16, void *scratch)
{
    NEED(ctx);
    if (!T || !H || !I) return MPP41_OK;
    if (H % 512 || I % 512) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden and intermediate must be multiples of 512");
    if (!x || !wg || !sg || !wu || !su || !wd || !sd || !out || !scratch)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(x) || !al16(wg) || !al16(sg) || !al16(wu) || !al16(su) || !al16(wd) || !al16(sd) || !al16(out) ||
        (reinterpret_cast<uintptr_t>(scratch) & 255u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "buffers must be 16-byte aligned (scratch 256-byte)");
    uint8_t *xq = static_cast<uint8_t *>(scratch);
    uint8_t *xs = xq + up256((size_t)T * H / 2);
    uint8_t *mq = xs + up256((size_t)T * H / 32);
    uint8_t *ms = mq + up256((size_t)T * I / 2);
    CK(launch_quantize_mxfp4_f16(x, T, H, xq, xs, ctx->stream), "quantize activations");
    MxLaunch g{};
    g.a = xq; g.sa = xs;
    g.b0 = wg; g.sb0 = sg; g.b1 = wu; g.sb1 = su;
    g.b_rows = I;
    g.out = mq; g.out_scales = ms;
    g.M = T; g.N = I; g.K = H; g.ldc = I;
    g.epi = 2;
    g.err = ctx->err;
    mpp41_status s = enqueue_mxf4(ctx, g, "W4A4 gate/up GEMM");
    if (s != MPP41_OK) return s;
    MxLaunch d{};
    d.a = mq; d.sa = ms;
    d.b0 = d.b1 = wd; d.sb0 = d.sb1 = sd;
    d.b_rows = H;
    d.out = out; d.M = T; d.N = H; d.K = I; d.ldc = H;
    d.epi = out_f16 ? 1 : 0;
    d.err = ctx->err;
    return enqueue_mxf4(ctx, d, "W4A4 down GEMM");
}

// ------------------------------------------------------------------ NVFP4
mpp41_status mpp41_quantize_nvfp4(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, uint8_t *packed,
                                  uint8_t *scales, float *tensor_scale)
{
    NEED(ctx);
    if (depth % 16) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "depth must be a multiple of 16");
    if (!rows || !depth) return MPP41_OK;
    if (!w || !packed || !scales || !tensor_scale) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(w) || (reinterpret_cast<uintptr_t>(packed) & 7u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "w must be 16-byte and packed 8-byte aligned");
    CK(launch_quantize_nvfp4(w, false, rows, depth, ctx->amax, packed, scales, tensor_scale, ctx->stream),
       "quantize NVFP4");
    return MPP41_OK;
}

mpp41_status mpp41_quantize_act_nvfp4(mpp41_ctx *ctx, const void *x, uint32_t tokens, uint32_t hidden,
                                      uint8_t *packed, uint8_t *scales, float *tensor_scale)
{
    NEED(ctx);
    if (hidden % 16) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden must be a multiple of 16");
    if (!tokens || !hidden) return MPP41_OK;
    if (!x || !packed || !scales || !tensor_scale) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if ((reinterpret_cast<uintptr_t>(packed) & 7u)) return fail(MPP41_ERR_INVALID_ARGUMENT, "packed must be 8-byte aligned");
    CK(launch_quantize_nvfp4(x, true, tokens, hidden, ctx->amax, packed, scales, tensor_scale, ctx->stream),
       "quantize NVFP4 activations");
    return MPP41_OK;
}

mpp41_status mpp41_matmul_nvf4(mpp41_ctx *ctx, const uint8_t *a, const uint8_t *sa, const float *ta,
                               const uint8_t *b, const uint8_t *sb, const float *tb, void *c, uint32_t M, uint32_t N,
                               uint32_t K, int c_f16)
{
    NEED(ctx);
    if (!M || !N || !K) return MPP41_OK;
    if (!a || !sa || !ta || !b || !sb || !tb || !c) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(a) || !al16(sa) || !al16(b) || !al16(sb) || !al16(c))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "buffers must be 16-byte aligned");
    MxLaunch L{};
    L.a = a; L.sa = sa;
    L.b0 = L.b1 = b; L.sb0 = L.sb1 = sb;
    L.b_rows = N;
    L.out = c; L.M = M; L.N = N; L.K = K; L.ldc = N;
    L.epi = c_f16 ? 1 : 0;
    L.nv = true; L.ts_a = ta; L.ts_b0 = L.ts_b1 = tb;
    L.err = ctx->err;
    return enqueue_mxf4(ctx, L, "nvf4 GEMM");
}

namespace {
struct NvScratch {
    uint8_t *xq, *xs, *mq, *ms;
    __half *mid;
    float *ts;   // [0] x's tensor scale, [1] mid's
    size_t bytes;
};
NvScratch nv_scratch(void *base, uint32_t T, uint32_t H, uint32_t I)
{
    NvScratch s{};
    uint8_t *p = static_cast<uint8_t *>(base);
    size_t o = 0;
    auto take = [&](size_t n) { uint8_t *r = p ? p + o : nullptr; o += up256(n); return r; };
    s.xq = take((size_t)T * H / 2);
    s.xs = take((size_t)T * H / 16);
    s.mid = reinterpret_cast<__half *>(take((size_t)T * I * 2));
    s.mq = take((size_t)T * I / 2);
    s.ms = take((size_t)T * I / 16);
    s.ts = reinterpret_cast<float *>(take(2 * sizeof(float)));
    s.bytes = o;
    return s;
}
}  // namespace

size_t mpp41_mlp_nvfp4_scratch_bytes(uint32_t T, uint32_t H, uint32_t I) { return nv_scratch(nullptr, T, H, I).bytes; }

mpp41_status mpp41_mlp_nvfp4(mpp41_ctx *ctx, uint32_t T, uint32_t H, uint32_t I, const void *x, const uint8_t *wg,
                             const uint8_t *sg, const float *tg, const uint8_t *wu, const uint8_t *su,
                             const float *tu, const uint8_t *wd, const uint8_t *sd, const float *td, void *out,
                             int out_f16, void *scratch)
{
    NEED(ctx);
    if (!T || !H || !I) return MPP41_OK;
    if (H % 256 || I % 256) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden and intermediate must be multiples of 256");
    if (!x || !wg || !sg || !tg || !wu || !su || !tu || !wd || !sd || !td || !out || !scratch)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(x) || !al16(wg) || !al16(sg) || !al16(wu) || !al16(su) || !al16(wd) || !al16(sd) || !al16(out) ||
        (reinterpret_cast<uintptr_t>(scratch) & 255u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "buffers must be 16-byte aligned (scratch 256-byte)");
    const NvScratch s = nv_scratch(scratch, T, H, I);
    cudaStream_t st = ctx->stream;
    CK(launch_quantize_nvfp4(x, true, T, H, ctx->amax, s.xq, s.xs, s.ts, st), "quantize activations");
    CK(cudaMemsetAsync(ctx->amax, 0, sizeof(uint32_t), st), "clear the mid maximum");
    MxLaunch g{};
    g.a = s.xq; g.sa = s.xs;
    g.b0 = wg; g.sb0 = sg; g.b1 = wu; g.sb1 = su;
    g.b_rows = I;
    g.out = s.mid; g.M = T; g.N = I; g.K = H; g.ldc = I;
    g.epi = 3;
    g.nv = true; g.ts_a = s.ts; g.ts_b0 = tg; g.ts_b1 = tu;
    g.amax_out = ctx->amax;   // the gate/up epilogue reduces |mid| for the mid's tensor scale
    g.err = ctx->err;
    mpp41_status r = enqueue_mxf4(ctx, g, "NVFP4 gate/up GEMM");
    if (r != MPP41_OK) return r;
    CK(launch_quantize_nvfp4(s.mid, true, T, I, ctx->amax, s.mq, s.ms, s.ts + 1, st, true), "quantize mid");
    MxLaunch d{};
    d.a = s.mq; d.sa = s.ms;
    d.b0 = d.b1 = wd; d.sb0 = d.sb1 = sd;
    d.b_rows = H;
    d.out = out; d.M = T; d.N = H; d.K = I; d.ldc = H;
    d.epi = out_f16 ? 1 : 0;
    d.nv = true; d.ts_a = s.ts + 1; d.ts_b0 = d.ts_b1 = td;
    d.err = ctx->err;
    return enqueue_mxf4(ctx, d, "NVFP4 down GEMM");
}

// ------------------------------------------------------------------ scaled W8A8 / W4A8 / W2A8
mpp41_status mpp41_quantize_weights_int(mpp41_ctx *ctx, const float *w, uint32_t rows, uint32_t depth, int bits,
                                        void *packed, float *scales)
{
    NEED(ctx);
    if (bits != 8 && bits != 4 && bits != 2) return fail(MPP41_ERR_INVALID_ARGUMENT, "bits must be 8, 4 or 2");
    if (depth % 8) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "depth must be a multiple of 8");
    if (!rows || !depth) return MPP41_OK;
    if (!w || !packed || !scales) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_quantize_int_rows(w, rows, depth, bits, static_cast<uint8_t *>(packed), scales, ctx->stream),
       "quantize weights");
    return MPP41_OK;
}

size_t mpp41_mlp_w8a8_scratch_bytes(uint32_t T, uint32_t H, uint32_t I)
{
    return up256((size_t)T * H) + up256((size_t)T * 4) + up256((size_t)T * I * 2) + up256((size_t)T * I) +
           up256((size_t)T * 4);
}

mpp41_status mpp41_mlp_w8a8(mpp41_ctx *ctx, int wfmt, uint32_t T, uint32_t H, uint32_t I, const void *x,
                            const void *wg, const float *sg, const void *wu, const float *su, const void *wd,
                            const float *sd, void *out, void *scratch)
{
    NEED(ctx);
    if (wfmt != MPP41_W_I8 && wfmt != MPP41_W_I4 && wfmt != MPP41_W_I2)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "weights must be INT8, INT4 or INT2");
    if (!T || !H || !I) return MPP41_OK;
    if (H % 128 || I % 128) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden and intermediate must be multiples of 128");
    if (!x || !wg || !sg || !wu || !su || !wd || !sd || !out || !scratch)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!al16(x) || !al16(wg) || !al16(wu) || !al16(wd) || !al16(out) || (reinterpret_cast<uintptr_t>(scratch) & 255u))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "buffers must be 16-byte aligned (scratch 256-byte)");
    uint8_t *xq = static_cast<uint8_t *>(scratch);
    float *xs = reinterpret_cast<float *>(xq + up256((size_t)T * H));
    __half *mid = reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(xs) + up256((size_t)T * 4));
    uint8_t *mq = reinterpret_cast<uint8_t *>(mid) + up256((size_t)T * I * 2);
    float *ms = reinterpret_cast<float *>(mq + up256((size_t)T * I));
    cudaStream_t st = ctx->stream;
    CK(launch_quantize_act_s8(x, T, H, reinterpret_cast<int8_t *>(xq), xs, st), "quantize x");
    I8Launch g{};
    g.wfmt = wfmt; g.epi = 3;
    g.a = xq; g.b0 = wg; g.b1 = wu; g.out = mid;
    g.row_scale = xs; g.col_scale0 = sg; g.col_scale1 = su;
    g.M = T; g.N = I; g.K = H; g.ldc = I; g.splits = 1;
    g.err = ctx->err;
    const char *why = "";
    int rc = launch_i8_gemm(g, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "W8A8 gate/up GEMM: %s", why);
    CK(launch_quantize_act_s8(mid, T, I, reinterpret_cast<int8_t *>(mq), ms, st), "quantize mid");
    I8Launch d{};
    d.wfmt = wfmt; d.epi = 4;
    d.a = mq; d.b0 = wd; d.out = out;
    d.row_scale = ms; d.col_scale0 = sd;
    d.M = T; d.N = H; d.K = I; d.ldc = H; d.splits = 1;
    d.err = ctx->err;
    rc = launch_i8_gemm(d, st, &why);
    if (rc) return fail(rc == 1 ? MPP41_ERR_UNSUPPORTED_SHAPE : MPP41_ERR_CUDA, "W8A8 down GEMM: %s", why);
    return MPP41_OK;
}

// ------------------------------------------------------------------ MoE
static mpp41_status check_moe(const mpp41_moe_desc *d)
{
    if (!d) return fail(MPP41_ERR_INVALID_ARGUMENT, "null MoE descriptor");
    if (d->hidden % 512 || d->intermediate % 512 || d->shared_intermediate % 512)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "hidden and intermediate sizes must be multiples of 512");
    if (!d->experts || d->experts % 32 || d->experts > 512)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "experts must be a multiple of 32, at most 512");
    if (!d->top_k || d->top_k > 16 || d->top_k > d->experts)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "top_k must be in [1, min(16, experts)]");
    return MPP41_OK;
}

size_t mpp41_moe_scratch_layout(const mpp41_moe_desc *d, size_t *offsets)
{
    if (!d) return 0;
    const size_t T = d->tokens, H = d->hidden, I = d->intermediate, E = d->experts, R = T * d->top_k;
    const size_t Is = d->shared_intermediate;
    const size_t max_tiles = R / 128 + E + 1;
    const size_t sizes[MPP41_MOE_PARTS] = {
        T * H / 2, T * H / 32, R * 4, R * 4, E * 4, (E + 1) * 4, 4, max_tiles * 16, R * 4, R * 4,
        R * H / 2, R * H / 32, R * I / 2, R * I / 32, R * H * 4, T * Is / 2, T * Is / 32, Is ? T * H * 4 : 0};
    size_t o = 0;
    for (int i = 0; i < MPP41_MOE_PARTS; ++i) {
        if (offsets) offsets[i] = o;
        o += up256(sizes[i]);
    }
    return o;
}

mpp41_status mpp41_moe_route(mpp41_ctx *ctx, const float *logits, uint32_t T, uint32_t E, uint32_t k, int32_t *ids,
                             float *weights)
{
    NEED(ctx);
    if (!E || E % 32 || E > 512 || !k || k > 16 || k > E)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "experts must be a multiple of 32 up to 512, top_k in [1, 16]");
    if (!T) return MPP41_OK;
    if (!logits || !ids || !weights) return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    CK(launch_moe_route(logits, T, E, k, ids, weights, ctx->stream), "route");
    return MPP41_OK;
}

namespace {
// Scratch views of the single-GPU layout.
struct MoeBuf {
    uint8_t *b;
    size_t off[MPP41_MOE_PARTS];
    uint8_t *u8(int part) const { return b + off[part]; }
    uint32_t *u32(int part) const { return reinterpret_cast<uint32_t *>(b + off[part]); }
    float *f32(int part) const { return reinterpret_cast<float *>(b + off[part]); }
};

mpp41_status moe_check_ptrs(const mpp41_moe_desc *d, const void *x, const float *logits, const void *wg,
                            const void *sg, const void *wu, const void *su, const void *wd, const void *sd,
                            const void *const shared[6], const void *out, const void *scratch)
{
    if (!x || !logits || !wg || !sg || !wu || !su || !wd || !sd || !out || !scratch)
        return fail(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (d->shared_intermediate)
        for (int i = 0; i < 6; ++i)
            if (!shared[i]) return fail(MPP41_ERR_INVALID_ARGUMENT, "shared expert weights missing");
    if ((reinterpret_cast<uintptr_t>(scratch) & 255u) || !al16(x) || !al16(out))
        return fail(MPP41_ERR_INVALID_ARGUMENT, "x and out must be 16-byte aligned, scratch 256-byte");
    return MPP41_OK;
}

// Quantize x, route, group this rank's assignments by expert (all E experts)
// and gather the quantized rows into that order.
mpp41_status moe_front(mpp41_ctx *ctx, const mpp41_moe_desc *d, const void *x, const float *logits, const MoeBuf &m)
{
    const uint32_t T = d->tokens, H = d->hidden, E = d->experts, k = d->top_k, R = T * k;
    cudaStream_t st = ctx->stream;
    CK(launch_quantize_mxfp4_f16(x, T, H, m.u8(MPP41_MOE_XQ), m.u8(MPP41_MOE_XS), st), "quantize x");
    CK(launch_moe_route(logits, T, E, k, reinterpret_cast<int32_t *>(m.u8(MPP41_MOE_IDS)), m.f32(MPP41_MOE_WEIGHTS),
                        st), "route");
    CK(launch_moe_permute(reinterpret_cast<int32_t *>(m.u8(MPP41_MOE_IDS)), R, E, 128, m.u32(MPP41_MOE_COUNTS),
                          m.u32(MPP41_MOE_OFFSETS), reinterpret_cast<uint4 *>(m.u8(MPP41_MOE_TILES)),
                          m.u32(MPP41_MOE_NTILES), m.u32(MPP41_MOE_PERM), m.u32(MPP41_MOE_INV), ctx->err, st),
       "permute");
    const uint32_t *n_rows = m.u32(MPP41_MOE_OFFSETS) + E;
    CK(launch_moe_gather(m.u8(MPP41_MOE_XQ), H / 2, m.u32(MPP41_MOE_PERM), k, n_rows, R, m.u8(MPP41_MOE_PQ), st),
       "gather x");
    CK(launch_moe_gather(m.u8(MPP41_MOE_XS), H / 32, m.u32(MPP41_MOE_PERM), k, n_rows, R, m.u8(MPP41_MOE_PS), st),
       "gather x scales");
    return MPP41_OK;
}

// Grouped expert MLP over rows already grouped by expert: aq/as -> y [rows][H] fp32.
mpp41_status moe_experts(mpp41_ctx *ctx, uint32_t H, uint32_t I, uint32_t E, uint32_t rows, uint32_t max_tiles,
                         const uint4 *tiles, const uint32_t *n_tiles, const uint8_t *aq, const uint8_t *as,
                         const uint8_t *wg, const uint8_t *sg, const uint8_t *wu, const uint8_t *su,
                         const uint8_t *wd, const uint8_t *sd, uint8_t *mq, uint8_t *ms, float *y)
{
    if (!rows) return MPP41_OK;
    MxLaunch g{};
    g.a = aq; g.sa = as;
    g.b0 = wg; g.sb0 = sg; g.b1 = wu; g.sb1 = su;
    g.b_rows = E * I;
    g.out = mq; g.out_scales = ms;
    g.M = rows; g.N = I; g.K = H; g.ldc = I; g.epi = 2;
    g.tiles = tiles; g.n_tiles = n_tiles; g.max_tiles = max_tiles; g.b_expert_rows = I;
    g.err = ctx->err;
    mpp41_status s = enqueue_mxf4(ctx, g, "MoE gate/up GEMM");
    if (s != MPP41_OK) return s;
    MxLaunch dn{};
    dn.a = mq; dn.sa = ms;
    dn.b0 = dn.b1 = wd; dn.sb0 = dn.sb1 = sd;
    dn.b_rows = E * H;
    dn.out = y; dn.M = rows; dn.N = H; dn.K = I; dn.ldc = H; dn.epi = 0;
    dn.tiles = tiles; dn.n_tiles = n_tiles; dn.max_tiles = max_tiles; dn.b_expert_rows = H;
    dn.err = ctx->err;
    return enqueue_mxf4(ctx, dn, "MoE down GEMM");
}

// Shared expert on this rank's quantized x, then the weighted combine.
mpp41_status moe_back(mpp41_ctx *ctx, const mpp41_moe_desc *d, const void *const shared[6], const MoeBuf &m,
                      void *out)
{
    const uint32_t T = d->tokens, H = d->hidden, Is = d->shared_intermediate;
    const float *shared_y = nullptr;
    if (Is) {
        MxLaunch g{};
        g.a = m.u8(MPP41_MOE_XQ); g.sa = m.u8(MPP41_MOE_XS);
        g.b0 = shared[0]; g.sb0 = shared[1]; g.b1 = shared[2]; g.sb1 = shared[3];
        g.b_rows = Is;
        g.out = m.u8(MPP41_MOE_SMQ); g.out_scales = m.u8(MPP41_MOE_SMS);
        g.M = T; g.N = Is; g.K = H; g.ldc = Is; g.epi = 2;
        g.err = ctx->err;
        mpp41_status s = enqueue_mxf4(ctx, g, "shared expert gate/up GEMM");
        if (s != MPP41_OK) return s;
        MxLaunch dn{};
        dn.a = m.u8(MPP41_MOE_SMQ); dn.sa = m.u8(MPP41_MOE_SMS);
        dn.b0 = dn.b1 = shared[4]; dn.sb0 = dn.sb1 = shared[5];
        dn.b_rows = H;
        dn.out = m.u8(MPP41_MOE_SY); dn.M = T; dn.N = H; dn.K = Is; dn.ldc = H; dn.epi = 0;
        dn.err = ctx->err;
        s = enqueue_mxf4(ctx, dn, "shared expert down GEMM");
        if (s != MPP41_OK) return s;
        shared_y = m.f32(MPP41_MOE_SY);
    }
    CK(launch_moe_combine(m.f32(MPP41_MOE_Y), m.u32(MPP41_MOE_INV), m.f32(MPP41_MOE_WEIGHTS), T, d->top_k, H,
                          shared_y, out, d->out_f16 != 0, ctx->stream), "combine");
    return MPP41_OK;
}
}  // namespace

mpp41_status mpp41_moe_w4a4(mpp41_ctx *ctx, const mpp41_moe_desc *d, const void *x, const float *logits,
                            const uint8_t *wg, const uint8_t *sg, const uint8_t *wu, const uint8_t *su,
                            const uint8_t *wd, const uint8_t *sd, const uint8_t *shared_wg, const uint8_t *shared_sg,
                            const uint8_t *shared_wu, const uint8_t *shared_su, const uint8_t *shared_wd,
                            const uint8_t *shared_sd, void *out, void *scratch)
{
    NEED(ctx);
    mpp41_status s = check_moe(d);
    if (s != MPP41_OK) return s;
    if (!d->tokens) return MPP41_OK;
    const void *const shared[6] = {shared_wg, shared_sg, shared_wu, shared_su, shared_wd, shared_sd};
    s = moe_check_ptrs(d, x, logits, wg, sg, wu, su, wd, sd, shared, out, scratch);
    if (s != MPP41_OK) return s;
    MoeBuf m;
    m.b = static_cast<uint8_t *>(scratch);
    mpp41_moe_scratch_layout(d, m.off);
    s = moe_front(ctx, d, x, logits, m);
    if (s != MPP41_OK) return s;
    const uint32_t R = d->tokens * d->top_k;
    s = moe_experts(ctx, d->hidden, d->intermediate, d->experts, R, R / 128 + d->experts + 1,
                    reinterpret_cast<const uint4 *>(m.u8(MPP41_MOE_TILES)), m.u32(MPP41_MOE_NTILES),
                    m.u8(MPP41_MOE_PQ), m.u8(MPP41_MOE_PS), wg, sg, wu, su, wd, sd, m.u8(MPP41_MOE_MQ),
                    m.u8(MPP41_MOE_MS), m.f32(MPP41_MOE_Y));
    if (s != MPP41_OK) return s;
    return moe_back(ctx, d, shared, m, out);
}

// ------------------------------------------------------------------ expert parallel
size_t mpp41_moe_ep_scratch_layout(const mpp41_moe_desc *d, int nranks, uint32_t capacity, size_t *offsets)
{
    if (!d || nranks < 1 || d->experts % (uint32_t)nranks) return 0;
    const size_t P = (size_t)nranks, E = d->experts, El = E / P, H = d->hidden, I = d->intermediate, C = capacity;
    size_t o = mpp41_moe_scratch_layout(d, nullptr);
    const size_t sizes[MPP41_MOE_EP_PARTS] = {P * E * 4, P * El * 16, (C / 128 + El + 1) * 16, 4,
                                              C * H / 2, C * H / 32, C * H / 2, C * H / 32, C * I / 2, C * I / 32,
                                              C * H * 4, C * H * 4};
    for (int i = 0; i < MPP41_MOE_EP_PARTS; ++i) {
        if (offsets) offsets[i] = o;
        o += up256(sizes[i]);
    }
    return o;
}

mpp41_status mpp41_moe_ep(mpp41_ctx *ctx, const mpp41_moe_desc *d, uint32_t capacity, const void *x,
                          const float *logits, const uint8_t *wg, const uint8_t *sg, const uint8_t *wu,
                          const uint8_t *su, const uint8_t *wd, const uint8_t *sd, const uint8_t *shared_wg,
                          const uint8_t *shared_sg, const uint8_t *shared_wu, const uint8_t *shared_su,
                          const uint8_t *shared_wd, const uint8_t *shared_sd, void *out, void *scratch)
{
    NEED(ctx);
    mpp41_status s = check_moe(d);
    if (s != MPP41_OK) return s;
    const int P = comm_size(ctx), rank = comm_rank(ctx);
    if (P < 1) return fail(MPP41_ERR_COMM, "mpp41_comm_init has not been called on this context");
    if (d->experts % (uint32_t)P) return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "experts must divide over the ranks");
    const uint32_t H = d->hidden, I = d->intermediate, E = d->experts, El = E / (uint32_t)P;
    const void *const shared[6] = {shared_wg, shared_sg, shared_wu, shared_su, shared_wd, shared_sd};
    if (d->tokens) {
        s = moe_check_ptrs(d, x, logits, wg, sg, wu, su, wd, sd, shared, out, scratch);
        if (s != MPP41_OK) return s;
    } else if (!scratch) {
        return fail(MPP41_ERR_INVALID_ARGUMENT, "null scratch");
    }
    MoeBuf m;
    m.b = static_cast<uint8_t *>(scratch);
    mpp41_moe_scratch_layout(d, m.off);
    size_t eo[MPP41_MOE_EP_PARTS];
    mpp41_moe_ep_scratch_layout(d, P, capacity, eo);
    auto ep = [&](int part) { return m.b + eo[part]; };
    cudaStream_t st = ctx->stream;
    if (d->tokens) {
        s = moe_front(ctx, d, x, logits, m);
        if (s != MPP41_OK) return s;
    } else {
        CK(cudaMemsetAsync(m.u32(MPP41_MOE_COUNTS), 0, E * 4, st), "clear counts");
    }
    // every rank's per-expert counts; the host sizes the exchanges from them
    s = comm_allgather(ctx, m.u32(MPP41_MOE_COUNTS), ep(MPP41_MOE_EP_ALLC), E * 4);
    if (s != MPP41_OK) return s;
    std::vector<uint32_t> allc((size_t)P * E);
    CK(cudaMemcpyAsync(allc.data(), ep(MPP41_MOE_EP_ALLC), allc.size() * 4, cudaMemcpyDeviceToHost, st),
       "read expert counts");
    CK(cudaStreamSynchronize(st), "read expert counts");
    std::vector<size_t> send_rows(P, 0), recv_rows(P, 0), send_off(P, 0), recv_off(P, 0);
    for (int p = 0; p < P; ++p)
        for (uint32_t le = 0; le < El; ++le) {
            send_rows[p] += allc[(size_t)rank * E + (size_t)p * El + le];
            recv_rows[p] += allc[(size_t)p * E + (size_t)rank * El + le];
        }
    size_t total_recv = 0, total_send = 0;
    for (int p = 0; p < P; ++p) {
        send_off[p] = total_send;
        recv_off[p] = total_recv;
        total_send += send_rows[p];
        total_recv += recv_rows[p];
    }
    if (total_recv > capacity)
        return fail(MPP41_ERR_UNSUPPORTED_SHAPE, "rank %d receives %zu rows, capacity is %u", rank, total_recv,
                    capacity);
    auto scaled = [&](const std::vector<size_t> &v, size_t unit) {
        std::vector<size_t> r(v.size());
        for (size_t i = 0; i < v.size(); ++i) r[i] = v[i] * unit;
        return r;
    };
    // dispatch: quantized rows and their scales, grouped by destination rank
    s = comm_alltoallv(ctx, m.u8(MPP41_MOE_PQ), scaled(send_rows, H / 2).data(), scaled(send_off, H / 2).data(),
                       ep(MPP41_MOE_EP_RQ), scaled(recv_rows, H / 2).data(), scaled(recv_off, H / 2).data());
    if (s != MPP41_OK) return s;
    s = comm_alltoallv(ctx, m.u8(MPP41_MOE_PS), scaled(send_rows, H / 32).data(), scaled(send_off, H / 32).data(),
                       ep(MPP41_MOE_EP_RS), scaled(recv_rows, H / 32).data(), scaled(recv_off, H / 32).data());
    if (s != MPP41_OK) return s;
    // received rows are source-major; the experts want them expert-major
    const uint32_t max_tiles = capacity / 128 + El + 1;
    uint4 *segs = reinterpret_cast<uint4 *>(ep(MPP41_MOE_EP_SEGS));
    CK(launch_moe_ep_plan(reinterpret_cast<const uint32_t *>(ep(MPP41_MOE_EP_ALLC)), P, E, rank, 128, segs,
                          reinterpret_cast<uint4 *>(ep(MPP41_MOE_EP_TILES)),
                          reinterpret_cast<uint32_t *>(ep(MPP41_MOE_EP_NTILES)), st), "plan");
    CK(launch_moe_segments(ep(MPP41_MOE_EP_RQ), ep(MPP41_MOE_EP_GQ), H / 2, segs, P * El, false, st), "group rows");
    CK(launch_moe_segments(ep(MPP41_MOE_EP_RS), ep(MPP41_MOE_EP_GS), H / 32, segs, P * El, false, st), "group scales");
    s = moe_experts(ctx, H, I, El, (uint32_t)total_recv, max_tiles, reinterpret_cast<const uint4 *>(ep(MPP41_MOE_EP_TILES)),
                    reinterpret_cast<const uint32_t *>(ep(MPP41_MOE_EP_NTILES)), ep(MPP41_MOE_EP_GQ),
                    ep(MPP41_MOE_EP_GS), wg, sg, wu, su, wd, sd, ep(MPP41_MOE_EP_GMQ), ep(MPP41_MOE_EP_GMS),
                    reinterpret_cast<float *>(ep(MPP41_MOE_EP_GY)));
    if (s != MPP41_OK) return s;
    CK(launch_moe_segments(ep(MPP41_MOE_EP_GY), ep(MPP41_MOE_EP_RY), H * 4, segs, P * El, true, st), "ungroup rows");
    // combine exchange: fp32 rows go back to the ranks that own the tokens, in
    // the order those ranks sent them (their expert-major local order)
    s = comm_alltoallv(ctx, ep(MPP41_MOE_EP_RY), scaled(recv_rows, H * 4).data(), scaled(recv_off, H * 4).data(),
                       m.u8(MPP41_MOE_Y), scaled(send_rows, H * 4).data(), scaled(send_off, H * 4).data());
    if (s != MPP41_OK) return s;
    if (!d->tokens) return MPP41_OK;
    return moe_back(ctx, d, shared, m, out);
}

mpp41_status mpp41_mlp_benchmark(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg,
                                 const void *wu, const void *wd, const uint8_t *sg, const uint8_t *su,
                                 const uint8_t *sd, void *scratch, void *out, int iterations, double *gpu_seconds)
{
    NEED(ctx);
    mpp41_status s = check_mlp_desc(d);
    if (s) return s;
    if (iterations <= 0 || !gpu_seconds) return fail(MPP41_ERR_INVALID_ARGUMENT, "iterations must be positive");
    // capture needs a real stream: order after the caller's stream, then run
    // on the context's private stream
    CK(cudaStreamSynchronize(ctx->stream), "caller stream");
    cudaStream_t st = ctx->own_stream;
    // untimed warm-up run (main.swift:2015-2020), which also validates the row
    s = enqueue_mlp(ctx, d, x, wg, wu, wd, sg, su, sd, scratch, out, st);
    if (s) return s;
    CK(cudaStreamSynchronize(st), "warm-up");
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture");
    for (int i = 0; i < iterations && s == MPP41_OK; ++i) s = enqueue_mlp(ctx, d, x, wg, wu, wd, sg, su, sd, scratch, out, st);
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (s) { if (graph) cudaGraphDestroy(graph); return s; }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    e = cudaGraphLaunch(exec, st);   // warm the graph once
    if (e == cudaSuccess) e = cudaEventRecord(ctx->ev0, st);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) e = cudaEventRecord(ctx->ev1, st);
    if (e == cudaSuccess) e = cudaEventSynchronize(ctx->ev1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
    cudaGraphExecDestroy(exec);
    if (e != cudaSuccess) return cuda_fail(e, "timed replay");
    *gpu_seconds = ms * 1e-3;
    CK(cudaStreamSynchronize(st), "benchmark stream");
    return mpp41_synchronize(ctx);
}

}  // extern "C"

// Lets other translation units of the library report through mpp41_last_error().
namespace mpp41 {
mpp41_status set_last_error(mpp41_status s, const char *msg) { return fail(s, "%s", msg); }

int gemm_kernel_wfmt(const char *name)
{
    const KernelInfo *k = find_kernel(name);
    return k && k->kind == K_GEMM && k->afmt == 0 ? k->arg0 : -1;
}
}  // namespace mpp41
