/*
 * CPU oracle for the quantized-weight MLP hot path: TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic. Each function names
 * the reference file:line it follows (paths are relative to the reference
 * project root). Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline arm load this library; the product never does.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off). FP contraction
 * is disabled so that every float expression rounds exactly as written.
 */
#include "mpp41_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* Seeded generators: main.swift:2785-2842.                             */
/* state = state * 1664525 + 1013904223 + index  (wrapping uint32)      */
/* ------------------------------------------------------------------ */

static inline uint32_t lcg_step(uint32_t s, size_t index)
{
    return s * 1664525u + 1013904223u + (uint32_t)index;
}

/* makePackedMatrixBytes, main.swift:2785-2793 */
void orc_make_packed_bytes(uint8_t *out, size_t n, uint32_t seed)
{
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = lcg_step(s, i);
        out[i] = (uint8_t)(s >> 16);
    }
}

/* makeBytePatternValues, main.swift:2813-2821 */
void orc_make_pattern_bytes(uint8_t *out, size_t n, uint32_t seed,
                            const uint8_t *pattern, size_t pattern_len)
{
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = lcg_step(s, i);
        out[i] = pattern[s % (uint32_t)pattern_len];
    }
}

/* makeFiniteFP8E4M3Bytes, main.swift:2795-2801 */
void orc_make_fp8_e4m3_bytes(uint8_t *out, size_t n, uint32_t seed)
{
    static const uint8_t pat[10] = {0x00, 0x20, 0x30, 0x38, 0x40, 0xb0, 0xb8, 0xc0, 0x58, 0xd8};
    orc_make_pattern_bytes(out, n, seed, pat, 10);
}

/* makeFiniteFP8E5M2Bytes, main.swift:2803-2809 */
void orc_make_fp8_e5m2_bytes(uint8_t *out, size_t n, uint32_t seed)
{
    static const uint8_t pat[10] = {0x00, 0x34, 0x38, 0x3c, 0x40, 0xb4, 0xb8, 0xbc, 0xc0, 0x64};
    orc_make_pattern_bytes(out, n, seed, pat, 10);
}

/* makeHalfMatrixValues, main.swift:2823-2833: ((s>>28)^8)-8 times scale */
void orc_make_half_values(uint16_t *out, size_t n, uint32_t seed, float scale)
{
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = lcg_step(s, i);
        int nib = (int)((s >> 28) & 0x0f);
        int v = (nib ^ 8) - 8;
        out[i] = orc_float_to_half((float)v * scale);
    }
}

/* makeInt8MatrixValues, main.swift:2835-2842 */
void orc_make_int8_values(int8_t *out, size_t n, uint32_t seed)
{
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = lcg_step(s, i);
        int nib = (int)((s >> 28) & 0x0f);
        out[i] = (int8_t)((nib ^ 8) - 8);
    }
}

/* ------------------------------------------------------------------ */
/* Codecs                                                              */
/* ------------------------------------------------------------------ */

float orc_half_to_float(uint16_t h)
{
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t orc_float_to_half(float f)
{
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline uint16_t dbl_to_half(double d)
{
    _Float16 v = (_Float16)d;  /* single rounding, round to nearest even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

/* kFP4E2M1Table, MXFP4Kernels.metal:33-36 (docs/MXFP4-MPP41-GUIDE.md:57-62) */
static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

float orc_e2m1_decode(uint8_t nibble) { return kE2M1[nibble & 0x0f]; }

float orc_e4m3_decode(uint8_t c)
{
    int s = c >> 7, e = (c >> 3) & 0x0f, m = c & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m / 8.0f, -6);
    else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -v : v;
}

float orc_e5m2_decode(uint8_t c)
{
    int s = c >> 7, e = (c >> 2) & 0x1f, m = c & 3;
    float v;
    if (e == 31) v = (m == 0) ? INFINITY : NAN;
    else if (e == 0) v = ldexpf((float)m / 4.0f, -14);
    else v = ldexpf(1.0f + (float)m / 4.0f, e - 15);
    return s ? -v : v;
}

/* e8m0_to_float, MXFP4Kernels.metal:26-29: as_type<float>(bits << 23).
 * Byte 0 decodes to +0.0 and byte 255 to +inf (not the OCP NaN). */
float orc_e8m0_decode(uint8_t code)
{
    uint32_t bits = (uint32_t)code << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* signed_int4_to_half, PackedNumericKernels.metal:30-33 */
int orc_int4_decode(uint8_t nibble) { return ((int)(nibble & 0x0f) ^ 8) - 8; }
/* signed_int2_to_half, PackedNumericKernels.metal:25-28 */
int orc_int2_decode(uint8_t bits) { return ((int)(bits & 0x03) ^ 2) - 2; }

/* Round-to-nearest-even onto a table of the positive finite values of a
 * minifloat (index == positive code), saturating at the largest finite
 * value. Used by the three encoders below; the reference pins saturation
 * (main.swift:112-130: E2M1 +-8 -> +-6, E4M3 +-512 -> +-448) and exact
 * values; ties follow OCP round-to-nearest-even. */
static uint8_t rne_table(double a, const double *vals, int count)
{
    if (a >= vals[count - 1]) return (uint8_t)(count - 1);
    int lo = 0, hi = count - 1;           /* vals[lo] <= a < vals[hi] */
    while (hi - lo > 1) {
        int mid = (lo + hi) / 2;
        if (vals[mid] <= a) lo = mid; else hi = mid;
    }
    double d0 = a - vals[lo], d1 = vals[hi] - a;
    if (d0 < d1) return (uint8_t)lo;
    if (d1 < d0) return (uint8_t)hi;
    return (uint8_t)((lo & 1) ? hi : lo);
}

static double g_e4m3_vals[127];   /* codes 0x00..0x7e */
static double g_e5m2_vals[124];   /* codes 0x00..0x7b */
static const double g_e2m1_vals[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};
static int g_tables_ready = 0;

static void init_tables(void)
{
    if (g_tables_ready) return;
    for (int c = 0; c < 127; ++c) g_e4m3_vals[c] = orc_e4m3_decode((uint8_t)c);
    for (int c = 0; c < 124; ++c) g_e5m2_vals[c] = orc_e5m2_decode((uint8_t)c);
    g_tables_ready = 1;
}

/* pack<metal_fp4_e2m1_format>, PackedNumericKernels.metal:35-54 */
uint8_t orc_e2m1_encode(float x)
{
    uint8_t sign = signbit(x) ? 0x8 : 0x0;
    double a = fabs((double)x);
    if (isnan(x)) return 0x7 | sign;
    return rne_table(a, g_e2m1_vals, 8) | sign;
}

/* pack<metal_fp8_e4m3_format>, PackedNumericKernels.metal:56-75 */
uint8_t orc_e4m3_encode(float x)
{
    init_tables();
    if (isnan(x)) return 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    return rne_table(fabs((double)x), g_e4m3_vals, 127) | sign;
}

/* pack<metal_fp8_e5m2_format>, PackedNumericKernels.metal:77-96 */
uint8_t orc_e5m2_encode(float x)
{
    init_tables();
    if (isnan(x)) return 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    return rne_table(fabs((double)x), g_e5m2_vals, 124) | sign;
}

void orc_pack(int fmt, const float *in, size_t n, uint8_t *packed)
{
    init_tables();
    if (fmt == 0) {
        for (size_t i = 0; i < n; i += 2) {
            uint8_t lo = orc_e2m1_encode(in[i]);
            uint8_t hi = (i + 1 < n) ? orc_e2m1_encode(in[i + 1]) : 0;
            packed[i / 2] = (uint8_t)(lo | (hi << 4));   /* low nibble = even index */
        }
    } else if (fmt == 1) {
        for (size_t i = 0; i < n; ++i) packed[i] = orc_e4m3_encode(in[i]);
    } else {
        for (size_t i = 0; i < n; ++i) packed[i] = orc_e5m2_encode(in[i]);
    }
}

void orc_unpack(int fmt, const uint8_t *packed, size_t n, float *out)
{
    if (fmt == 0) {
        for (size_t i = 0; i < n; ++i)
            out[i] = orc_e2m1_decode((uint8_t)(packed[i / 2] >> ((i & 1) * 4)));
    } else if (fmt == 1) {
        for (size_t i = 0; i < n; ++i) out[i] = orc_e4m3_decode(packed[i]);
    } else {
        for (size_t i = 0; i < n; ++i) out[i] = orc_e5m2_decode(packed[i]);
    }
}

/* ------------------------------------------------------------------ */
/* Weight decode. Layout [rows][depth], depth = K contiguous:          */
/* MPPMLPKernels.metal:14-37 (B extents {n,k}, strides {k,1});         */
/* MXFP4 scales[j*(k/32)+kb], MXFP4Kernels.metal:3-4.                  */
/* ------------------------------------------------------------------ */
void orc_decode_weights(int wfmt, const void *w, const uint8_t *scales,
                        uint32_t rows, uint32_t depth, double *out)
{
    const uint8_t *b = (const uint8_t *)w;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        double *o = out + (size_t)r * depth;
        for (uint32_t k = 0; k < depth; ++k) {
            double v = 0.0;
            switch (wfmt) {
            case ORC_W_F16: v = orc_half_to_float(((const uint16_t *)w)[(size_t)r * depth + k]); break;
            case ORC_W_I8: v = ((const int8_t *)w)[(size_t)r * depth + k]; break;
            case ORC_W_I4: {
                uint8_t byte = b[(size_t)r * (depth / 2) + k / 2];
                v = orc_int4_decode((uint8_t)(byte >> ((k & 1) * 4)));
                break;
            }
            case ORC_W_I2: {
                uint8_t byte = b[(size_t)r * (depth / 4) + k / 4];
                v = orc_int2_decode((uint8_t)(byte >> ((k & 3) * 2)));
                break;
            }
            case ORC_W_FP4: {
                uint8_t byte = b[(size_t)r * (depth / 2) + k / 2];
                v = orc_e2m1_decode((uint8_t)(byte >> ((k & 1) * 4)));
                break;
            }
            case ORC_W_E4M3: v = orc_e4m3_decode(b[(size_t)r * depth + k]); break;
            case ORC_W_E5M2: v = orc_e5m2_decode(b[(size_t)r * depth + k]); break;
            case ORC_W_MXFP4: {
                uint8_t byte = b[(size_t)r * (depth / 2) + k / 2];
                double e = orc_e2m1_decode((uint8_t)(byte >> ((k & 1) * 4)));
                double s = orc_e8m0_decode(scales[(size_t)r * (depth / 32) + k / 32]);
                v = e * s;
                break;
            }
            case ORC_W_E4M3_MX:
            case ORC_W_E5M2_MX: {
                const uint8_t c = b[(size_t)r * depth + k];
                const float e = wfmt == ORC_W_E4M3_MX ? orc_e4m3_decode(c) : orc_e5m2_decode(c);
                const float s = orc_e8m0_decode(scales[(size_t)r * (depth / 32) + k / 32]);
                v = orc_half_to_float(orc_float_to_half(e * s));   /* e * 2^n is exact in fp32 */
                break;
            }
            default: v = 0.0;
            }
            o[k] = v;
        }
    }
}

/* mxfp4_dequant_lut_half / mxfp4_dequant_native_half, MXFP4Kernels.metal:509-564:
 * out = half(float(table[nibble]) * e8m0_to_float(scale)). */
void orc_mxfp4_dequant_half(const uint8_t *packed, const uint8_t *scales,
                            uint16_t *out, uint32_t rows, uint32_t depth)
{
    uint32_t kblocks = depth / 32, bpr = depth / 2;
    for (uint32_t r = 0; r < rows; ++r) {
        for (uint32_t k = 0; k < depth; ++k) {
            uint8_t byte = packed[(size_t)r * bpr + k / 2];
            float s = orc_e8m0_decode(scales[(size_t)r * kblocks + k / 32]);
            float v = kE2M1[(byte >> ((k & 1) * 4)) & 0xf] * s;
            out[(size_t)r * depth + k] = orc_float_to_half(v);
        }
    }
}

void orc_gemm_f64(const double *a, const double *b, double *c,
                  uint32_t m, uint32_t n, uint32_t k)
{
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i = 0; i < (int64_t)m; ++i) {
        for (int64_t j = 0; j < (int64_t)n; ++j) {
            const double *ar = a + (size_t)i * k, *br = b + (size_t)j * k;
            double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
            uint32_t t = 0;
            for (; t + 4 <= k; t += 4) {
                s0 += ar[t] * br[t];
                s1 += ar[t + 1] * br[t + 1];
                s2 += ar[t + 2] * br[t + 2];
                s3 += ar[t + 3] * br[t + 3];
            }
            for (; t < k; ++t) s0 += ar[t] * br[t];
            c[(size_t)i * n + j] = (s0 + s1) + (s2 + s3);
        }
    }
}

/* ------------------------------------------------------------------ */
/* SwiGLU epilogues, MPPMLPKernels.metal:186-257. exp() is evaluated   */
/* in double and rounded to float, identically on the GPU side, so the */
/* integer epilogue is reproducible bit for bit.                        */
/* ------------------------------------------------------------------ */
static inline float exp_ref(float x) { return (float)exp((double)x); }

/* mpp_mlp_swiglu_float, MPPMLPKernels.metal:186-202 */
float orc_swiglu_float(float g, float u)
{
    return (g / (1.0f + exp_ref(-g))) * u;
}

static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* mpp_mlp_swiglu_half, MPPMLPKernels.metal:204-220 */
uint16_t orc_swiglu_half(float g, float u)
{
    float gs = clampf(g * 0.0625f, -20.0f, 20.0f);
    float us = u * 0.0625f;
    return orc_float_to_half((gs / (1.0f + exp_ref(-gs))) * us);
}

/* mpp_mlp_swiglu_half_from_half, MPPMLPKernels.metal:222-238 */
uint16_t orc_swiglu_half_from_half(uint16_t g, uint16_t u)
{
    return orc_swiglu_half(orc_half_to_float(g), orc_half_to_float(u));
}

/* mpp_mlp_swiglu_i8, MPPMLPKernels.metal:240-257 */
int8_t orc_swiglu_i8(int32_t g, int32_t u)
{
    float gs = clampf((float)g * 0.000244140625f, -20.0f, 20.0f);
    float us = (float)u * 0.000244140625f;
    float value = (gs / (1.0f + exp_ref(-gs))) * us * 32.0f;
    return (int8_t)(int)rintf(clampf(value, -128.0f, 127.0f));
}

/* ------------------------------------------------------------------ */
/* Whole MLP row: gate GEMM, up GEMM, swiglu, down GEMM                 */
/* (encodeMPPMLP main.swift:2636-2722, encodeMXFP4FusedMLP 2033-2135).  */
/* ------------------------------------------------------------------ */
static void mlp_impl(int act, int wfmt, int epi, int out_kind,
                     uint32_t T, uint32_t H, uint32_t I,
                     const void *x, const void *wg, const void *wu, const void *wd,
                     const uint8_t *sg, const uint8_t *su, const uint8_t *sd,
                     const uint16_t *rsg, const uint16_t *rsu, const uint16_t *rsd,
                     void *mid_out, void *out);

void orc_mlp(int act, int wfmt, int epi, int out_kind,
             uint32_t T, uint32_t H, uint32_t I,
             const void *x, const void *wg, const void *wu, const void *wd,
             const uint8_t *sg, const uint8_t *su, const uint8_t *sd,
             void *mid_out, void *out)
{
    mlp_impl(act, wfmt, epi, out_kind, T, H, I, x, wg, wu, wd, sg, su, sd, NULL, NULL, NULL, mid_out, out);
}

void orc_mlp_row_scaled(int wfmt, int epi, int out_kind,
                        uint32_t T, uint32_t H, uint32_t I,
                        const void *x, const void *wg, const void *wu, const void *wd,
                        const uint16_t *sg, const uint16_t *su, const uint16_t *sd,
                        void *mid_out, void *out)
{
    mlp_impl(0, wfmt, epi, out_kind, T, H, I, x, wg, wu, wd, NULL, NULL, NULL, sg, su, sd, mid_out, out);
}

/* Per-output-channel scale (fp16) of column c applied to an exact sum. */
static void scale_columns(double *m, uint32_t rows, uint32_t cols, const uint16_t *scale)
{
    if (!scale) return;
    for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t c = 0; c < cols; ++c) m[(size_t)r * cols + c] *= orc_half_to_float(scale[c]);
}

static void mlp_impl(int act, int wfmt, int epi, int out_kind,
                     uint32_t T, uint32_t H, uint32_t I,
                     const void *x, const void *wg, const void *wu, const void *wd,
                     const uint8_t *sg, const uint8_t *su, const uint8_t *sd,
                     const uint16_t *rsg, const uint16_t *rsu, const uint16_t *rsd,
                     void *mid_out, void *out)
{
    double *xd = malloc(sizeof(double) * (size_t)T * H);
    double *w = malloc(sizeof(double) * (size_t)I * H);
    double *gate = malloc(sizeof(double) * (size_t)T * I);
    double *up = malloc(sizeof(double) * (size_t)T * I);
    double *mid = malloc(sizeof(double) * (size_t)T * I);
    double *o = malloc(sizeof(double) * (size_t)T * H);

    for (size_t i = 0; i < (size_t)T * H; ++i)
        xd[i] = act == 0 ? orc_half_to_float(((const uint16_t *)x)[i]) : ((const int8_t *)x)[i];

    orc_decode_weights(wfmt, wg, sg, I, H, w);
    orc_gemm_f64(xd, w, gate, T, I, H);
    orc_decode_weights(wfmt, wu, su, I, H, w);
    orc_gemm_f64(xd, w, up, T, I, H);
    scale_columns(gate, T, I, rsg);
    scale_columns(up, T, I, rsu);

    for (size_t i = 0; i < (size_t)T * I; ++i) {
        switch (epi) {
        case 0: {
            float v = orc_swiglu_float((float)gate[i], (float)up[i]);
            if (mid_out) ((float *)mid_out)[i] = v;
            mid[i] = v;
            break;
        }
        case 1: {
            uint16_t h = orc_swiglu_half((float)gate[i], (float)up[i]);
            if (mid_out) ((uint16_t *)mid_out)[i] = h;
            mid[i] = orc_half_to_float(h);
            break;
        }
        case 2: {
            uint16_t h = orc_swiglu_half_from_half(dbl_to_half(gate[i]), dbl_to_half(up[i]));
            if (mid_out) ((uint16_t *)mid_out)[i] = h;
            mid[i] = orc_half_to_float(h);
            break;
        }
        case 4: {
            /* BASELINE config 0: silu(g)*u in fp32 (no prescale), fp16 mid */
            uint16_t h = orc_float_to_half(orc_swiglu_float((float)gate[i], (float)up[i]));
            if (mid_out) ((uint16_t *)mid_out)[i] = h;
            mid[i] = orc_half_to_float(h);
            break;
        }
        default: {
            int8_t q = orc_swiglu_i8((int32_t)gate[i], (int32_t)up[i]);
            if (mid_out) ((int8_t *)mid_out)[i] = q;
            mid[i] = q;
            break;
        }
        }
    }

    orc_decode_weights(wfmt, wd, sd, H, I, w);
    orc_gemm_f64(mid, w, o, T, H, I);
    scale_columns(o, T, H, rsd);
    for (size_t i = 0; i < (size_t)T * H; ++i) {
        if (out_kind == 0) ((float *)out)[i] = (float)o[i];
        else if (out_kind == 1) ((uint16_t *)out)[i] = dbl_to_half(o[i]);
        else ((int32_t *)out)[i] = (int32_t)o[i];
    }
    free(xd); free(w); free(gate); free(up); free(mid); free(o);
}

/* ------------------------------------------------------------------ */
/* Scalar half-accumulate kernels, PackedNumericKernels.metal:98-832.  */
/* Metal fma(half, half, half) rounds once; restated exactly below.     */
/* ------------------------------------------------------------------ */

static double half_dbl(uint16_t h) { return orc_half_to_float(h); }

/* next representable half above (dir>0) or below (dir<0) a finite half. */
static double half_neighbor(double v, int dir)
{
    uint16_t h = dbl_to_half(v), n;
    if (v == 0.0) n = dir > 0 ? 0x0001 : 0x8001;
    else if ((v > 0) == (dir > 0)) n = (uint16_t)(h + 1);
    else n = (uint16_t)(h - 1);
    return half_dbl(n);
}

uint16_t orc_half_fma(uint16_t a, uint16_t b, uint16_t c)
{
    double p = half_dbl(a) * half_dbl(b);       /* exact: 22 significant bits */
    double cc = half_dbl(c);
    double s = p + cc;
    double bb = s - p;
    double err = (p - (s - bb)) + (cc - bb);     /* TwoSum: s + err == p + cc exactly */
    uint16_t r = dbl_to_half(s);
    if (err != 0.0 && isfinite(s)) {
        double rd = half_dbl(r);
        if (isfinite(rd) && rd != s) {
            double other = half_neighbor(rd, s > rd ? 1 : -1);
            if (isfinite(other) && (rd + other) * 0.5 == s) {
                /* s is a midpoint only because of rounding: break the tie by err */
                double want = (err > 0) ? (rd > other ? rd : other) : (rd < other ? rd : other);
                r = dbl_to_half(want);
            }
        }
    }
    return r;
}

static uint16_t half_mul(uint16_t a, uint16_t b)
{
    return orc_float_to_half(orc_half_to_float(a) * orc_half_to_float(b));
}

/* silu_half, PackedNumericKernels.metal:19-23 */
static uint16_t silu_half(uint16_t v)
{
    float x = orc_half_to_float(v);
    return orc_float_to_half(x / (1.0f + exp_ref(-x)));
}

/* weight element k of row r as a half, per scalar-kernel format */
static uint16_t scalar_weight(int wfmt, const void *w, uint32_t r, uint32_t depth, uint32_t k)
{
    const uint8_t *b = (const uint8_t *)w;
    switch (wfmt) {
    case ORC_W_F16: return ((const uint16_t *)w)[(size_t)r * depth + k];
    case ORC_W_I8: return orc_float_to_half((float)((const int8_t *)w)[(size_t)r * depth + k]);
    case ORC_W_I4: return orc_float_to_half((float)orc_int4_decode((uint8_t)(b[(size_t)r * (depth / 2) + k / 2] >> ((k & 1) * 4))));
    case ORC_W_I2: return orc_float_to_half((float)orc_int2_decode((uint8_t)(b[(size_t)r * (depth / 4) + k / 4] >> ((k & 3) * 2))));
    case ORC_W_FP4: return orc_float_to_half(orc_e2m1_decode((uint8_t)(b[(size_t)r * (depth / 2) + k / 2] >> ((k & 1) * 4))));
    default: return 0;
    }
}

/* half_*_mlp_gate_up_benchmark, PackedNumericKernels.metal:425-664 */
void orc_scalar_mlp_gate_up(int wfmt, uint32_t T, uint32_t H, uint32_t I,
                            const uint16_t *x, const void *wg, const void *wu, uint16_t *mid)
{
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        for (int64_t c = 0; c < (int64_t)I; ++c) {
            uint16_t gate = 0, up = 0;
            for (uint32_t i = 0; i < H; ++i) {
                uint16_t xv = x[(size_t)t * H + i];
                gate = orc_half_fma(xv, scalar_weight(wfmt, wg, (uint32_t)c, H, i), gate);
                up = orc_half_fma(xv, scalar_weight(wfmt, wu, (uint32_t)c, H, i), up);
            }
            mid[(size_t)t * I + c] = half_mul(silu_half(gate), up);
        }
    }
}

/* half_*_mlp_down_benchmark, PackedNumericKernels.metal:666-832 */
void orc_scalar_mlp_down(int wfmt, uint32_t T, uint32_t H, uint32_t I,
                         const uint16_t *mid, const void *wd, uint16_t *out)
{
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        for (int64_t c = 0; c < (int64_t)H; ++c) {
            uint16_t acc = 0;
            for (uint32_t i = 0; i < I; ++i)
                acc = orc_half_fma(mid[(size_t)t * I + i], scalar_weight(wfmt, wd, (uint32_t)c, I, i), acc);
            out[(size_t)t * H + c] = acc;
        }
    }
}

/* Big-matmul rows, PackedNumericKernels.metal:98-423 */
void orc_scalar_matmul(int kind, uint32_t M, uint32_t N, uint32_t K,
                       const void *a, const void *b, void *c)
{
    const uint8_t *ab = (const uint8_t *)a, *bb = (const uint8_t *)b;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t r = 0; r < (int64_t)M; ++r) {
        for (int64_t col = 0; col < (int64_t)N; ++col) {
            size_t idx = (size_t)r * N + col;
            if (kind == 0) {          /* fp4_e2m1_matmul_benchmark :98 */
                float acc = 0.0f;
                for (uint32_t k = 0; k < K; ++k) {
                    float av = orc_e2m1_decode((uint8_t)(ab[(size_t)r * (K / 2) + k / 2] >> ((k & 1) * 4)));
                    float bv = orc_e2m1_decode((uint8_t)(bb[(size_t)col * (K / 2) + k / 2] >> ((k & 1) * 4)));
                    acc = fmaf(av, bv, acc);
                }
                ((float *)c)[idx] = acc;
            } else if (kind == 1 || kind == 2) {   /* half_fp4 :246, half_int4 :312 */
                uint16_t acc = 0;
                const uint16_t *ah = (const uint16_t *)a;
                for (uint32_t k = 0; k < K; ++k) {
                    uint16_t bw = scalar_weight(kind == 1 ? ORC_W_FP4 : ORC_W_I4, b, (uint32_t)col, K, k);
                    acc = orc_half_fma(ah[(size_t)r * K + k], bw, acc);
                }
                ((uint16_t *)c)[idx] = acc;
            } else if (kind == 3) {   /* int8_half_matmul_half_benchmark :370 */
                uint16_t acc = 0;
                const int8_t *ai = (const int8_t *)a;
                const uint16_t *bh = (const uint16_t *)b;
                for (uint32_t k = 0; k < K; ++k)
                    acc = orc_half_fma(orc_float_to_half((float)ai[(size_t)r * K + k]), bh[(size_t)col * K + k], acc);
                ((uint16_t *)c)[idx] = acc;
            } else {                  /* int4_int8_matmul_benchmark :393 */
                int32_t acc = 0;
                for (uint32_t k = 0; k < K; ++k) {
                    int av = orc_int4_decode((uint8_t)(ab[(size_t)r * (K / 2) + k / 2] >> ((k & 1) * 4)));
                    int bv = orc_int4_decode((uint8_t)(bb[(size_t)col * (K / 2) + k / 2] >> ((k & 1) * 4)));
                    acc += av * bv;
                }
                ((int32_t *)c)[idx] = acc;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Checksums, main.swift:2844-2884: 32 samples at stride count/32.      */
/* ------------------------------------------------------------------ */
double orc_sample_float_sum(const float *p, size_t count, int *samples)
{
    size_t step = count / 32 > 0 ? count / 32 : 1;
    double sum = 0.0;
    int n = 0;
    for (size_t i = 0; i < count; i += step) { sum += (double)p[i]; ++n; }
    if (samples) *samples = n;
    return sum;
}

int64_t orc_sample_int_sum(const int32_t *p, size_t count, int *samples)
{
    size_t step = count / 32 > 0 ? count / 32 : 1;
    int64_t sum = 0;
    int n = 0;
    for (size_t i = 0; i < count; i += step) { sum += p[i]; ++n; }
    if (samples) *samples = n;
    return sum;
}

uint64_t orc_sample_half_raw_sum(const uint16_t *p, size_t count, int *samples)
{
    size_t step = count / 32 > 0 ? count / 32 : 1;
    uint64_t sum = 0;
    int n = 0;
    for (size_t i = 0; i < count; i += step) { sum += p[i]; ++n; }
    if (samples) *samples = n;
    return sum;
}

/* Elementwise SwiGLU over n elements; kind as the standalone kernels:
 * 0 float->float, 1 float->half, 2 half->half, 3 int32->int8. */
void orc_swiglu_array(int kind, const void *gate, const void *up, void *mid, size_t n)
{
    for (size_t i = 0; i < n; ++i) {
        switch (kind) {
        case 0: ((float *)mid)[i] = orc_swiglu_float(((const float *)gate)[i], ((const float *)up)[i]); break;
        case 1: ((uint16_t *)mid)[i] = orc_swiglu_half(((const float *)gate)[i], ((const float *)up)[i]); break;
        case 2: ((uint16_t *)mid)[i] = orc_swiglu_half_from_half(((const uint16_t *)gate)[i], ((const uint16_t *)up)[i]); break;
        default: ((int8_t *)mid)[i] = orc_swiglu_i8(((const int32_t *)gate)[i], ((const int32_t *)up)[i]); break;
        }
    }
}

/* OCP Microscaling (MX) v1.0 quantization of fp32 weights to MXFP4 along K:
 * per block of 32, shared exponent e = floor(log2(amax)) - 2 (emax of E2M1),
 * clamped so that e + 127 is in [0, 254] and stored as that E8M0 byte;
 * elements RNE(w / 2^e) onto E2M1 with saturation. No reference counterpart
 * (the reference draws random packed bytes, main.swift:2785-2793); this is
 * the BASELINE config-0 weight recipe. */
void orc_quantize_mxfp4(const float *w, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales)
{
    for (uint32_t r = 0; r < rows; ++r) {
        for (uint32_t j = 0; j < depth / 32; ++j) {
            const float *b = w + (size_t)r * depth + (size_t)j * 32;
            double amax = 0.0;
            for (int i = 0; i < 32; ++i) amax = fmax(amax, fabs((double)b[i]));
            int e = 0, code = 0;
            if (amax > 0.0 && isfinite(amax)) {
                int ex;
                frexp(amax, &ex);
                code = ex - 1 - 2 + 127;
                code = code < 0 ? 0 : (code > 254 ? 254 : code);
                e = code - 127;
            }
            scales[(size_t)r * (depth / 32) + j] = (uint8_t)code;
            for (int i = 0; i < 32; i += 2) {
                uint8_t lo = orc_e2m1_encode((float)ldexp((double)b[i], -e));
                uint8_t hi = orc_e2m1_encode((float)ldexp((double)b[i + 1], -e));
                packed[(size_t)r * (depth / 2) + (size_t)j * 16 + i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

/* NVFP4 (no reference counterpart beyond its emulation note, README.md:383-389):
 * E2M1 elements, one UE4M3 scale per 16 along K, one fp32 tensor scale g.
 * Every step is an IEEE single-precision operation rounded to nearest even:
 *   g = amax(tensor) / 2688 (6 * 448), or 1 for an all-zero tensor;
 *   s = UE4M3((amax(block) / 6) / g), saturating at 448;
 *   element = E2M1(v * (1 / (decode(s) * g))), one correctly rounded
 *   reciprocal per block (0 when decode(s) * g == 0). */
float orc_nvfp4_tensor_scale(const float *w, size_t n)
{
    float amax = 0.0f;
    for (size_t i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(w[i]));
    return (amax > 0.0f && isfinite(amax)) ? amax / 2688.0f : 1.0f;
}

void orc_quantize_nvfp4(const float *w, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales,
                        float *tensor_scale)
{
    const float g = orc_nvfp4_tensor_scale(w, (size_t)rows * depth);
    *tensor_scale = g;
    for (uint32_t r = 0; r < rows; ++r) {
        for (uint32_t j = 0; j < depth / 16; ++j) {
            const float *b = w + (size_t)r * depth + (size_t)j * 16;
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(b[i]));
            volatile float s = amax / 6.0f;
            s = s / g;
            const uint8_t code = (uint8_t)(orc_e4m3_encode(s) & 0x7f);
            scales[(size_t)r * (depth / 16) + j] = code;
            volatile float denom = orc_e4m3_decode(code) * g;
            volatile float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
            for (int i = 0; i < 16; i += 2) {
                volatile float qa = b[i] * inv, qc = b[i + 1] * inv;
                const float a = qa, c = qc;
                const uint8_t lo = orc_e2m1_encode(a), hi = orc_e2m1_encode(c);
                packed[(size_t)r * (depth / 2) + (size_t)j * 8 + i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

void orc_decode_nvfp4(const uint8_t *packed, const uint8_t *scales, float tensor_scale, uint32_t rows,
                      uint32_t depth, double *out)
{
    for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t k = 0; k < depth; ++k) {
            const uint8_t byte = packed[(size_t)r * (depth / 2) + k / 2];
            const double e = orc_e2m1_decode((uint8_t)(byte >> ((k & 1) * 4)));
            const double s = orc_e4m3_decode(scales[(size_t)r * (depth / 16) + k / 16]);
            out[(size_t)r * depth + k] = e * s * (double)tensor_scale;
        }
}
