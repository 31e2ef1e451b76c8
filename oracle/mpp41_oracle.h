/*
 * CPU oracle for the quantized-weight MLP hot path: TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's shader arithmetic (the
 * Metal kernels under Sources/MetalFP41Probe/Shaders/ and the host data
 * generators in Sources/MetalFP41Probe/main.swift). Only tests/, the
 * smoke() check in __graft_entry__.py and bench.py's cpu_baseline / reference
 * arm may load it. The product (libmpp41) never links or calls it.
 *
 * Parity pins: the roundtrip known-answer vectors of main.swift:108-132 and
 * the published MXFP4 MLP checksum "403573 over 32 samples"
 * (README.md:292-295) -- see tests/test_oracle.py.
 */
#ifndef MPP41_ORACLE_H
#define MPP41_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded generators (main.swift:2785-2842) ---- */
void orc_make_packed_bytes(uint8_t *out, size_t n, uint32_t seed);
void orc_make_pattern_bytes(uint8_t *out, size_t n, uint32_t seed,
                            const uint8_t *pattern, size_t pattern_len);
void orc_make_fp8_e4m3_bytes(uint8_t *out, size_t n, uint32_t seed);
void orc_make_fp8_e5m2_bytes(uint8_t *out, size_t n, uint32_t seed);
void orc_make_half_values(uint16_t *out, size_t n, uint32_t seed, float scale);
void orc_make_int8_values(int8_t *out, size_t n, uint32_t seed);

/* ---- scalar codecs ---- */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);          /* round to nearest even */
float orc_e2m1_decode(uint8_t nibble);         /* MXFP4Kernels.metal:33-36 */
uint8_t orc_e2m1_encode(float x);              /* RNE, saturate to +-6 */
float orc_e4m3_decode(uint8_t code);
uint8_t orc_e4m3_encode(float x);              /* RNE, saturate to +-448 */
float orc_e5m2_decode(uint8_t code);
uint8_t orc_e5m2_encode(float x);              /* RNE, saturate to +-57344 */
float orc_e8m0_decode(uint8_t code);           /* MXFP4Kernels.metal:26-29 */
int orc_int4_decode(uint8_t nibble);           /* PackedNumericKernels.metal:30-33 */
int orc_int2_decode(uint8_t bits);             /* PackedNumericKernels.metal:25-28 */

/* ---- bulk pack / unpack (fmt: 0 = E2M1, 1 = E4M3, 2 = E5M2) ---- */
void orc_pack(int fmt, const float *in, size_t n, uint8_t *packed);
void orc_unpack(int fmt, const uint8_t *packed, size_t n, float *out);

/* ---- weight formats (shared with include/mpp41.h) ---- */
enum {
    ORC_W_F16 = 0, ORC_W_I8 = 1, ORC_W_I4 = 2, ORC_W_I2 = 3,
    ORC_W_FP4 = 4, ORC_W_E4M3 = 5, ORC_W_E5M2 = 6, ORC_W_MXFP4 = 7,
    ORC_W_E4M3_MX = 8, ORC_W_E5M2_MX = 9
};
/* Decode a weight matrix stored [rows][depth] (depth = K, contiguous) into
 * doubles. scales is [rows][depth/32] E8M0 and only read for ORC_W_MXFP4 and
 * the MXFP8 formats ORC_W_E4M3_MX / ORC_W_E5M2_MX, whose weights are
 * half(value * 2^(scale - 127)) (the fp16 dequantization rule of
 * mxfp4_dequant_*_half, MXFP4Kernels.metal:509-564, applied to FP8 elements;
 * the reference has unscaled FP8 rows only). */
void orc_decode_weights(int wfmt, const void *w, const uint8_t *scales,
                        uint32_t rows, uint32_t depth, double *out);

/* mxfp4_dequant_{native,lut}_half (MXFP4Kernels.metal:509-564). */
void orc_mxfp4_dequant_half(const uint8_t *packed, const uint8_t *scales,
                            uint16_t *out, uint32_t rows, uint32_t depth);

/* C[m][n] = sum_k A[m][k] * B[n][k] in double (full-width accumulator). */
void orc_gemm_f64(const double *a, const double *b, double *c,
                  uint32_t m, uint32_t n, uint32_t k);

/* ---- SwiGLU epilogues (MPPMLPKernels.metal:186-257) ---- */
float orc_swiglu_float(float g, float u);
uint16_t orc_swiglu_half(float g, float u);
uint16_t orc_swiglu_half_from_half(uint16_t g, uint16_t u);
int8_t orc_swiglu_i8(int32_t g, int32_t u);
/* elementwise: kind 0 float->float, 1 float->half, 2 half->half, 3 int32->int8 */
void orc_swiglu_array(int kind, const void *gate, const void *up, void *mid, size_t n);

/* ---- whole MLP rows ----
 * act: 0 = fp16 x, 1 = int8 x. epi: 0 = swiglu_float (fp32 mid),
 * 1 = swiglu_half (fp16 mid), 2 = half gate/up then swiglu_half_from_half,
 * 3 = swiglu_i8 (int8 mid, int32 accumulate), 4 = silu(g)*u in fp32 without
 * prescale and an fp16 mid.
 * out_kind: 0 = fp32, 1 = fp16 bits, 2 = int32.
 * Gate/up are exact sums rounded once to the destination type; the down
 * projection is an exact sum rounded once to the output type. */
void orc_mlp(int act, int wfmt, int epi, int out_kind,
             uint32_t tokens, uint32_t hidden, uint32_t intermediate,
             const void *x, const void *wg, const void *wu, const void *wd,
             const uint8_t *sg, const uint8_t *su, const uint8_t *sd,
             void *mid_out, void *out);
/* As orc_mlp with per-output-channel fp16 scales (INT
 * weights; no reference counterpart): sg / su / sd are fp16 [intermediate],
 * [intermediate], [hidden]; gate[t][c] = sg[c] * sum_k x[t][k] Wg[c][k] (and
 * up, down alike), each exact sum scaled before its rounding / SwiGLU. */
void orc_mlp_row_scaled(int wfmt, int epi, int out_kind,
                        uint32_t tokens, uint32_t hidden, uint32_t intermediate,
                        const void *x, const void *wg, const void *wu, const void *wd,
                        const uint16_t *sg, const uint16_t *su, const uint16_t *sd,
                        void *mid_out, void *out);

/* OCP-MX fp32 -> MXFP4 quantizer (E2M1 [rows][depth/2], E8M0 [rows][depth/32]). */
void orc_quantize_mxfp4(const float *w, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales);
float orc_nvfp4_tensor_scale(const float *w, size_t n);
void orc_quantize_nvfp4(const float *w, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales,
                        float *tensor_scale);
void orc_decode_nvfp4(const uint8_t *packed, const uint8_t *scales, float tensor_scale, uint32_t rows,
                      uint32_t depth, double *out);

/* CPU formulation of the MXFP4 MLP, timed as the CPU baseline: LUT dequant,
 * fp32 dot products, swiglu_half (plain = 0) or silu(g)*u without prescale
 * (plain = 1), fp32 down projection. nthreads <= 0 uses all OpenMP threads.
 * Returns the thread count used. */
int orc_mlp_mxfp4_cpu(uint32_t tokens, uint32_t hidden, uint32_t intermediate,
                      const uint16_t *x, const uint8_t *wg, const uint8_t *wu,
                      const uint8_t *wd, const uint8_t *sg, const uint8_t *su,
                      const uint8_t *sd, float *out, int nthreads,
                      uint32_t token_begin, uint32_t token_end, int plain);

/* ---- scalar (half-accumulate) kernels of PackedNumericKernels.metal ---- */
uint16_t orc_half_fma(uint16_t a, uint16_t b, uint16_t c);  /* fused, one rounding */
/* scalar MLP gate_up: wfmt in {F16, I8, I4, I2, FP4}; mid fp16 bits [T][I] */
void orc_scalar_mlp_gate_up(int wfmt, uint32_t tokens, uint32_t hidden,
                            uint32_t intermediate, const uint16_t *x,
                            const void *wg, const void *wu, uint16_t *mid);
void orc_scalar_mlp_down(int wfmt, uint32_t tokens, uint32_t hidden,
                         uint32_t intermediate, const uint16_t *mid,
                         const void *wd, uint16_t *out);
/* scalar big-matmul rows, kind: 0 fp4xfp4->f32, 1 half x fp4 -> half,
 * 2 half x int4 -> half, 3 int8 x half -> half, 4 int4 x int4 -> int32 */
void orc_scalar_matmul(int kind, uint32_t rows, uint32_t cols, uint32_t depth,
                       const void *a, const void *b, void *c);

/* ---- checksums (main.swift:2844-2884) ---- */
double orc_sample_float_sum(const float *p, size_t count, int *samples);
int64_t orc_sample_int_sum(const int32_t *p, size_t count, int *samples);
uint64_t orc_sample_half_raw_sum(const uint16_t *p, size_t count, int *samples);

#ifdef __cplusplus
}
#endif
#endif
