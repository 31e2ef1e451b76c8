/*
 * CPU formulation of the MXFP4 MLP (TEST / BASELINE INFRASTRUCTURE ONLY).
 *
 * The reference has no CPU path for this workload; its arithmetic lives in
 * Metal shaders. This file restates the MXFP4 row of the reference --
 * LUT dequant (MXFP4Kernels.metal:543-564), fp32 dot products over K,
 * mpp_mlp_swiglu_half (MPPMLPKernels.metal:204-220), fp32 down projection
 * -- as plain C with OpenMP, so that bench.py can time it on the GPU box's
 * host cores next to the CUDA path. It is never part of the product.
 *
 * Compiled separately from mpp41_oracle.c with -O3 -march=native so the
 * compiler may vectorise and contract; it is a timing baseline, checked
 * against the oracle only within a tolerance.
 */
#include "mpp41_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

static const float kLut[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                               -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

static inline float e8m0(uint8_t b)
{
    uint32_t bits = (uint32_t)b << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float h2f(uint16_t h)
{
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static inline uint16_t f2h(float f)
{
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline void dequant_row(const uint8_t *w, const uint8_t *s, uint32_t depth, float *row)
{
    for (uint32_t kb = 0; kb < depth / 32; ++kb) {
        float sc = e8m0(s[kb]);
        for (uint32_t j = 0; j < 16; ++j) {
            uint8_t byte = w[kb * 16 + j];
            row[kb * 32 + 2 * j] = kLut[byte & 0xf] * sc;
            row[kb * 32 + 2 * j + 1] = kLut[byte >> 4] * sc;
        }
    }
}

static inline float dot(const float *a, const float *b, uint32_t n)
{
    float s = 0.0f;
    #pragma omp simd reduction(+ : s)
    for (uint32_t i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

int orc_mlp_mxfp4_cpu(uint32_t T, uint32_t H, uint32_t I,
                      const uint16_t *x, const uint8_t *wg, const uint8_t *wu,
                      const uint8_t *wd, const uint8_t *sg, const uint8_t *su,
                      const uint8_t *sd, float *out, int nthreads,
                      uint32_t t0, uint32_t t1, int plain)
{
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    if (t1 > T) t1 = T;
    uint32_t nt = t1 > t0 ? t1 - t0 : 0;
    float *xf = malloc(sizeof(float) * (size_t)nt * H);
    uint16_t *mid = malloc(sizeof(uint16_t) * (size_t)nt * I);
    float *midf = malloc(sizeof(float) * (size_t)nt * I);

    for (size_t i = 0; i < (size_t)nt * H; ++i) xf[i] = h2f(x[(size_t)t0 * H + i]);

    #pragma omp parallel num_threads(nthreads)
    {
        float *rg = malloc(sizeof(float) * H);
        float *ru = malloc(sizeof(float) * H);
        #pragma omp for schedule(static)
        for (int64_t c = 0; c < (int64_t)I; ++c) {
            dequant_row(wg + (size_t)c * (H / 2), sg + (size_t)c * (H / 32), H, rg);
            dequant_row(wu + (size_t)c * (H / 2), su + (size_t)c * (H / 32), H, ru);
            for (uint32_t t = 0; t < nt; ++t) {
                float g = dot(xf + (size_t)t * H, rg, H);
                float u = dot(xf + (size_t)t * H, ru, H);
                if (plain) {
                    mid[(size_t)t * I + c] = f2h((g / (1.0f + expf(-g))) * u);
                } else {
                    float gs = g * 0.0625f;
                    gs = gs < -20.0f ? -20.0f : (gs > 20.0f ? 20.0f : gs);
                    float us = u * 0.0625f;
                    mid[(size_t)t * I + c] = f2h((gs / (1.0f + expf(-gs))) * us);
                }
            }
        }
        #pragma omp for schedule(static)
        for (int64_t i = 0; i < (int64_t)nt * I; ++i) midf[i] = h2f(mid[i]);
        float *rd = malloc(sizeof(float) * I);
        #pragma omp for schedule(static)
        for (int64_t c = 0; c < (int64_t)H; ++c) {
            dequant_row(wd + (size_t)c * (I / 2), sd + (size_t)c * (I / 32), I, rd);
            for (uint32_t t = 0; t < nt; ++t)
                out[(size_t)(t0 + t) * H + c] = dot(midf + (size_t)t * I, rd, I);
        }
        free(rg); free(ru); free(rd);
    }
    free(xf); free(mid); free(midf);
    return nthreads;
}
