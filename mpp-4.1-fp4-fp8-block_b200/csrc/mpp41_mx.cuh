// OCP-MX (Microscaling v1.0) MXFP4 encoding shared by the standalone
// quantizer kernels and the W4A4 GEMM epilogue, so that both produce the same
// bytes for the same fp32 block.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace mpp41 {

// cvt.rn.satfinite.e2m1x2.f32 rounds to nearest even and saturates to +-6,
// the behaviour the reference's pack<> shows (main.swift:112-130).
__device__ __forceinline__ uint32_t enc_e2m1x2(float lo, float hi)
{
    uint16_t r;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}" : "=h"(r) : "f"(hi), "f"(lo));
    return r & 0xFFu;
}

// One block of 32 values -> 16 packed bytes (low nibble = even index) and the
// E8M0 scale byte. Shared exponent e = floor(log2(amax)) - 2 (2 = emax of
// E2M1), stored as e + 127 clamped to [0, 254]; elements are v * 2^-e rounded
// to nearest even E2M1 with saturation. An all-zero (or non-finite) block gets
// scale byte 0 and zero elements.
__device__ __forceinline__ uint32_t mx_quant32(const float (&v)[32], uint4 &packed)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    int e = 0;
    uint32_t code = 0;
    if (amax > 0.0f && isfinite(amax)) {
        int ex;
        frexpf(amax, &ex);   // amax = m * 2^ex, m in [0.5, 1): floor(log2) = ex - 1
        int c = ex - 1 - 2 + 127;
        c = c < 0 ? 0 : (c > 254 ? 254 : c);
        code = (uint32_t)c;
        e = c - 127;
    }
    const float inv = ldexpf(1.0f, -e);   // exact power of two
    uint32_t out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) word |= enc_e2m1x2(v[8 * q + 2 * i] * inv, v[8 * q + 2 * i + 1] * inv) << (8 * i);
        out[q] = word;
    }
    packed = make_uint4(out[0], out[1], out[2], out[3]);
    return code;
}

// ------------------------------------------------------------------ NVFP4
// NVFP4: E2M1 elements, one UE4M3 scale per 16 and an fp32 tensor scale g.
// Recipe (all steps IEEE fp32, round to nearest even):
//   g = amax(tensor) / (6 * 448)            (1 for an all-zero tensor)
//   s = E4M3((amax(block) / 6) / g)         (saturating; 0 when it underflows)
//   q = E2M1(v * (1 / (decode(s) * g)))     (0 when decode(s) == 0; one
//                                            correctly rounded reciprocal per block)
// so value = q * decode(s) * g, and the largest block scale lands on 448.
__host__ __device__ __forceinline__ float nvfp4_tensor_scale(float amax)
{
    return (amax > 0.0f && amax <= 3.4e38f) ? amax / 2688.0f : 1.0f;
}

__device__ __forceinline__ uint32_t enc_ue4m3(float s)
{
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(s));
    return r & 0xFFu;
}

__device__ __forceinline__ float dec_ue4m3(uint32_t code)
{
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((uint16_t)code));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// One block of 16 values -> 8 packed bytes (low nibble = even index) and the
// UE4M3 scale byte.
__device__ __forceinline__ uint32_t nv_quant16(const float (&v)[16], float g, uint2 &packed)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint32_t code = enc_ue4m3(__fdiv_rn(__fdiv_rn(amax, 6.0f), g));
    const float denom = __fmul_rn(dec_ue4m3(code), g);
    const float inv = denom > 0.0f ? __frcp_rn(denom) : 0.0f;
    uint32_t out[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            word |= enc_e2m1x2(__fmul_rn(v[8 * q + 2 * i], inv), __fmul_rn(v[8 * q + 2 * i + 1], inv)) << (8 * i);
        out[q] = word;
    }
    packed = make_uint2(out[0], out[1]);
    return code;
}

}  // namespace mpp41
