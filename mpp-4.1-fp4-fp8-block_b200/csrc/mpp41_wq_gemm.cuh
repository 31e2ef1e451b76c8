// Quantized-weight GEMM on the sm_100a tensor cores (tcgen05 kind::f16).
//
//   C[m][n] = sum_k A[m][k] * W[n][k]       A: fp16 activations [M][K]
//                                            W: packed weights [N][K] in any
//                                               reference format, decoded to
//                                               fp16 inside the CTA
//
// This is the B200 replacement for the reference's matmul2d rows:
// mpp_matmul_tile (MPPMLPKernels.metal:14-37, 13 dtype instantiations) and
// the MXFP4 native scale-plane / fused / coop-input kernels
// (MXFP4Kernels.metal:42-215, 298-359). Same operand layouts as the
// reference: A [m][k] k-contiguous, W [n][k] row-major (low nibble = even k
// for 4-bit, LSB-first pairs for 2-bit), MXFP4 scales [n][k/32] E8M0.
//
// One CTA computes a 128 x BN tile with fp32 accumulators in TMEM:
//   warp 0      TMA producer: A tile (128x64 fp16, 128B swizzle) and the raw
//               packed W tile (BN x 64 elements, unswizzled) per K stage
//   warp 1      TMEM allocation + single-thread MMA issuer (4 x K=16 / stage)
//   warps 2..5  decode W to fp16 straight into the swizzled B operand
//               (MXFP4 scale applied in the decode), then the epilogue:
//               tcgen05.ld -> fused SwiGLU / store / split-K atomic add.
// With the SwiGLU epilogue the B tile holds BN/2 gate rows then BN/2 up rows
// of the same channels, so each thread sees gate and up of its token and the
// gate/up activations never leave the SM (fusing mpp_mlp_swiglu_*,
// MPPMLPKernels.metal:186-238, into the GEMM).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"

namespace mpp41 {

enum Epi : int {
    EPI_STORE_F32 = 0,       // C fp32 (matmul2d ..._f rows)
    EPI_STORE_F16 = 1,       // C fp16, one rounding of the fp32 sum (..._h rows)
    EPI_ATOMIC_F32 = 2,      // C += partial (split-K), fp32
    EPI_SWIGLU_FLOAT = 3,    // mid fp32 = silu(g) * u                 (mpp_mlp_swiglu_float)
    EPI_SWIGLU_HALF = 4,     // mid fp16 = silu(clamp(g/16)) * u/16    (mpp_mlp_swiglu_half)
    EPI_SWIGLU_HALF_H = 5,   // g,u rounded to fp16 first              (mpp_mlp_swiglu_half_from_half)
    EPI_SWIGLU_PLAIN = 6,    // mid fp16 = silu(g) * u in fp32, no prescale (OCP-MX model rows)
    EPI_SPLITK_F16 = 7,      // split-K: fp32 partials into a workspace, last CTA of a tile writes fp16
};

constexpr int kBM = 128;        // tokens per tile (MMA M)
constexpr int kBK = 64;         // K per stage: one 128-byte swizzle atom of fp16
constexpr int kStages = 6;
constexpr int kThreads = 192;   // 6 warps

struct WqGemmParams {
    CUtensorMap tmap_a;         // A [M][K] fp16, box {64, 128}, swizzle 128B
    CUtensorMap tmap_b0;        // W (or gate W): raw bytes, or fp16 swizzled for W_F16
    CUtensorMap tmap_b1;        // up W for the SwiGLU pair
    const uint8_t *scales0;     // MXFP4 scales [N][K/32] for b0
    const uint8_t *scales1;     // ... for b1
    void *out;                  // C [M][ldc] or mid [M][ldc]
    uint32_t M, N, K;           // N = output columns (channels)
    uint32_t k_per_split;       // K range of blockIdx.z
    uint32_t ldc;
    uint32_t *err;              // device error word
    float4 *zero;               // optional buffer cleared by this grid (for a later split-K GEMM)
    uint32_t zero_vec4;         // its size in float4 units
    float *ws;                  // EPI_SPLITK_F16: fp32 workspace [M][ldc], clear on entry
    uint32_t *tile_count;       // EPI_SPLITK_F16: one arrival counter per output tile, clear on entry
};

template <int W, int BN, int E>
struct WqCfg {
    static constexpr bool kPair = (E >= EPI_SWIGLU_FLOAT && E <= EPI_SWIGLU_PLAIN);
    static constexpr bool kDirect = (W == W_F16);
    static constexpr int kRawRow = (W == W_F16) ? 0 : kBK * wfmt_bits(W) / 8;   // bytes per row per stage
    static constexpr int kCols = kPair ? BN / 2 : BN;                         // output columns per CTA
    static constexpr uint32_t kABytes = kBM * 128;
    static constexpr uint32_t kBBytes = BN * 128;
    static constexpr uint32_t kRawBytes = BN * kRawRow;
    static constexpr uint32_t kStageTx = kABytes + (kDirect ? kBBytes : kRawBytes);
    static constexpr uint32_t kOffB = kStages * kABytes;
    static constexpr uint32_t kOffRaw = kOffB + kStages * kBBytes;
    static constexpr uint32_t kOffScales = kOffRaw + kStages * kRawBytes;
    static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
    static uint32_t smem_bytes(uint32_t k_per_split)
    {
        uint32_t sc = (W == W_MXFP4) ? BN * (k_per_split / 32) : 0;
        sc = (sc + 15u) & ~15u;
        return 1024 /*align slack*/ + kOffScales + sc + 256 /*barriers*/;
    }
    static_assert(BN % 64 == 0 && BN <= 256, "BN must be 64, 128, 192 or 256");
};

// ----------------------------------------------------------------- decode
// Decode 32 consecutive weights, given as their packed bytes in wr (FP4/
// INT4: wr[0..3]; INT2: wr[0..1]; 8-bit formats: wr[0..7]; little-endian,
// element 0 in the lowest bits), into 16 fp16x2 words (element 2i in the low
// half of word i).
template <int W>
__device__ __forceinline__ void decode_words(const uint32_t (&wr)[8], uint32_t scale_byte, uint32_t (&o)[16])
{
    if constexpr (W == W_FP4 || W == W_MXFP4) {
        // hardware E2M1 pair conversion (low nibble -> low half): the exact E2M1
        // values in fp16; then value * 2^(s-127) with one exact fp16 multiply when
        // 2^(s-127) is a normal fp16 (s in [113,142]); otherwise fp32 math and a
        // single rounding, as half(float(lut) * e8m0) in mxfp4_dequant_*_half.
        const uint32_t *w = wr;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
                "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
                "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
                "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
                "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
                "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
                : "=r"(o[4 * q]), "=r"(o[4 * q + 1]), "=r"(o[4 * q + 2]), "=r"(o[4 * q + 3])
                : "r"(w[q]));
        }
        if constexpr (W == W_MXFP4) {
            const uint32_t s = scale_byte;
            if (s >= 113u && s <= 142u) {
                if (s != 127u) {
                    const uint32_t f = ((s - 112u) << 10) * 0x10001u;   // 2^(s-127) as fp16x2
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = hmul2_bits(o[i], f);
                }
            } else {
                const float sf = e8m0_to_float(s);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    __half2 h = *reinterpret_cast<__half2 *>(&o[i]);
                    o[i] = half2_bits(__low2float(h) * sf, __high2float(h) * sf);
                }
            }
        }
    } else if constexpr (W == W_I4) {
        const uint32_t *w = wr;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t lo = w[q] & 0x0F0F0F0Fu, hi = (w[q] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t h = __byte_perm(lo, hi, j | ((4 + j) << 8));
                const uint32_t x = ((h & 0x000F000Fu) | 0x64006400u) ^ 0x00080008u;   // 1024 + (n ^ 8)
                o[4 * q + j] = hsub2_bits(x, 0x64086408u);                          // - 1032
            }
        }
    } else if constexpr (W == W_I2) {
        const uint32_t *w = wr;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t t = (w[q] >> (8 * j)) & 0xFFu;
                const uint32_t x0 = (t | (t << 14)) & 0x00030003u;           // codes 0,1 of the byte
                const uint32_t x1 = ((t >> 4) | (t << 10)) & 0x00030003u;    // codes 2,3
                o[8 * q + 2 * j] = hsub2_bits((x0 ^ 0x00020002u) | 0x64006400u, 0x64026402u);
                o[8 * q + 2 * j + 1] = hsub2_bits((x1 ^ 0x00020002u) | 0x64006400u, 0x64026402u);
            }
        }
    } else if constexpr (W == W_I8) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t *w = wr + 4 * q;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t a = __byte_perm(w[i], 0x64646464u, 0x4140) ^ 0x00800080u;
                const uint32_t b = __byte_perm(w[i], 0x64646464u, 0x4342) ^ 0x00800080u;
                o[8 * q + 2 * i] = hsub2_bits(a, 0x64806480u);        // 1024 + (v+128) - 1152
                o[8 * q + 2 * i + 1] = hsub2_bits(b, 0x64806480u);
            }
        }
    } else if constexpr (W == W_E4M3_MX || W == W_E5M2_MX) {
        // FP8 bytes decoded exactly (as below), then value * 2^(s-127) rounded
        // once to fp16: one fp16 multiply by an exactly representable power of
        // two (both operands exact, so RN(product) = half(value * scale)), else
        // fp32 math and a single rounding -- the rule of mxfp4_dequant_*_half.
        decode_words<W == W_E4M3_MX ? W_E4M3 : W_E5M2>(wr, 127u, o);
        const uint32_t s = scale_byte;
        if (s >= 113u && s <= 142u) {
            if (s != 127u) {
                const uint32_t f = ((s - 112u) << 10) * 0x10001u;   // 2^(s-127) as fp16x2
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = hmul2_bits(o[i], f);
            }
        } else {
            const float sf = e8m0_to_float(s);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                __half2 h = *reinterpret_cast<__half2 *>(&o[i]);
                o[i] = half2_bits(__low2float(h) * sf, __high2float(h) * sf);
            }
        }
    } else if constexpr (W == W_E4M3) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t *w = wr + 4 * q;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    // bytes (2p, 2p+1) -> halves; E4M3 bits placed as fp16 bits of value * 2^-8
                    const uint32_t x = __byte_perm(w[i], 0u, p == 0 ? 0x4140 : 0x4342);  // byte in low 8 bits of each half
                    const uint32_t r = ((x & 0x007F007Fu) << 7) | ((x & 0x00800080u) << 8);
                    o[8 * q + 2 * i + p] = hmul2_bits(r, 0x5C005C00u);   // * 256
                }
            }
        }
    } else if constexpr (W == W_E5M2) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t *w = wr + 4 * q;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[8 * q + 2 * i] = __byte_perm(w[i], 0u, 0x1404);      // E5M2 byte == fp16 high byte
                o[8 * q + 2 * i + 1] = __byte_perm(w[i], 0u, 0x3424);
            }
        }
    }
}


// Packed bytes per 32 weights of format W.
template <int W>
__host__ __device__ constexpr int chunk_bytes() { return 32 * wfmt_bits(W) / 8; }

// Decode the 32 consecutive weights at `raw` (shared memory, 8-byte aligned)
// into 16 fp16x2 words.
template <int W>
__device__ __forceinline__ void decode_chunk(const uint8_t *raw, uint32_t scale_byte, uint32_t (&o)[16])
{
    uint32_t w[8];
    if constexpr (chunk_bytes<W>() == 8) {
        const uint2 v = *reinterpret_cast<const uint2 *>(raw);
        w[0] = v.x; w[1] = v.y;
    } else {
#pragma unroll
        for (int q = 0; q < chunk_bytes<W>() / 16; ++q) {
            const uint4 v = *reinterpret_cast<const uint4 *>(raw + 16 * q);
            w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
        }
    }
    decode_words<W>(w, scale_byte, o);
}

// ----------------------------------------------------------------- epilogue math
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

template <int E>
__device__ __forceinline__ float swiglu(float g, float u)
{
    if constexpr (E == EPI_SWIGLU_PLAIN) {
        // OCP-MX model rows (no reference bit pattern to match): hardware
        // exp2 and fast divide; silu(g) -> 0 when exp(-g) overflows
        return __fdividef(g, 1.0f + __expf(-g)) * u;
    } else if constexpr (E == EPI_SWIGLU_FLOAT) {
        return (g / (1.0f + expf(-g))) * u;
    } else {
        if constexpr (E == EPI_SWIGLU_HALF_H) {
            g = __half2float(__float2half_rn(g));
            u = __half2float(__float2half_rn(u));
        }
        float gs = fminf(fmaxf(g * 0.0625f, -20.0f), 20.0f);
        float us = u * 0.0625f;
        return (gs / (1.0f + expf(-gs))) * us;
    }
}

// ----------------------------------------------------------------- kernel
template <int W, int BN, int E>
__global__ void __launch_bounds__(kThreads, 1) wq_gemm_kernel(const __grid_constant__ WqGemmParams p)
{
    using Cfg = WqCfg<W, BN, E>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + Cfg::kOffB;
    uint8_t *sRaw = smem + Cfg::kOffRaw;
    uint8_t *sScale = smem + Cfg::kOffScales;
    const uint32_t kbc = p.k_per_split / 32;   // scale blocks per CTA
    uint32_t scale_bytes = (W == W_MXFP4) ? ((BN * kbc + 15u) & ~15u) : 0u;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sScale + scale_bytes);
    uint64_t *raw_full = bars;
    uint64_t *b_ready = bars + kStages;
    uint64_t *empty = bars + 2 * kStages;
    uint64_t *done = bars + 3 * kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * kStages + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile uint32_t *s_last = tmem_slot + 2;   // split-K: this CTA finishes its tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_tile = blockIdx.x, m0 = blockIdx.y * kBM;
    const uint32_t k0 = blockIdx.z * p.k_per_split;
    const uint32_t nk = p.k_per_split / kBK;
    const uint32_t c0 = n_tile * Cfg::kCols;   // first output column of this CTA

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&b_ready[s], 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.tmap_a);
        tma_prefetch_desc(&p.tmap_b0);
        if (Cfg::kPair) tma_prefetch_desc(&p.tmap_b1);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    if (p.zero && warp <= 1 && lane >= 1) {
        // lanes 1..31 of warps 0 and 1 have no pipeline role: clear this CTA's
        // slice of the buffer a following split-K GEMM accumulates into
        const uint32_t ctas = gridDim.x * gridDim.y * gridDim.z;
        const uint32_t cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        const uint32_t per = (p.zero_vec4 + ctas - 1) / ctas;
        const uint32_t beg = cta * per, end = min(beg + per, p.zero_vec4);
        for (uint32_t i = beg + warp * 31 + (lane - 1); i < end; i += 62) p.zero[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t s = 0;
            for (; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&empty[st], ph ^ 1u, abort, p.err, 0x101)) break;
                mbar_arrive_expect_tx(&raw_full[st], Cfg::kStageTx);
                const int32_t kk = (int32_t)(k0 + s * kBK);
                tma_load_2d(sA + st * Cfg::kABytes, &p.tmap_a, kk, (int32_t)m0, &raw_full[st]);
                if constexpr (Cfg::kDirect) {
                    uint8_t *dst = sB + st * Cfg::kBBytes;
                    if constexpr (Cfg::kPair) {
                        tma_load_2d(dst, &p.tmap_b0, kk, (int32_t)c0, &raw_full[st]);
                        tma_load_2d(dst + (BN / 2) * 128, &p.tmap_b1, kk, (int32_t)c0, &raw_full[st]);
                    } else {
                        tma_load_2d(dst, &p.tmap_b0, kk, (int32_t)c0, &raw_full[st]);
                    }
                } else {
                    uint8_t *dst = sRaw + st * Cfg::kRawBytes;
                    const int32_t kb = (int32_t)((k0 / kBK + s) * Cfg::kRawRow);
                    if constexpr (Cfg::kPair) {
                        tma_load_2d(dst, &p.tmap_b0, kb, (int32_t)c0, &raw_full[st]);
                        tma_load_2d(dst + (BN / 2) * Cfg::kRawRow, &p.tmap_b1, kb, (int32_t)c0, &raw_full[st]);
                    } else {
                        tma_load_2d(dst, &p.tmap_b0, kb, (int32_t)c0, &raw_full[st]);
                    }
                }
            }
            // Never leave the CTA with loads in flight: wait for the last issued
            // round of every stage (immediate in the normal case).
            for (uint32_t t = (s > kStages ? s - kStages : 0); t < s; ++t)
                mbar_wait(&raw_full[t % kStages], (t / kStages) & 1u, nullptr, p.err, 0x102);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
            for (uint32_t s = 0; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&raw_full[st], ph, abort, p.err, 0x201)) break;
                if constexpr (!Cfg::kDirect) {
                    if (!mbar_wait(&b_ready[st], ph, abort, p.err, 0x202)) break;
                }
                tc_fence_after();
                const uint64_t ad = smem_desc_sw128(sA + st * Cfg::kABytes);
                const uint64_t bd = smem_desc_sw128(sB + st * Cfg::kBBytes);
#pragma unroll
                for (uint32_t k = 0; k < kBK / 16; ++k)
                    mma_f16(tmem_d, ad + 2 * k, bd + 2 * k, idesc, (s | k) != 0u);
                mma_commit(&empty[st]);
            }
            mma_commit(done);
        }
    } else {
        // ------------------------------------------------ decode, then epilogue
        const uint32_t t = threadIdx.x - 64;   // 0..127
        if constexpr (W == W_MXFP4) {
            // This CTA's scales: BN rows x kbc bytes. Rows are contiguous in the
            // [N][K/32] plane, so with 16-byte aligned rows every thread issues its
            // 16-byte loads back to back (one memory latency for the whole set).
            const uint32_t kb0 = k0 / 32, kblocks = p.K / 32;
            if ((kblocks & 15u) == 0 && (kb0 & 15u) == 0 && (kbc & 15u) == 0) {
                const uint32_t per_row = kbc / 16, nchunk = BN * per_row;
                for (uint32_t base = t; base < nchunk; base += 128 * 4) {
                    uint4 v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t c = base + 128u * j;
                        if (c < nchunk) {
                            const uint32_t r = c / per_row, q = c % per_row;
                            uint32_t row = c0 + r;
                            const uint8_t *sp = p.scales0;
                            if (Cfg::kPair && r >= BN / 2) { row = c0 + r - BN / 2; sp = p.scales1; }
                            v[j] = row < p.N ? __ldg(reinterpret_cast<const uint4 *>(sp + (size_t)row * kblocks + kb0) + q)
                                             : make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t c = base + 128u * j;
                        if (c < nchunk) reinterpret_cast<uint4 *>(sScale)[c] = v[j];
                    }
                }
            } else {
                for (uint32_t i = t; i < BN * kbc; i += 128) {
                    const uint32_t r = i / kbc, j = i % kbc;
                    uint32_t row = c0 + r;
                    const uint8_t *sp = p.scales0;
                    if (Cfg::kPair && r >= BN / 2) { row = c0 + r - BN / 2; sp = p.scales1; }
                    sScale[i] = (row < p.N) ? __ldg(sp + (size_t)row * kblocks + kb0 + j) : (uint8_t)127;
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        if constexpr (!Cfg::kDirect) {
            for (uint32_t s = 0; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&raw_full[st], ph, abort, p.err, 0x301)) break;
                const uint8_t *raw = sRaw + st * Cfg::kRawBytes;
                uint8_t *bt = sB + st * Cfg::kBBytes;
#pragma unroll
                for (int j = 0; j < BN / 64; ++j) {
                    const uint32_t c = t + 128u * j, r = c >> 1, h = c & 1u;
                    uint32_t sb = 127u;
                    if constexpr (W == W_MXFP4) sb = sScale[r * kbc + 2 * s + h];
                    uint32_t o[16];
                    decode_chunk<W>(raw + r * Cfg::kRawRow + h * (Cfg::kRawRow / 2), sb, o);
                    uint8_t *row = bt + r * 128;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t phys = ((h * 4 + q) ^ (r & 7u)) * 16u;
                        *reinterpret_cast<uint4 *>(row + phys) =
                            make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&b_ready[st]);
            }
        }
        // ---------------------------------------------- epilogue
        // all 128 epilogue threads take the same branch: a wait that gave up set
        // *abort before this barrier
        mbar_wait(done, 0, abort, p.err, 0x401);
        asm volatile("bar.sync 3, 128;" ::: "memory");
        const bool ok = (*abort == 0);
        tc_fence_after();
        const uint32_t quarter = warp & 3;               // TMEM lanes 32*quarter .. +31
        const uint32_t row = quarter * 32 + lane;
        const uint32_t m = m0 + row;
        const uint32_t taddr = tmem_d + ((quarter * 32u) << 16);
        if (ok) {
            if constexpr (Cfg::kPair) {
#pragma unroll 1
                for (int cc = 0; cc < Cfg::kCols / 32; ++cc) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(taddr + cc * 32, g);
                    tmem_ld_32x32b_x32(taddr + Cfg::kCols + cc * 32, u);
                    tmem_ld_wait();
                    const uint32_t col = c0 + cc * 32;
                    if (m < p.M && col < p.N) {
                        if constexpr (E == EPI_SWIGLU_FLOAT) {
                            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                dst[i] = make_float4(swiglu<E>(__uint_as_float(g[4 * i]), __uint_as_float(u[4 * i])),
                                                     swiglu<E>(__uint_as_float(g[4 * i + 1]), __uint_as_float(u[4 * i + 1])),
                                                     swiglu<E>(__uint_as_float(g[4 * i + 2]), __uint_as_float(u[4 * i + 2])),
                                                     swiglu<E>(__uint_as_float(g[4 * i + 3]), __uint_as_float(u[4 * i + 3])));
                        } else {
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint32_t w[4];
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const int e = 8 * i + 2 * j;
                                    w[j] = half2_bits(swiglu<E>(__uint_as_float(g[e]), __uint_as_float(u[e])),
                                                      swiglu<E>(__uint_as_float(g[e + 1]), __uint_as_float(u[e + 1])));
                                }
                                dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                            }
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(taddr + cc * 32, v);
                    tmem_ld_wait();
                    const uint32_t col = c0 + cc * 32;
                    if (m < p.M && col < p.N) {
                        if constexpr (E == EPI_STORE_F32) {
                            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                     __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                        } else if constexpr (E == EPI_ATOMIC_F32 || E == EPI_SPLITK_F16) {
                            float4 *dst = reinterpret_cast<float4 *>((E == EPI_ATOMIC_F32 ? static_cast<float *>(p.out) : p.ws) +
                                                                     (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                atomicAdd(dst + i, make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                               __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
                        } else {
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int e = 8 * i;
                                dst[i] = make_uint4(half2_bits(__uint_as_float(v[e]), __uint_as_float(v[e + 1])),
                                                    half2_bits(__uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])),
                                                    half2_bits(__uint_as_float(v[e + 4]), __uint_as_float(v[e + 5])),
                                                    half2_bits(__uint_as_float(v[e + 6]), __uint_as_float(v[e + 7])));
                            }
                        }
                    }
                }
            }
            if constexpr (E == EPI_SPLITK_F16) {
                // Publish this CTA's partial, count arrivals per output tile; the
                // last CTA of the tile converts the fp32 sum to fp16.
                __threadfence();
                asm volatile("bar.sync 2, 128;" ::: "memory");
                const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
                if (threadIdx.x == 64) *s_last = (atomicAdd(p.tile_count + tile, 1u) == gridDim.z - 1) ? 1u : 0u;
                asm volatile("bar.sync 2, 128;" ::: "memory");
                if (*s_last) {
                    __threadfence();
                    // 128 threads x 16 columns per row-pass: coalesced 64-byte row segments
                    const uint32_t r0 = threadIdx.x - 64;
                    for (uint32_t i = r0; i < kBM * (BN / 8); i += 128) {
                        const uint32_t rr = i / (BN / 8), cc = (i % (BN / 8)) * 8;
                        const uint32_t mm = m0 + rr;
                        if (mm < p.M) {
                            const float *src = p.ws + (size_t)mm * p.ldc + c0 + cc;
                            const float4 a = __ldcg(reinterpret_cast<const float4 *>(src));
                            const float4 b = __ldcg(reinterpret_cast<const float4 *>(src) + 1);
                            *reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)mm * p.ldc + c0 + cc) =
                                make_uint4(half2_bits(a.x, a.y), half2_bits(a.z, a.w), half2_bits(b.x, b.y),
                                           half2_bits(b.z, b.w));
                        }
                    }
                }
            }
        }
    }

    // ---------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (*abort) {
            // the final commit was issued unconditionally; let in-flight MMAs drain
            mbar_wait(done, 0, nullptr, p.err, 0x501);
        }
        tc_fence_after();
        tmem_dealloc(tmem_d, Cfg::kTmemCols);
    }
}

}  // namespace mpp41
