// Integer tensor-core GEMM for the int8-activation rows (W8A8 / W4A8 / W2A8):
// C[m][n] = sum_k A[m][k] * B[n][k], A int8 [M][K], B int8 / INT4 / INT2
// [N][K] (the reference's packed layouts), exact int32 accumulation with
// tcgen05.mma kind::i8 (mpp_mlp_i8_{i8,i4,i2}_i32_n128, MPPMLPKernels.metal:61,
// 140, 152). INT8 weights are copied by TMA straight into the 128-byte-swizzled
// B operand; INT4/INT2 weights are sign-extended to int8 in shared memory by
// the decode warps ((n ^ 8) - 8 and ((b & 3) ^ 2) - 2, PackedNumericKernels.metal
// :330-331, 413-416).
//
// Epilogues: int32 store; int32 split-K reduction (exact, so the order of the
// atomic adds does not matter); and the gate/up pair, where one CTA holds 64
// gate and 64 up rows of the same channels and applies mpp_mlp_swiglu_i8
// (MPPMLPKernels.metal:240-257) to the int32 accumulators, writing the int8 mid.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2..5 decode, then epilogue (one TMEM lane quarter each).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace i8 {

constexpr int kBM = 128;          // tokens per tile (MMA M)
constexpr int kBN = 128;          // weight rows per tile (MMA N)
constexpr int kBK = 128;          // K per stage: one 128-byte swizzle atom of int8
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr uint32_t kATile = kBM * kBK;   // 16 KB
constexpr uint32_t kBTile = kBN * kBK;   // 16 KB

// I8_DQ_SWIGLU / I8_DQ: the scaled W8A8 layer. The int32 sums are dequantized
// as ((float)acc * row_scale[m]) * col_scale[n] (two fp32 products, in this
// order); the pair form then writes silu(g) * u as fp16, the other fp16 C.
enum I8Epi : int { I8_STORE = 0, I8_ATOMIC = 1, I8_SWIGLU = 2, I8_DQ_SWIGLU = 3, I8_DQ = 4 };

struct Params {
    CUtensorMap tm_a;         // int8 [M][K], box {128, 128}, SW128
    CUtensorMap tm_b0, tm_b1; // INT8: [N][K] box {128, rows}, SW128; INT4/INT2: packed bytes, box {raw_row, rows}
    void *out;                // int32 [M][ldc], (I8_SWIGLU) int8 mid, (I8_DQ*) fp16 [M][ldc]
    const float *row_scale;   // I8_DQ*: per-row (token) scale of A
    const float *col_scale0;  // I8_DQ*: per-output-channel scale of B (gate rows for the pair)
    const float *col_scale1;  // I8_DQ_SWIGLU: up rows
    uint32_t M, N, K, ldc;
    uint32_t k_per_split;
    uint32_t *err;
};

template <int W>
struct Cfg {
    static constexpr bool kDirect = (W == W_I8);
    static constexpr uint32_t kRawRow = kBK * wfmt_bits(W) / 8;   // packed bytes per row per stage
    static constexpr uint32_t kRawTile = kDirect ? 0 : kBN * kRawRow;
    static constexpr uint32_t kOffB = kStages * kATile;
    static constexpr uint32_t kOffRaw = kOffB + kStages * kBTile;
    static constexpr uint32_t kOffBar = kOffRaw + kStages * kRawTile;
    static constexpr uint32_t kSmem = 1024 + kOffBar + 256;
};

// 16 packed INT4 bytes (32 values, element 2i in the low nibble of byte i)
// to 32 int8 values.
__device__ __forceinline__ void int4_to_s8(uint4 v, uint32_t (&o)[8])
{
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t lo = __vsub4((w[q] & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        const uint32_t hi = __vsub4(((w[q] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        o[2 * q] = __byte_perm(lo, hi, 0x5140);       // lo0 hi0 lo1 hi1
        o[2 * q + 1] = __byte_perm(lo, hi, 0x7362);   // lo2 hi2 lo3 hi3
    }
}

// 8 packed INT2 bytes (32 values, LSB pair first) to 32 int8 values.
__device__ __forceinline__ void int2_to_s8(uint2 v, uint32_t (&o)[8])
{
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        uint32_t t[4];   // t[j] byte i = value j of input byte i
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = __vsub4(((w[q] >> (2 * j)) & 0x03030303u) ^ 0x02020202u, 0x02020202u);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t a01 = __byte_perm(t[0], t[1], b | ((4 + b) << 4));
            const uint32_t a23 = __byte_perm(t[2], t[3], b | ((4 + b) << 4));
            o[4 * q + b] = __byte_perm(a01, a23, 0x5410);
        }
    }
}

__device__ __forceinline__ int8_t swiglu_i8(int32_t g, int32_t u)
{
    // mpp_mlp_swiglu_i8, exp in double rounded to float (as the CPU oracle)
    const float gs = fminf(fmaxf((float)g * 0.000244140625f, -20.0f), 20.0f);
    const float us = (float)u * 0.000244140625f;
    const float value = (gs / (1.0f + (float)exp(-(double)gs))) * us * 32.0f;
    return (int8_t)(int)rintf(fminf(fmaxf(value, -128.0f), 127.0f));
}

template <int W, int E>
__global__ void __launch_bounds__(kThreads, 1) i8_gemm_kernel(const __grid_constant__ Params p)
{
    using C = Cfg<W>;
    constexpr bool kPair = (E == I8_SWIGLU || E == I8_DQ_SWIGLU);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + C::kOffB;
    uint8_t *sRaw = smem + C::kOffRaw;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBar);
    uint64_t *full = bars;                 // [kStages] TMA landed
    uint64_t *b_ready = bars + kStages;    // [kStages] decoded (INT4/INT2)
    uint64_t *empty = bars + 2 * kStages;  // [kStages] MMA done with the stage
    uint64_t *done = bars + 3 * kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * kStages + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m0 = blockIdx.y * kBM;
    const uint32_t c0 = blockIdx.x * (kPair ? kBN / 2 : kBN);   // first output column (pair: channel)
    const uint32_t k0 = blockIdx.z * p.k_per_split;
    const uint32_t nk = p.k_per_split / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&b_ready[s], 4);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            constexpr uint32_t tx = kATile + (C::kDirect ? kBTile : C::kRawTile);
            uint32_t s = 0;
            for (; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&empty[st], ph ^ 1u, abort, p.err, 0xA01)) break;
                mbar_arrive_expect_tx(&full[st], tx);
                const int32_t kk = (int32_t)(k0 + s * kBK);
                tma_load_2d(sA + st * kATile, &p.tm_a, kk, (int32_t)m0, &full[st]);
                uint8_t *dst = C::kDirect ? sB + st * kBTile : sRaw + st * C::kRawTile;
                const uint32_t rowb = C::kDirect ? 128u : C::kRawRow;
                const int32_t kb = (int32_t)(C::kDirect ? kk : (k0 / kBK + s) * C::kRawRow);
                if (kPair) {
                    tma_load_2d(dst, &p.tm_b0, kb, (int32_t)c0, &full[st]);
                    tma_load_2d(dst + (kBN / 2) * rowb, &p.tm_b1, kb, (int32_t)c0, &full[st]);
                } else {
                    tma_load_2d(dst, &p.tm_b0, kb, (int32_t)c0, &full[st]);
                }
            }
            for (uint32_t t = (s > kStages ? s - kStages : 0); t < s; ++t)
                mbar_wait(&full[t % kStages], (t / kStages) & 1u, nullptr, p.err, 0xA02);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_s8_s32(kBM, kBN);
            for (uint32_t s = 0; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&full[st], ph, abort, p.err, 0xA03)) break;
                if constexpr (!C::kDirect) {
                    if (!mbar_wait(&b_ready[st], ph, abort, p.err, 0xA04)) break;
                }
                tc_fence_after();
                const uint64_t ad = smem_desc_sw128(sA + st * kATile);
                const uint64_t bd = smem_desc_sw128(sB + st * kBTile);
#pragma unroll
                for (uint32_t k = 0; k < kBK / 32; ++k) mma_i8(tmem_d, ad + 2 * k, bd + 2 * k, idesc, (s | k) != 0u);
                mma_commit(&empty[st]);
            }
            mma_commit(done);
        }
    } else {
        // ------------------------------------------------ decode, then epilogue
        const uint32_t t = threadIdx.x - 64;   // 0..127: one B row per thread
        if constexpr (!C::kDirect) {
            for (uint32_t s = 0; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&full[st], ph, abort, p.err, 0xA05)) break;
                const uint8_t *raw = sRaw + st * C::kRawTile + t * C::kRawRow;
                uint8_t *row = sB + st * kBTile + t * 128;
#pragma unroll
                for (int c = 0; c < 4; ++c) {   // 32 values per chunk, 2 swizzle units of 16 bytes
                    uint32_t o[8];
                    if constexpr (W == W_I4) int4_to_s8(*reinterpret_cast<const uint4 *>(raw + 16 * c), o);
                    else int2_to_s8(*reinterpret_cast<const uint2 *>(raw + 8 * c), o);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t phys = ((2 * c + h) ^ (t & 7u)) * 16u;
                        *reinterpret_cast<uint4 *>(row + phys) = make_uint4(o[4 * h], o[4 * h + 1], o[4 * h + 2], o[4 * h + 3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_ready[st]);
            }
        }
        // ---------------------------------------------- epilogue
        mbar_wait(done, 0, abort, p.err, 0xA06);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool ok = (*abort == 0);
        tc_fence_after();
        const uint32_t quarter = warp & 3;
        const uint32_t m = m0 + quarter * 32 + lane;
        const uint32_t taddr = tmem_d + ((quarter * 32u) << 16);
        if (ok) {
            if constexpr (kPair) {
#pragma unroll 1
                for (int cc = 0; cc < kBN / 64; ++cc) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(taddr + cc * 32, g);
                    tmem_ld_32x32b_x32(taddr + kBN / 2 + cc * 32, u);
                    tmem_ld_wait();
                    const uint32_t col = c0 + cc * 32;
                    if constexpr (E == I8_DQ_SWIGLU) {
                        if (m < p.M && col < p.N) {
                            const float rs = p.row_scale[m];
                            uint32_t w[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float gf = ((float)(int32_t)g[2 * i] * rs) * p.col_scale0[col + 2 * i];
                                const float uf = ((float)(int32_t)u[2 * i] * rs) * p.col_scale1[col + 2 * i];
                                const float gf2 = ((float)(int32_t)g[2 * i + 1] * rs) * p.col_scale0[col + 2 * i + 1];
                                const float uf2 = ((float)(int32_t)u[2 * i + 1] * rs) * p.col_scale1[col + 2 * i + 1];
                                const __half2 h = __floats2half2_rn(__fdividef(gf, 1.0f + __expf(-gf)) * uf,
                                                                    __fdividef(gf2, 1.0f + __expf(-gf2)) * uf2);
                                w[i] = *reinterpret_cast<const uint32_t *>(&h);
                            }
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                        }
                    } else if (m < p.M && col < p.N) {
                        uint32_t w[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            uint32_t b = 0;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                b |= (uint32_t)(uint8_t)swiglu_i8((int32_t)g[4 * i + j], (int32_t)u[4 * i + j]) << (8 * j);
                            w[i] = b;
                        }
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<int8_t *>(p.out) + (size_t)m * p.ldc + col);
                        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                }
            } else {
#pragma unroll 1
                for (int cc = 0; cc < kBN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(taddr + cc * 32, v);
                    tmem_ld_wait();
                    const uint32_t col = c0 + cc * 32;
                    if (m < p.M && col < p.N) {
                        int32_t *dst = static_cast<int32_t *>(p.out) + (size_t)m * p.ldc + col;
                        if constexpr (E == I8_DQ) {
                            const float rs = p.row_scale[m];
                            uint32_t w[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const __half2 h = __floats2half2_rn(((float)(int32_t)v[2 * i] * rs) * p.col_scale0[col + 2 * i],
                                                                    ((float)(int32_t)v[2 * i + 1] * rs) * p.col_scale0[col + 2 * i + 1]);
                                w[i] = *reinterpret_cast<const uint32_t *>(&h);
                            }
                            uint4 *hd = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) hd[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                        } else if constexpr (E == I8_ATOMIC) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) atomicAdd(dst + i, (int32_t)v[i]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                reinterpret_cast<uint4 *>(dst)[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
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
        if (*abort) mbar_wait(done, 0, nullptr, p.err, 0xA07);   // let in-flight MMAs drain
        tc_fence_after();
        tmem_dealloc(tmem_d, kBN);
    }
}

}  // namespace i8
}  // namespace mpp41
