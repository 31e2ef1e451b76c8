// Persistent form of the block-scaled FP4 GEMM (same math, operands, scale
// layout and epilogues as mpp41_mxf4_gemm.cuh) for weight-streaming shapes:
// grouped expert GEMMs and launches with few rows. One CTA per SM walks the
// (row tile, column tile) grid with a static stride; its loads never stop at a
// tile boundary, so the next tile's operands stream in while this tile's MMAs
// finish and its epilogue runs.
//
// Tile 128 x 128, 6 shared-memory stages (216 KB). Tensor memory: two 128-column
// accumulators, then the scale ring (6 stages x 16 or 32 columns). The
// epilogue copies a whole accumulator into registers and releases it before
// converting and storing, so the MMAs of the tile after next can start.
//
// Warp roles (320 threads): 0 TMA producer, 1 TMEM owner + MMA issuer, 2..5
// scales into tensor memory, 6..9 epilogue (warp w reads lane quarter w % 4).
#pragma once

#include "mpp41_mxf4_gemm.cuh"

namespace mpp41 {
namespace mxf4 {

constexpr int kPBN = 128;
constexpr int kPStages = 6;
constexpr int kPThreads = 320;
constexpr uint32_t kPBHalf = 64 * 128;
constexpr uint32_t kPBTile = kPBN * 128;
constexpr uint32_t kPSfbBytes = kPBN * kSfRow;
constexpr uint32_t kPOffB = kPStages * kATile;
constexpr uint32_t kPOffSfa = kPOffB + kPStages * kPBTile;
constexpr uint32_t kPOffSfb = kPOffSfa + kPStages * kSfaBytes;
constexpr uint32_t kPOffBar = kPOffSfb + kPStages * kPSfbBytes;
constexpr uint32_t kPSmem = 1024 + kPOffBar + 256;
static_assert(kPSmem <= 227 * 1024, "shared memory");
static_assert(2 * kPBN + kPStages * (SfCols<true, 128>::kA + SfCols<true, 128>::kB) <= 512, "tensor memory");

struct PTile {
    uint32_t m0, m_end, col;
    int32_t rb0, rb1;
};

__device__ __forceinline__ bool ptile(const Params &p, uint32_t t, PTile &o)
{
    const uint32_t r = t / p.col_tiles, c = t % p.col_tiles;
    uint32_t b_off = 0;
    if (p.tiles) {
        const uint4 e = p.tiles[r];
        o.m0 = e.y;
        o.m_end = e.z;
        b_off = e.x * p.b_expert_rows;
    } else {
        o.m0 = r * kBM;
        o.m_end = p.M;
    }
    o.col = c;
    o.rb0 = (int32_t)(b_off + p.b0_row0 + c * p.b_row_step);
    o.rb1 = (int32_t)(b_off + p.b1_row0 + c * p.b_row_step);
    return true;
}

template <int E, bool NV>
__global__ void __launch_bounds__(kPThreads, 1) mxf4_persist_kernel(const __grid_constant__ Params p)
{
    constexpr int S = kPStages;
    constexpr uint32_t kSfaCols = SfCols<NV, kPBN>::kA, kSfbCols = SfCols<NV, kPBN>::kB;
    constexpr uint32_t kRing0 = 2 * kPBN;   // scale ring after the two accumulators
    constexpr int RB = kPBN / 32;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem, *sB = smem + kPOffB, *sSa = smem + kPOffSfa, *sSb = smem + kPOffSfb;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kPOffBar);
    uint64_t *full = bars;                  // [S] TMA landed
    uint64_t *sf_ready = bars + S;          // [S] scales in tensor memory
    uint64_t *empty = bars + 2 * S;         // [S] MMA done with the stage
    uint64_t *acc_full = bars + 3 * S;      // [2] accumulator complete
    uint64_t *acc_empty = bars + 3 * S + 2; // [2] accumulator copied out by the epilogue
    uint64_t *drain = bars + 3 * S + 4;     // all MMAs issued have completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 5);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row_tiles = p.tiles ? *p.n_tiles : (p.M + kBM - 1) / kBM;
    const uint32_t total = row_tiles * p.col_tiles;
    const uint32_t nk = p.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&sf_ready[s], 4);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // The producer and MMA warps run converged: every wait is made by the whole
    // warp, every copy / MMA issued by one elected lane.
    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        uint32_t g = 0;
        bool alive = true;
        for (uint32_t t = blockIdx.x; t < total && alive; t += gridDim.x) {
            PTile tl;
            ptile(p, t, tl);
            for (uint32_t kk = 0; kk < nk; ++kk, ++g) {
                const uint32_t st = g % S, ph = (g / S) & 1u;
                if (!warp_wait(&empty[st], ph ^ 1u, abort, p.err, 0xD01)) { alive = false; break; }
                if (elect_one_sync()) {
                    mbar_arrive_expect_tx(&full[st], kATile + kPBTile + kSfaBytes + kPSfbBytes);
                    const int32_t kb = (int32_t)(kk * (kBK / 2));
                    const int32_t ks = (int32_t)((NV ? kk : (kk >> 1)) * kSfRow);
                    tma_load_2d(sA + st * kATile, &p.tm_a, kb, (int32_t)tl.m0, &full[st]);
                    tma_load_2d(sB + st * kPBTile, &p.tm_b0, kb, tl.rb0, &full[st]);
                    tma_load_2d(sB + st * kPBTile + kPBHalf, &p.tm_b1, kb, tl.rb1, &full[st]);
                    tma_load_2d(sSa + st * kSfaBytes, &p.tm_sa, ks, (int32_t)tl.m0, &full[st]);
                    tma_load_2d(sSb + st * kPSfbBytes, &p.tm_sb0, ks, tl.rb0, &full[st]);
                    tma_load_2d(sSb + st * kPSfbBytes + 64 * kSfRow, &p.tm_sb1, ks, tl.rb1, &full[st]);
                }
                __syncwarp();
            }
        }
        // drain: no copy may still be landing when the CTA exits
        for (uint32_t q = (g > (uint32_t)S ? g - S : 0); q < g; ++q)
            mbar_wait(&full[q % S], (q / S) & 1u, nullptr, p.err, 0xD02);
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        uint32_t g = 0, j = 0;
        bool alive = true;
        for (uint32_t t = blockIdx.x; t < total && alive; t += gridDim.x, ++j) {
            const uint32_t b = j & 1u, use = j >> 1;
            if (!warp_wait(&acc_empty[b], (use & 1u) ^ 1u, abort, p.err, 0xD03)) break;
            tc_fence_after();
            const uint32_t acc = tmem + b * kPBN;
            for (uint32_t kk = 0; kk < nk; ++kk, ++g) {
                const uint32_t st = g % S, ph = (g / S) & 1u;
                if (!warp_wait(&sf_ready[st], ph, abort, p.err, 0xD04)) { alive = false; break; }
                tc_fence_after();
                if (elect_one_sync()) {
                    const uint64_t ad = smem_desc_sw128(sA + st * kATile);
                    const uint64_t bd = smem_desc_sw128(sB + st * kPBTile);
                    const uint32_t sfa0 = tmem + kRing0 + st * (kSfaCols + kSfbCols);
                    const uint32_t sfb0 = sfa0 + kSfaCols;
#pragma unroll
                    for (uint32_t k = 0; k < kBK / 64; ++k) {
                        if constexpr (NV) {
                            mma_nvf4(acc, ad + 2 * k, bd + 2 * k, idesc_nvf4(kBM, kPBN), sfa0 + (kBM / 32) * k,
                                     sfb0 + RB * k, (kk | k) != 0u);
                        } else {
                            const uint32_t gq = k >> 1, h = (k & 1u) * 2u;
                            mma_mxf4(acc, ad + 2 * k, bd + 2 * k, idesc_mxf4(kBM, kPBN, h, h),
                                     (sfa0 + (kBM / 32) * gq) | (h << 30), (sfb0 + RB * gq) | (h << 30),
                                     (kk | k) != 0u);
                        }
                    }
                    mma_commit(&empty[st]);
                }
                __syncwarp();
            }
            if (alive && elect_one_sync()) mma_commit(&acc_full[b]);
            __syncwarp();
        }
        if (elect_one_sync()) mma_commit(drain);
        __syncwarp();
    } else if (warp < 6) {
        // ------------------------------------------------ scales into tensor memory
        const uint32_t lane_base = ((uint32_t)(warp & 3) * 32u) << 16;
        uint32_t g = 0;
        bool alive = true;
        for (uint32_t t = blockIdx.x; t < total && alive; t += gridDim.x) {
            for (uint32_t kk = 0; kk < nk; ++kk, ++g) {
                const uint32_t st = g % S, ph = (g / S) & 1u;
                // full[] of this slot follows empty[] of its previous use: the MMAs
                // that read the slot's scale columns have completed
                if (!mbar_wait(&full[st], ph, abort, p.err, 0xD05)) { alive = false; break; }
                tc_fence_after();
                const uint32_t col = tmem + lane_base + kRing0 + st * (kSfaCols + kSfbCols);
                if constexpr (NV) {
                    uint32_t va[16], vb[4 * RB];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(sSa + st * kSfaBytes + (32 * i + lane) * kSfRow);
                        va[i] = v.x; va[4 + i] = v.y; va[8 + i] = v.z; va[12 + i] = v.w;
                    }
#pragma unroll
                    for (int i = 0; i < RB; ++i) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(sSb + st * kPSfbBytes + (32 * i + lane) * kSfRow);
                        vb[i] = v.x; vb[RB + i] = v.y; vb[2 * RB + i] = v.z; vb[3 * RB + i] = v.w;
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        uint32_t w[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) w[i] = va[8 * q + i];
                        tmem_st_x8(col + 8 * q, w);
                    }
#pragma unroll
                    for (int q = 0; q < RB / 2; ++q) {
                        uint32_t w[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) w[i] = vb[8 * q + i];
                        tmem_st_x8(col + kSfaCols + 8 * q, w);
                    }
                } else {
                    const uint32_t off = (kk & 1u) * 8u;
                    uint32_t va[8], vb[2 * RB];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        load_u2(sSa + st * kSfaBytes + (32 * i + lane) * kSfRow + off, va[i], va[4 + i]);
#pragma unroll
                    for (int i = 0; i < RB; ++i)
                        load_u2(sSb + st * kPSfbBytes + (32 * i + lane) * kSfRow + off, vb[i], vb[RB + i]);
                    tmem_st_x8(col, va);
                    tmem_st_x8(col + kSfaCols, vb);
                }
                st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sf_ready[st]);
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const uint32_t quarter = warp & 3;
        const uint32_t lane_base = (quarter * 32u) << 16;
        float alpha0 = 1.0f, alpha1 = 1.0f;   // scale of the first / second 64 columns
        if constexpr (NV) {
            alpha0 = *p.ts_a * *p.ts_b0;
            alpha1 = *p.ts_a * *p.ts_b1;
        }
        uint32_t j = 0;
        for (uint32_t t = blockIdx.x; t < total; t += gridDim.x, ++j) {
            const uint32_t b = j & 1u, use = j >> 1;
            if (!mbar_wait(&acc_full[b], use & 1u, abort, p.err, 0xD06)) break;
            tc_fence_after();
            PTile tl;
            ptile(p, t, tl);
            uint32_t v[kPBN];
            const uint32_t acc = tmem + lane_base + b * kPBN;
            tmem_ld_32x32b_x32(acc, *reinterpret_cast<uint32_t(*)[32]>(v));
            tmem_ld_32x32b_x32(acc + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
            tmem_ld_32x32b_x32(acc + 64, *reinterpret_cast<uint32_t(*)[32]>(v + 64));
            tmem_ld_32x32b_x32(acc + 96, *reinterpret_cast<uint32_t(*)[32]>(v + 96));
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);   // the MMAs may refill it now
            const uint32_t m = tl.m0 + quarter * 32 + lane;
            if constexpr (E == EPI_SWIGLU_MX || E == EPI_SWIGLU_F16) {
                const uint32_t c0 = tl.col * (kPBN / 2);
                float vmax = 0.0f;
#pragma unroll
                for (int cb = 0; cb < kPBN / 64; ++cb) {
                    float f[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float gf = __uint_as_float(v[cb * 32 + i]) * alpha0;
                        f[i] = __fdividef(gf, 1.0f + __expf(-gf)) * (__uint_as_float(v[kPBN / 2 + cb * 32 + i]) * alpha1);
                    }
                    const uint32_t c = c0 + cb * 32;
                    if constexpr (E == EPI_SWIGLU_MX) {
                        uint4 pk;
                        const uint32_t code = mx_quant32(f, pk);
                        if (m < tl.m_end && c < p.N) {
                            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(p.out) + (size_t)m * (p.ldc / 2) + c / 2) = pk;
                            p.out_scales[(size_t)m * (p.ldc / 32) + c / 32] = (uint8_t)code;
                        }
                    } else if (m < tl.m_end && c < p.N) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) vmax = fmaxf(vmax, fabsf(f[i]));
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + c);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t w[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const __half2 h = __floats2half2_rn(f[8 * i + 2 * q], f[8 * i + 2 * q + 1]);
                                w[q] = *reinterpret_cast<const uint32_t *>(&h);
                            }
                            dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
                }
                if constexpr (E == EPI_SWIGLU_F16) {
                    if (p.amax_out) {
                        float r = __half2float(__float2half_rn(vmax));
                        for (int o = 16; o; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
                        if (lane == 0) atomicMax(p.amax_out, __float_as_uint(r));
                    }
                }
            } else {
                const uint32_t n0 = tl.col * kPBN;
#pragma unroll
                for (int cc = 0; cc < kPBN / 32; ++cc) {
                    const float alpha = cc < kPBN / 64 ? alpha0 : alpha1;
                    const uint32_t col = n0 + cc * 32;
                    if (m < tl.m_end && col < p.N) {
                        if constexpr (E == EPI_F32) {
                            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                dst[i] = make_float4(__uint_as_float(v[cc * 32 + 4 * i]) * alpha,
                                                     __uint_as_float(v[cc * 32 + 4 * i + 1]) * alpha,
                                                     __uint_as_float(v[cc * 32 + 4 * i + 2]) * alpha,
                                                     __uint_as_float(v[cc * 32 + 4 * i + 3]) * alpha);
                        } else {
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint32_t w[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const __half2 h = __floats2half2_rn(__uint_as_float(v[cc * 32 + 8 * i + 2 * q]) * alpha,
                                                                        __uint_as_float(v[cc * 32 + 8 * i + 2 * q + 1]) * alpha);
                                    w[q] = *reinterpret_cast<const uint32_t *>(&h);
                                }
                                dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                            }
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
        mbar_wait(drain, 0, nullptr, p.err, 0xD07);   // every issued MMA has completed
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace mxf4
}  // namespace mpp41
