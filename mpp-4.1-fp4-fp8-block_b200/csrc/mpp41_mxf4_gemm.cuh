// Block-scaled FP4 GEMM on the FP4 tensor cores (W4A4):
// C[m][n] = sum_k A[m][k] * B[n][k], both operands MXFP4 (E2M1 packed two per
// byte, low nibble = even k, plus one E8M0 scale per 32 along k: the
// reference's weight layout, docs/MXFP4-MPP41-GUIDE.md:43-55, used for the
// activations too), fp32 accumulation, tcgen05.mma
// kind::mxf4.block_scale.block32. Nothing is decoded: TMA lands the packed
// tiles in 128-byte-swizzled shared memory and the MMA consumes them; only the
// E8M0 scales pass through registers on their way into tensor memory.
//
// Scale factors in tensor memory (block32, one SM; the arrangement of CUTLASS
// cute/atom/mma_traits_sm100.hpp tmem_sf_frg with four-fold lane replication):
// for operand row r = 32 i + j, the scales of k-blocks 4g..4g+3 of a stage are
// the 4 bytes of column (base + R/32 * g + i) at lane j of every lane quarter,
// R = 128 rows for A and BN for B. MMA number 2g + h of the stage (K = 64,
// two scales) reads bytes 2h and 2h+1: the byte offset rides in address bits
// 30-31 and in the instruction descriptor's scale-factor id.
//
// NVFP4 (NV = true): the same tiles with E2M1 elements, one UE4M3 scale per
// 16 along k and an fp32 tensor scale per operand, on
// kind::mxf4nvf4.block_scale.block16: an MMA (K = 64) takes four scales per
// row, one full 32-bit column, so stage k-group k of row 32 i + j sits in
// column base + R/32 * k + i with no byte offset. The two tensor scales
// multiply the accumulator in the epilogue.
//
// Epilogues: fp32 or fp16 C, SWIGLU_F16 (silu(g) * u as fp16, the columns
// arranged as below), or (SWIGLU_MX) the gate/up layer of a W4A4 MLP:
// B rows 0..BN/2-1 of the tile are gate rows, BN/2..BN-1 the up rows of the
// same BN/2 channels; each thread owns one token row, forms silu(g) * u and
// re-quantizes it to MXFP4 in registers (32-blocks never straddle threads), so
// the down GEMM reads the mid as its A operand directly.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2..5 move each stage's scales into tensor memory, then run the
// epilogue (warp w owns TMEM lane quarter w % 4).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_mx.cuh"

namespace mpp41 {
namespace mxf4 {

enum Epi { EPI_F32 = 0, EPI_F16 = 1, EPI_SWIGLU_MX = 2, EPI_SWIGLU_F16 = 3 };

constexpr int kBM = 128;          // rows of A per tile (MMA M)
constexpr int kBK = 256;          // K per stage: one 128-byte swizzle atom of packed E2M1
constexpr int kThreads = 192;
constexpr uint32_t kATile = kBM * 128;      // 16 KB
// Scales: a TMA box needs a 16-byte inner extent. MXFP4 has 8 scale bytes per
// row per stage, so each stage loads the 16-byte strip holding its own and the
// neighbour's; NVFP4 has exactly 16.
constexpr uint32_t kSfRow = 16;
constexpr uint32_t kSfaBytes = kBM * kSfRow;

// Column tile BN = MMA N (rows of B per tile). The library launches this
// one-tile-per-CTA kernel with BN = 256 (one CTA per SM, 4 stages, all 512
// tensor-memory columns) for M > 128; weight-streaming launches (grouped
// experts, M <= 128) use the persistent 128 x 128 kernel of
// mpp41_mxf4_persist.cuh instead. The BN = 128 configuration (two CTAs per
// SM, 3 stages, 256 columns each) compiles but is not launched: it measured
// no faster than BN = 256 on those shapes.
template <int BN> struct Tile {
    static constexpr int kStages = BN == 256 ? 4 : 3;
    static constexpr int kCtasPerSm = BN == 256 ? 1 : 2;
    static constexpr uint32_t kHalfRows = BN / 2;               // B rows per TMA box (two boxes per stage)
    static constexpr uint32_t kBHalf = kHalfRows * 128;
    static constexpr uint32_t kBTile = BN * 128;
    static constexpr uint32_t kSfbBytes = BN * kSfRow;
    static constexpr uint32_t kTmemCols = BN == 256 ? 512 : 256;
    static constexpr uint32_t kOffB = kStages * kATile;
    static constexpr uint32_t kOffSfa = kOffB + kStages * kBTile;
    static constexpr uint32_t kOffSfb = kOffSfa + kStages * kSfaBytes;
    static constexpr uint32_t kOffBar = kOffSfb + kStages * kSfbBytes;
    static constexpr uint32_t kSmem = 1024 + kOffBar + 256;
    static_assert((kSmem + 1024) * kCtasPerSm <= 228 * 1024, "shared memory");
};
// tensor-memory columns per stage: 2 (MXFP4) or 4 (NVFP4) per 32 operand rows;
// the accumulator takes the first BN columns, the scale ring follows
template <bool NV, int BN> struct SfCols {
    static constexpr uint32_t kA = kBM / 32 * (NV ? 4 : 2), kB = BN / 32 * (NV ? 4 : 2);
    static_assert(BN + Tile<BN>::kStages * (kA + kB) <= Tile<BN>::kTmemCols, "tensor memory");
};

// kind::mxf4 instruction descriptor: E2M1 x E2M1 (format 1), UE8M0 scales,
// K = 64, both operands K-major (cute/arch/mma_sm100_desc.hpp InstrDescriptorBlockScaled).
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N, uint32_t sfa_id, uint32_t sfb_id)
{
    return (sfb_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(M >> 4) << 24) | (sfa_id << 29);
}

// kind::mxf4nvf4 block16: E2M1 x E2M1, UE4M3 scales (bit 23 clear), K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(int M, int N)
{
    return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa, uint32_t sfb, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa, uint32_t sfb, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct Params {
    CUtensorMap tm_a;         // packed A [M][K/2], box {128, 128}, SW128
    CUtensorMap tm_b0;        // packed B rows of the tile's first half, box {128, 128}, SW128
    CUtensorMap tm_b1;        // ... second half (the up weights for SWIGLU_MX)
    CUtensorMap tm_sa;        // E8M0 A [M][K/32], box {16, 128}
    CUtensorMap tm_sb0;       // E8M0 B, box {16, 128}
    CUtensorMap tm_sb1;
    uint32_t b0_row0, b1_row0;   // row of tile 0's first / second half in tm_b0 / tm_b1
    uint32_t b_row_step;         // rows between consecutive column tiles in those maps
    void *out;                   // fp32 / fp16 [M][ldc]; SWIGLU_MX: packed mid [M][ldc/2]
    uint8_t *out_scales;         // SWIGLU_MX: mid scales [M][ldc/32]
    uint32_t M, N, K, ldc;       // N = columns written (SWIGLU_MX: mid channels)
    // NVFP4: fp32 tensor scales (device) of A and of the two B maps
    const float *ts_a, *ts_b0, *ts_b1;
    uint32_t *amax_out;          // SWIGLU_F16: atomicMax of |stored mid| as float bits (null: off)
    // Grouped (MoE) launch: row tile blockIdx.y is tiles[blockIdx.y] = {expert,
    // first row, end row, 0} while blockIdx.y < *n_tiles (other CTAs exit), and
    // B rows are offset by expert * b_expert_rows. Null tiles: plain GEMM.
    const uint4 *tiles;
    const uint32_t *n_tiles;
    uint32_t b_expert_rows;
    uint32_t col_tiles;          // persistent kernel: column tiles per row tile
    uint32_t *err;
};

__device__ __forceinline__ void load_u2(const uint8_t *p, uint32_t &lo, uint32_t &hi)
{
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    lo = v.x;
    hi = v.y;
}

template <int E, bool NV, int BN>
__global__ void __launch_bounds__(kThreads, Tile<BN>::kCtasPerSm) mxf4_gemm_kernel(const __grid_constant__ Params p)
{
    using Tl = Tile<BN>;
    constexpr int kStages = Tl::kStages;
    constexpr uint32_t kSfaCols = SfCols<NV, BN>::kA, kSfbCols = SfCols<NV, BN>::kB;
    constexpr uint32_t kSfCol0 = BN;   // scale ring after the accumulator
    constexpr int RB = BN / 32;        // B row groups of 32
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem, *sB = smem + Tl::kOffB, *sSa = smem + Tl::kOffSfa, *sSb = smem + Tl::kOffSfb;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Tl::kOffBar);
    uint64_t *full = bars;                 // [kStages] TMA landed
    uint64_t *sf_ready = bars + kStages;   // [kStages] scales in tensor memory
    uint64_t *empty = bars + 2 * kStages;  // [kStages] MMA done with the stage
    uint64_t *done = bars + 3 * kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * kStages + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t m0 = blockIdx.y * kBM, m_end = p.M, b_off = 0;
    if (p.tiles) {
        if (blockIdx.y >= *p.n_tiles) return;   // whole CTA, before any barrier or allocation
        const uint4 t = p.tiles[blockIdx.y];
        m0 = t.y;
        m_end = t.z;
        b_off = t.x * p.b_expert_rows;
    }
    const uint32_t nk = p.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&sf_ready[s], 4);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Tl::kTmemCols);
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
        const int32_t rb0 = (int32_t)(b_off + p.b0_row0 + blockIdx.x * p.b_row_step);
        const int32_t rb1 = (int32_t)(b_off + p.b1_row0 + blockIdx.x * p.b_row_step);
        uint32_t s = 0;
        for (; s < nk; ++s) {
            const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
            if (!warp_wait(&empty[st], ph ^ 1u, abort, p.err, 0xC01)) break;
            if (elect_one_sync()) {
                mbar_arrive_expect_tx(&full[st], kATile + Tl::kBTile + kSfaBytes + Tl::kSfbBytes);
                const int32_t kb = (int32_t)(s * (kBK / 2));
                const int32_t ks = (int32_t)((NV ? s : (s >> 1)) * kSfRow);
                tma_load_2d(sA + st * kATile, &p.tm_a, kb, (int32_t)m0, &full[st]);
                tma_load_2d(sB + st * Tl::kBTile, &p.tm_b0, kb, rb0, &full[st]);
                tma_load_2d(sB + st * Tl::kBTile + Tl::kBHalf, &p.tm_b1, kb, rb1, &full[st]);
                tma_load_2d(sSa + st * kSfaBytes, &p.tm_sa, ks, (int32_t)m0, &full[st]);
                tma_load_2d(sSb + st * Tl::kSfbBytes, &p.tm_sb0, ks, rb0, &full[st]);
                tma_load_2d(sSb + st * Tl::kSfbBytes + Tl::kHalfRows * kSfRow, &p.tm_sb1, ks, rb1, &full[st]);
            }
            __syncwarp();
        }
        // drain: no copy may still be landing when the CTA exits
        for (uint32_t t = (s > kStages ? s - kStages : 0); t < s; ++t)
            mbar_wait(&full[t % kStages], (t / kStages) & 1u, nullptr, p.err, 0xC02);
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        for (uint32_t s = 0; s < nk; ++s) {
            const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
            if (!warp_wait(&sf_ready[st], ph, abort, p.err, 0xC03)) break;
            tc_fence_after();
            if (elect_one_sync()) {
                const uint64_t ad = smem_desc_sw128(sA + st * kATile);
                const uint64_t bd = smem_desc_sw128(sB + st * Tl::kBTile);
                const uint32_t sfa0 = tmem + kSfCol0 + st * (kSfaCols + kSfbCols);
                const uint32_t sfb0 = sfa0 + kSfaCols;
#pragma unroll
                for (uint32_t k = 0; k < kBK / 64; ++k) {   // 32 packed bytes = 64 K per MMA
                    if constexpr (NV) {
                        mma_nvf4(tmem, ad + 2 * k, bd + 2 * k, idesc_nvf4(kBM, BN), sfa0 + (kBM / 32) * k,
                                 sfb0 + RB * k, (s | k) != 0u);
                    } else {
                        const uint32_t g = k >> 1, h = (k & 1u) * 2u;
                        const uint32_t sfa = (sfa0 + (kBM / 32) * g) | (h << 30);
                        const uint32_t sfb = (sfb0 + RB * g) | (h << 30);
                        mma_mxf4(tmem, ad + 2 * k, bd + 2 * k, idesc_mxf4(kBM, BN, h, h), sfa, sfb, (s | k) != 0u);
                    }
                }
                mma_commit(&empty[st]);
            }
            __syncwarp();
        }
        if (elect_one_sync()) mma_commit(done);
        __syncwarp();
    } else {
        // ------------------------------------------------ scales into tensor memory
        const uint32_t quarter = warp & 3;
        const uint32_t lane_base = (quarter * 32u) << 16;
        for (uint32_t s = 0; s < nk; ++s) {
            const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
            // full[] of stage s follows empty[] of stage s - kStages, so the MMAs
            // that read this slot's scale columns have completed
            if (!mbar_wait(&full[st], ph, abort, p.err, 0xC04)) break;
            tc_fence_after();
            const uint32_t col = tmem + lane_base + kSfCol0 + st * (kSfaCols + kSfbCols);
            // every lane quarter writes the same copy: lane j of any quarter holds rows 32 i + j
            if constexpr (NV) {
                uint32_t va[16], vb[4 * RB];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(sSa + st * kSfaBytes + (32 * i + lane) * kSfRow);
                    va[i] = v.x; va[4 + i] = v.y; va[8 + i] = v.z; va[12 + i] = v.w;
                }
#pragma unroll
                for (int i = 0; i < RB; ++i) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(sSb + st * Tl::kSfbBytes + (32 * i + lane) * kSfRow);
                    vb[i] = v.x; vb[RB + i] = v.y; vb[2 * RB + i] = v.z; vb[3 * RB + i] = v.w;
                }
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint32_t t[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) t[i] = va[8 * q + i];
                    tmem_st_x8(col + 8 * q, t);
                }
#pragma unroll
                for (int q = 0; q < RB / 2; ++q) {
                    uint32_t t[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) t[i] = vb[8 * q + i];
                    tmem_st_x8(col + kSfaCols + 8 * q, t);
                }
            } else {
                const uint32_t off = (s & 1u) * 8u;
                uint32_t va[8], vb[2 * RB];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    load_u2(sSa + st * kSfaBytes + (32 * i + lane) * kSfRow + off, va[i], va[4 + i]);
#pragma unroll
                for (int i = 0; i < RB; ++i)
                    load_u2(sSb + st * Tl::kSfbBytes + (32 * i + lane) * kSfRow + off, vb[i], vb[RB + i]);
                tmem_st_x8(col, va);
#pragma unroll
                for (int q = 0; q < RB / 4; ++q) {
                    uint32_t t[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) t[i] = vb[8 * q + i];
                    tmem_st_x8(col + kSfaCols + 8 * q, t);
                }
            }
            st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sf_ready[st]);
        }
        // ---------------------------------------------- epilogue
        mbar_wait(done, 0, abort, p.err, 0xC05);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool ok = (*abort == 0);
        tc_fence_after();
        const uint32_t m = m0 + quarter * 32 + lane;
        const uint32_t acc = tmem + lane_base;
        float alpha0 = 1.0f, alpha1 = 1.0f;   // scale of the tile's first / second BN/2 columns
        if constexpr (NV) {
            alpha0 = *p.ts_a * *p.ts_b0;
            alpha1 = *p.ts_a * *p.ts_b1;
        }
        if (ok) {
            if constexpr (E == EPI_SWIGLU_MX || E == EPI_SWIGLU_F16) {
                const uint32_t c0 = blockIdx.x * (BN / 2);   // mid channel of column 0
                float vmax = 0.0f;   // rounding to fp16 is monotonic: max of rounded = rounded max
#pragma unroll 1
                for (int cb = 0; cb < BN / 64; ++cb) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(acc + cb * 32, g);
                    tmem_ld_32x32b_x32(acc + BN / 2 + cb * 32, u);
                    tmem_ld_wait();
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float gf = __uint_as_float(g[i]) * alpha0;
                        v[i] = __fdividef(gf, 1.0f + __expf(-gf)) * (__uint_as_float(u[i]) * alpha1);
                    }
                    const uint32_t c = c0 + cb * 32;
                    if constexpr (E == EPI_SWIGLU_MX) {
                        uint4 pk;
                        const uint32_t code = mx_quant32(v, pk);
                        if (m < m_end && c < p.N) {
                            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(p.out) + (size_t)m * (p.ldc / 2) + c / 2) = pk;
                            p.out_scales[(size_t)m * (p.ldc / 32) + c / 32] = (uint8_t)code;
                        }
                    } else if (m < m_end && c < p.N) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) vmax = fmaxf(vmax, fabsf(v[i]));
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + c);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t w[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const __half2 h = __floats2half2_rn(v[8 * i + 2 * q], v[8 * i + 2 * q + 1]);
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
                const uint32_t n0 = blockIdx.x * BN;
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(acc + cc * 32, v);
                    tmem_ld_wait();
                    if constexpr (NV) {
                        const float alpha = cc < BN / 64 ? alpha0 : alpha1;
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                    }
                    const uint32_t col = n0 + cc * 32;
                    if (m < m_end && col < p.N) {
                        if constexpr (E == EPI_F32) {
                            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                     __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                        } else {
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)m * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint32_t w[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const __half2 h = __floats2half2_rn(__uint_as_float(v[8 * i + 2 * q]),
                                                                        __uint_as_float(v[8 * i + 2 * q + 1]));
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
        if (*abort) mbar_wait(done, 0, nullptr, p.err, 0xC06);   // let in-flight MMAs drain
        tc_fence_after();
        tmem_dealloc(tmem, Tl::kTmemCols);
    }
}

}  // namespace mxf4
}  // namespace mpp41
