// fp32-activation GEMM for the down projection of the fp32-mid rows:
// C[m][n] = sum_k A[m][k] * B[n][k], A fp32 [M][K] (the swiglu_float mid),
// B half or int8 [N][K] -> fp32 (mpp_mlp_f_h_f_n128 / mpp_mlp_f_i8_f_n128,
// MPPMLPKernels.metal:164-184).
//
// tcgen05.mma kind::tf32 reads 19 bits of each fp32 operand. Half and int8
// weights are exact in tf32. Each A value is split into a tf32 head (low 13
// bits cleared) and the exact fp32 remainder, and both halves are multiplied
// with B into the same fp32 accumulator: the product error is then about
// 2^-21 relative instead of tf32's 2^-11 ("3xTF32" without the lo*lo term,
// which B's exactness makes unnecessary).
//
// Warp roles (192 threads): warp 0 TMA producer (A fp32 tile, B packed tile),
// warp 1 TMEM owner + MMA issuer, warps 2..5 split A and widen B in shared
// memory, then run the epilogue.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace f32 {

constexpr int kBM = 128;          // tokens per tile (MMA M)
constexpr int kBN = 128;          // weight rows per tile (MMA N)
constexpr int kBK = 32;           // K per stage: one 128-byte swizzle atom of fp32
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr uint32_t kATile = kBM * kBK * 4;   // 16 KB
constexpr uint32_t kBTile = kBN * kBK * 4;   // 16 KB

__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N)
{
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

struct Params {
    CUtensorMap tm_a;         // fp32 [M][K], box {32, 128}, SW128
    CUtensorMap tm_b;         // half / int8 [N][K], box {32, 128}, no swizzle
    float *out;               // fp32 [M][ldc]
    uint32_t M, N, K, ldc;
    uint32_t k_per_split;
    uint32_t *err;
};

template <int W>
struct Cfg {
    static constexpr uint32_t kRawRow = kBK * (W == W_F16 ? 2 : 1);   // packed bytes per row per stage
    static constexpr uint32_t kRawTile = kBN * kRawRow;
    static constexpr uint32_t kOffLo = kStages * kATile;
    static constexpr uint32_t kOffB = kOffLo + kStages * kATile;
    static constexpr uint32_t kOffRaw = kOffB + kStages * kBTile;
    static constexpr uint32_t kOffBar = kOffRaw + kStages * kRawTile;
    static constexpr uint32_t kSmem = 1024 + kOffBar + 256;
};

template <int W, bool ATOMIC>
__global__ void __launch_bounds__(kThreads, 1) f32_gemm_kernel(const __grid_constant__ Params p)
{
    using C = Cfg<W>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;                // tf32 heads (written over the loaded A tile)
    uint8_t *sLo = smem + C::kOffLo;   // fp32 remainders
    uint8_t *sB = smem + C::kOffB;     // widened weights
    uint8_t *sRaw = smem + C::kOffRaw;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBar);
    uint64_t *full = bars;                 // [kStages] TMA landed
    uint64_t *ready = bars + kStages;      // [kStages] A split and B widened
    uint64_t *empty = bars + 2 * kStages;  // [kStages] MMA done with the stage
    uint64_t *done = bars + 3 * kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * kStages + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m0 = blockIdx.y * kBM, c0 = blockIdx.x * kBN;
    const uint32_t k0 = blockIdx.z * p.k_per_split;
    const uint32_t nk = p.k_per_split / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], 4);
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
            uint32_t s = 0;
            for (; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&empty[st], ph ^ 1u, abort, p.err, 0xB01)) break;
                mbar_arrive_expect_tx(&full[st], kATile + C::kRawTile);
                const int32_t kk = (int32_t)(k0 + s * kBK);
                tma_load_2d(sA + st * kATile, &p.tm_a, kk, (int32_t)m0, &full[st]);
                tma_load_2d(sRaw + st * C::kRawTile, &p.tm_b, kk, (int32_t)c0, &full[st]);
            }
            for (uint32_t t = (s > kStages ? s - kStages : 0); t < s; ++t)
                mbar_wait(&full[t % kStages], (t / kStages) & 1u, nullptr, p.err, 0xB02);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32_f32(kBM, kBN);
            for (uint32_t s = 0; s < nk; ++s) {
                const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
                if (!mbar_wait(&ready[st], ph, abort, p.err, 0xB03)) break;
                tc_fence_after();
                const uint64_t ah = smem_desc_sw128(sA + st * kATile);
                const uint64_t al = smem_desc_sw128(sLo + st * kATile);
                const uint64_t bd = smem_desc_sw128(sB + st * kBTile);
#pragma unroll
                for (uint32_t k = 0; k < kBK / 8; ++k) {
                    mma_tf32(tmem_d, ah + 2 * k, bd + 2 * k, idesc, (s | k) != 0u);
                    mma_tf32(tmem_d, al + 2 * k, bd + 2 * k, idesc, 1u);
                }
                mma_commit(&empty[st]);
            }
            mma_commit(done);
        }
    } else {
        // ------------------------------------------------ split A, widen B, then epilogue
        const uint32_t t = threadIdx.x - 64;   // 0..127: row t of the A tile and of the B tile
        for (uint32_t s = 0; s < nk; ++s) {
            const uint32_t st = s % kStages, ph = (s / kStages) & 1u;
            // full[] of stage s follows empty[] of stage s - kStages (the producer
            // waited for it), so the MMA is done with this slot's lo and B tiles
            if (!mbar_wait(&full[st], ph, abort, p.err, 0xB04)) break;
            uint4 *arow = reinterpret_cast<uint4 *>(sA + st * kATile + t * 128);
            uint4 *lrow = reinterpret_cast<uint4 *>(sLo + st * kATile + t * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) {   // same swizzled position in both tiles
                const uint4 v = arow[c];
                const uint4 h = make_uint4(v.x & 0xFFFFE000u, v.y & 0xFFFFE000u, v.z & 0xFFFFE000u, v.w & 0xFFFFE000u);
                arow[c] = h;
                lrow[c] = make_uint4(__float_as_uint(__uint_as_float(v.x) - __uint_as_float(h.x)),
                                     __float_as_uint(__uint_as_float(v.y) - __uint_as_float(h.y)),
                                     __float_as_uint(__uint_as_float(v.z) - __uint_as_float(h.z)),
                                     __float_as_uint(__uint_as_float(v.w) - __uint_as_float(h.w)));
            }
            const uint8_t *raw = sRaw + st * C::kRawTile + t * C::kRawRow;
            uint8_t *brow = sB + st * kBTile + t * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {   // 4 weights per 16-byte unit
                float f[4];
                if constexpr (W == W_F16) {
                    const uint2 hv = *reinterpret_cast<const uint2 *>(raw + 8 * c);
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&hv.y));
                    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
                } else {
                    const uint32_t w = *reinterpret_cast<const uint32_t *>(raw + 4 * c);
#pragma unroll
                    for (int j = 0; j < 4; ++j) f[j] = (float)(int8_t)(w >> (8 * j));
                }
                *reinterpret_cast<uint4 *>(brow + ((c ^ (t & 7u)) * 16u)) =
                    make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[st]);
        }
        // ---------------------------------------------- epilogue
        mbar_wait(done, 0, abort, p.err, 0xB06);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool ok = (*abort == 0);
        tc_fence_after();
        const uint32_t quarter = warp & 3;
        const uint32_t m = m0 + quarter * 32 + lane;
        const uint32_t taddr = tmem_d + ((quarter * 32u) << 16);
        if (ok) {
#pragma unroll 1
            for (int cc = 0; cc < kBN / 32; ++cc) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(taddr + cc * 32, v);
                tmem_ld_wait();
                const uint32_t col = c0 + cc * 32;
                if (m < p.M && col < p.N) {
                    float *dst = p.out + (size_t)m * p.ldc + col;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 q = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                     __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                        if constexpr (ATOMIC) atomicAdd(reinterpret_cast<float4 *>(dst) + i, q);
                        else reinterpret_cast<float4 *>(dst)[i] = q;
                    }
                }
            }
        }
    }

    // ---------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (*abort) mbar_wait(done, 0, nullptr, p.err, 0xB07);   // let in-flight MMAs drain
        tc_fence_after();
        tmem_dealloc(tmem_d, kBN);
    }
}

}  // namespace f32
}  // namespace mpp41
