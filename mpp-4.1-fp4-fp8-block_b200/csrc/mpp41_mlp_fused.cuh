// One MLP layer, down(swiglu(gate(x), up(x))), as ONE persistent kernel on
// the sm_100a tensor cores.
//
// The reference runs four dispatches per layer (gate GEMM, up GEMM, SwiGLU,
// down GEMM; encodeMXFP4FusedMLP main.swift:2033-2135, encodeMPPMLP
// 2636-2722). Here a cooperative grid of one CTA per SM walks two tile lists:
//
//   G tiles  128 tokens x 32 channels: gate and up rows of the same channels
//            decoded into one 64-row B operand, one kind::f16 MMA chain,
//            SwiGLU applied to the TMEM accumulators, fp16 mid stored (L2)
//   D tiles  128 tokens x 64 outputs x one K split of the down projection;
//            fp32 partials reduced with vector atomics (fp32 output) or in a
//            workspace whose last arriving CTA writes fp16 (fp16 output)
//
// Every CTA finishes its G tiles before its D tiles; a D tile's activation
// loads wait (bounded) on a grid-wide count of finished G tiles, but its
// weight and scale loads are issued ahead, so the down projection's weight
// stream overlaps the gate/up phase. Weights are decoded from the packed
// reference formats (MXFP4 E2M1 + E8M0, FP4, INT8/4/2, FP8) to fp16 in shared
// memory; no TMA multicast is used anywhere.
//
// Warp roles (224 threads):
//   warp 0      TMA producer of activation tiles (x for G, mid for D)
//   warp 1      TMEM owner, single-thread MMA issuer (2 accumulators x 64 cols)
//   warps 2..5  weight decode into the swizzled B ring, then tile epilogues
//   warp 6      TMA producer of packed weight tiles (16-deep ring) and scales
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {

constexpr int kFThreads = 224;
constexpr int kFStagesAB = 6;      // activation + decoded-weight ring
constexpr int kFBN = 64;           // B rows per tile (G: 32 gate + 32 up)

struct FusedParams {
    CUtensorMap tm_x;       // x [T][H] fp16, box {64, 128}, SW128
    CUtensorMap tm_mid;     // mid [T][I] fp16, box {64, 128}, SW128
    CUtensorMap tm_wg, tm_wu;   // raw [I][H*bits/8], box {raw_row, 32}
    CUtensorMap tm_wd;          // raw [H][I*bits/8], box {raw_row, 64}
    CUtensorMap tm_sg, tm_su;   // E8M0 [I][H/32], box {kbc_g, 32}
    CUtensorMap tm_sd;          // E8M0 [H][I/32], box {kbc_d, 64}
    __half *mid;
    void *out;              // fp32 or fp16 [T][H]
    float *ws;              // fp16 output: fp32 workspace [T][H]
    uint32_t *sync;         // [0] finished G tiles, [1] finished CTAs, [2..] D tile arrivals (self-resetting)
    uint32_t *err;
    uint32_t T, H, I;
    uint32_t splits;        // K splits of the down projection
    uint32_t kbc_g, kbc_d;  // scale bytes per row per tile
    uint32_t n_gtiles, n_dtiles;
    uint32_t raw_stages;
};

template <int W>
struct FusedCfg {
    static constexpr int kRawRow = kBK * wfmt_bits(W) / 8;
    static constexpr uint32_t kRawBytes = kFBN * kRawRow;
    static constexpr uint32_t kABytes = kBM * 128;
    static constexpr uint32_t kBBytes = kFBN * 128;
    static constexpr uint32_t kOffB = kFStagesAB * kABytes;
    static constexpr uint32_t kOffRaw = kOffB + kFStagesAB * kBBytes;
    __host__ __device__ static uint32_t off_scales(uint32_t raw_stages) { return kOffRaw + raw_stages * kRawBytes; }
    __host__ __device__ static uint32_t scale_slot(uint32_t kbc_max) { return kFBN * kbc_max; }
    static uint32_t smem_bytes(uint32_t raw_stages, uint32_t kbc_max)
    {
        const uint32_t sc = (W == W_MXFP4) ? 2 * scale_slot(kbc_max) : 0;
        return 1024 + off_scales(raw_stages) + sc + 512;
    }
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *p >= target (grid-wide counter). Returns false on timeout.
__device__ __forceinline__ bool wait_counter(const uint32_t *p, uint32_t target, volatile int *abort, uint32_t *err,
                                             uint32_t site)
{
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        __nanosleep(64);
        if (ld_acquire_gpu(p) >= target) return true;
        if (abort && *abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            report_error(err, kErrTimeout, site);
            if (abort) *abort = 1;
            return false;
        }
    }
}

// Named barrier over the 128 epilogue threads that also ORs a predicate:
// every participant gets the same answer, so no thread can skip a later
// barrier the others wait on.
__device__ __forceinline__ bool epi_bar_any(bool pred)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

struct TileInfo {
    bool is_g;
    uint32_t m0;      // first token
    uint32_t c0;      // G: first channel; D: first output column
    uint32_t kb;      // D: split index
    uint32_t nk;      // K stages
};

__device__ __forceinline__ TileInfo tile_info(const FusedParams &p, uint32_t t)
{
    TileInfo ti;
    const uint32_t gch = p.I / 32;
    if (t < p.n_gtiles) {
        ti.is_g = true;
        ti.c0 = (t % gch) * 32;
        ti.m0 = (t / gch) * kBM;
        ti.kb = 0;
        ti.nk = p.H / kBK;
    } else {
        const uint32_t d = t - p.n_gtiles, nj = p.H / kFBN;
        ti.is_g = false;
        ti.c0 = (d % nj) * kFBN;
        ti.kb = (d / nj) % p.splits;
        ti.m0 = (d / (nj * p.splits)) * kBM;
        ti.nk = p.I / p.splits / kBK;
    }
    return ti;
}

template <int W, int EG, bool OUT_F16>
__global__ void __launch_bounds__(kFThreads, 1) mlp_fused_kernel(const __grid_constant__ FusedParams p)
{
    using Cfg = FusedCfg<W>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t RS = p.raw_stages;
    const uint32_t kbc_max = p.kbc_g > p.kbc_d ? p.kbc_g : p.kbc_d;
    uint8_t *sA = smem;
    uint8_t *sB = smem + Cfg::kOffB;
    uint8_t *sRaw = smem + Cfg::kOffRaw;
    uint8_t *sSc = smem + Cfg::off_scales(RS);
    const uint32_t sc_slot = (W == W_MXFP4) ? Cfg::scale_slot(kbc_max) : 0;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sSc + 2 * sc_slot);
    uint64_t *raw_full = bars;                  // [RS]
    uint64_t *raw_empty = raw_full + 16;        // [RS]
    uint64_t *ab_full_a = raw_empty + 16;       // [6] activation tile landed
    uint64_t *ab_full_b = ab_full_a + kFStagesAB;  // [6] decoded weights ready
    uint64_t *ab_empty = ab_full_b + kFStagesAB;   // [6] MMA done with the stage
    uint64_t *sc_full = ab_empty + kFStagesAB;  // [2]
    uint64_t *sc_empty = sc_full + 2;           // [2]
    uint64_t *acc_full = sc_empty + 2;          // [2]
    uint64_t *acc_empty = acc_full + 2;         // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile uint32_t *s_last = tmem_slot + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntiles = p.n_gtiles + p.n_dtiles;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < RS; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 128);
        }
        for (int s = 0; s < kFStagesAB; ++s) {
            mbar_init(&ab_full_a[s], 1);
            mbar_init(&ab_full_b[s], 128);
            mbar_init(&ab_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sc_full[s], 1);
            mbar_init(&sc_empty[s], 128);
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], 128);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 6 && lane == 0) {
        tma_prefetch_desc(&p.tm_wg);
        tma_prefetch_desc(&p.tm_wu);
        tma_prefetch_desc(&p.tm_wd);
        if (W == W_MXFP4) {
            tma_prefetch_desc(&p.tm_sg);
            tma_prefetch_desc(&p.tm_su);
            tma_prefetch_desc(&p.tm_sd);
        }
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.tm_x);
        tma_prefetch_desc(&p.tm_mid);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 6) {
        // ------------------------------------------------ weight / scale producer
        if (lane == 0) {
            uint32_t gs = 0, ti_n = 0;
            for (uint32_t t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++ti_n) {
                const TileInfo ti = tile_info(p, t);
                if constexpr (W == W_MXFP4) {
                    const uint32_t slot = ti_n & 1u;
                    if (!mbar_wait(&sc_empty[slot], ((ti_n >> 1) & 1u) ^ 1u, abort, p.err, 0x601)) break;
                    uint8_t *dst = sSc + slot * sc_slot;
                    if (ti.is_g) {
                        mbar_arrive_expect_tx(&sc_full[slot], 64u * p.kbc_g);
                        tma_load_2d(dst, &p.tm_sg, 0, (int32_t)ti.c0, &sc_full[slot]);
                        tma_load_2d(dst + 32 * p.kbc_g, &p.tm_su, 0, (int32_t)ti.c0, &sc_full[slot]);
                    } else {
                        mbar_arrive_expect_tx(&sc_full[slot], 64u * p.kbc_d);
                        tma_load_2d(dst, &p.tm_sd, (int32_t)(ti.kb * p.kbc_d), (int32_t)ti.c0, &sc_full[slot]);
                    }
                }
                const uint32_t kstage0 = ti.kb * ti.nk;
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    const uint32_t st = gs % RS, ph = (gs / RS) & 1u;
                    if (!mbar_wait(&raw_empty[st], ph ^ 1u, abort, p.err, 0x602)) break;
                    mbar_arrive_expect_tx(&raw_full[st], Cfg::kRawBytes);
                    uint8_t *dst = sRaw + st * Cfg::kRawBytes;
                    const int32_t kx = (int32_t)((kstage0 + s) * Cfg::kRawRow);
                    if (ti.is_g) {
                        tma_load_2d(dst, &p.tm_wg, kx, (int32_t)ti.c0, &raw_full[st]);
                        tma_load_2d(dst + 32 * Cfg::kRawRow, &p.tm_wu, kx, (int32_t)ti.c0, &raw_full[st]);
                    } else {
                        tma_load_2d(dst, &p.tm_wd, kx, (int32_t)ti.c0, &raw_full[st]);
                    }
                }
            }
            // no loads left in flight when the CTA exits
            for (uint32_t t = (gs > RS ? gs - RS : 0); t < gs; ++t)
                mbar_wait(&raw_full[t % RS], (t / RS) & 1u, nullptr, p.err, 0x603);
        }
    } else if (warp == 0) {
        // ------------------------------------------------ activation producer
        if (lane == 0) {
            uint32_t gs = 0;
            bool waited = false;
            for (uint32_t t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
                const TileInfo ti = tile_info(p, t);
                if (!ti.is_g && !waited) {
                    // mid is written by other CTAs' G tiles (generic stores); wait for
                    // all of them, then order those writes before our TMA reads
                    if (!wait_counter(p.sync, p.n_gtiles, abort, p.err, 0x701)) break;
                    fence_proxy_async_global();
                    waited = true;
                }
                const CUtensorMap *tm = ti.is_g ? &p.tm_x : &p.tm_mid;
                const uint32_t kstage0 = ti.kb * ti.nk;
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    const uint32_t st = gs % kFStagesAB, ph = (gs / kFStagesAB) & 1u;
                    if (!mbar_wait(&ab_empty[st], ph ^ 1u, abort, p.err, 0x702)) break;
                    mbar_arrive_expect_tx(&ab_full_a[st], Cfg::kABytes);
                    tma_load_2d(sA + st * Cfg::kABytes, tm, (int32_t)((kstage0 + s) * kBK), (int32_t)ti.m0,
                                &ab_full_a[st]);
                }
            }
            for (uint32_t t = (gs > kFStagesAB ? gs - kFStagesAB : 0); t < gs; ++t)
                mbar_wait(&ab_full_a[t % kFStagesAB], (t / kFStagesAB) & 1u, nullptr, p.err, 0x703);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, kFBN);
            uint32_t gs = 0, ti_n = 0;
            for (uint32_t t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++ti_n) {
                const TileInfo ti = tile_info(p, t);
                const uint32_t acc = ti_n & 1u;
                if (!mbar_wait(&acc_empty[acc], ((ti_n >> 1) & 1u) ^ 1u, abort, p.err, 0x801)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * kFBN;
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    const uint32_t st = gs % kFStagesAB, ph = (gs / kFStagesAB) & 1u;
                    if (!mbar_wait(&ab_full_a[st], ph, abort, p.err, 0x802)) break;
                    if (!mbar_wait(&ab_full_b[st], ph, abort, p.err, 0x803)) break;
                    tc_fence_after();
                    const uint64_t ad = smem_desc_sw128(sA + st * Cfg::kABytes);
                    const uint64_t bd = smem_desc_sw128(sB + st * Cfg::kBBytes);
#pragma unroll
                    for (uint32_t k = 0; k < kBK / 16; ++k)
                        mma_f16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (s | k) != 0u);
                    mma_commit(&ab_empty[st]);
                }
                mma_commit(&acc_full[acc]);
            }
        }
    } else {
        // ------------------------------------------------ decode + epilogue
        const uint32_t t128 = threadIdx.x - 64;
        const uint32_t quarter = warp & 3;
        const uint32_t row = quarter * 32 + lane;
        uint32_t gs = 0, ti_n = 0;
        for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++ti_n) {
            const TileInfo ti = tile_info(p, t);
            const uint32_t slot = ti_n & 1u;
            const uint32_t kbc = ti.is_g ? p.kbc_g : p.kbc_d;
            const uint8_t *scl = sSc + slot * sc_slot;
            if constexpr (W == W_MXFP4) mbar_wait(&sc_full[slot], (ti_n >> 1) & 1u, abort, p.err, 0x901);
            for (uint32_t s = 0; s < ti.nk && !*abort; ++s, ++gs) {
                const uint32_t rst = gs % RS, rph = (gs / RS) & 1u;
                const uint32_t st = gs % kFStagesAB, ph = (gs / kFStagesAB) & 1u;
                if (!mbar_wait(&raw_full[rst], rph, abort, p.err, 0x902)) break;
                if (!mbar_wait(&ab_empty[st], ph ^ 1u, abort, p.err, 0x903)) break;
                const uint8_t *raw = sRaw + rst * Cfg::kRawBytes;
                uint8_t *bt = sB + st * Cfg::kBBytes;
                const uint32_t r = t128 >> 1, h = t128 & 1u;
                uint32_t sb = 127u;
                if constexpr (W == W_MXFP4) {
                    // G: rows 0..31 gate scales, 32..63 up scales, each kbc_g wide
                    sb = scl[r * kbc + 2 * s + h];
                }
                uint32_t o[16];
                decode_chunk<W>(raw + r * Cfg::kRawRow + h * (Cfg::kRawRow / 2), sb, o);
                uint8_t *rowp = bt + r * 128;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t phys = ((h * 4 + q) ^ (r & 7u)) * 16u;
                    *reinterpret_cast<uint4 *>(rowp + phys) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                }
                fence_proxy_async_smem();
                mbar_arrive(&raw_empty[rst]);
                mbar_arrive(&ab_full_b[st]);
            }
            if constexpr (W == W_MXFP4) mbar_arrive(&sc_empty[slot]);

            // ---------------------------------------------- tile epilogue
            const uint32_t acc = ti_n & 1u;
            mbar_wait(&acc_full[acc], (ti_n >> 1) & 1u, abort, p.err, 0x904);
            if (epi_bar_any(*abort != 0)) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((quarter * 32u) << 16) + acc * kFBN;
            const uint32_t m = ti.m0 + row;
            if (ti.is_g) {
                uint32_t g[32], u[32];
                tmem_ld_32x32b_x32(taddr, g);
                tmem_ld_32x32b_x32(taddr + 32, u);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&acc_empty[acc]);
                if (m < p.T) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.mid + (size_t)m * p.I + ti.c0);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t w4[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int e = 8 * i + 2 * j;
                            w4[j] = half2_bits(swiglu<EG>(__uint_as_float(g[e]), __uint_as_float(u[e])),
                                               swiglu<EG>(__uint_as_float(g[e + 1]), __uint_as_float(u[e + 1])));
                        }
                        dst[i] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
                // G tile t also clears its share of the down projection's
                // accumulation target (out for fp32, the workspace for fp16)
                {
                    float4 *z = reinterpret_cast<float4 *>(OUT_F16 ? p.ws : static_cast<float *>(p.out));
                    const uint32_t total = p.T * p.H / 4;
                    const uint32_t per = (total + p.n_gtiles - 1) / p.n_gtiles;
                    const uint32_t beg = t * per, end = min(beg + per, total);
                    for (uint32_t i = beg + t128; i < end; i += 128) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                // publish: stores -> visible to other CTAs' TMA (async proxy) reads
                fence_proxy_async_global();
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (t128 == 0) atomicAdd(p.sync, 1u);
            } else {
                (void)ld_acquire_gpu(p.sync);   // orders the clears above before our atomics
                float4 *dst = reinterpret_cast<float4 *>((OUT_F16 ? p.ws : static_cast<float *>(p.out)) +
                                                         (size_t)m * p.H + ti.c0);
#pragma unroll 1
                for (int cc = 0; cc < kFBN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(taddr + cc * 32, v);
                    tmem_ld_wait();
                    if (m < p.T) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            atomicAdd(dst + cc * 8 + i,
                                      make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                  __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[acc]);
                if constexpr (OUT_F16) {
                    __threadfence();
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    const uint32_t tile = (ti.m0 / kBM) * (p.H / kFBN) + ti.c0 / kFBN;
                    if (t128 == 0) {
                        const uint32_t prev = atomicAdd(p.sync + 2 + tile, 1u);
                        *s_last = (prev == p.splits - 1) ? 1u : 0u;
                        if (prev == p.splits - 1) atomicExch(p.sync + 2 + tile, 0u);   // reset for the next launch
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (*s_last) {
                        __threadfence();
                        for (uint32_t i = t128; i < kBM * (kFBN / 8); i += 128) {
                            const uint32_t rr = i / (kFBN / 8), c8 = (i % (kFBN / 8)) * 8;
                            const uint32_t mm = ti.m0 + rr;
                            if (mm < p.T) {
                                const float *src = p.ws + (size_t)mm * p.H + ti.c0 + c8;
                                const float4 a = __ldcg(reinterpret_cast<const float4 *>(src));
                                const float4 b = __ldcg(reinterpret_cast<const float4 *>(src) + 1);
                                *reinterpret_cast<uint4 *>(static_cast<__half *>(p.out) + (size_t)mm * p.H + ti.c0 + c8) =
                                    make_uint4(half2_bits(a.x, a.y), half2_bits(a.z, a.w), half2_bits(b.x, b.y),
                                               half2_bits(b.z, b.w));
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
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
    // Every tile of this CTA is finished (no thread reads the grid counters any
    // more): count the CTA; the last one resets the counters for the next
    // launch on this stream.
    if (threadIdx.x == 0 && atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
        atomicExch(p.sync + 0, 0u);
        atomicExch(p.sync + 1, 0u);
    }
}

}  // namespace mpp41
