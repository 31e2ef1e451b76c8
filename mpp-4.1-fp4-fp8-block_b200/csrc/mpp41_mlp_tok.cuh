// One MLP layer, down(swiglu(gate(x), up(x))), as ONE persistent kernel on
// the sm_100a tensor cores -- token-major tile shape (tokens on the MMA's M
// side, weights decoded into shared memory as the B operand). Used where the
// weight-major kernel (mpp41_mlp_fused.cuh) would leave most SMs idle in each
// phase: 128 tokens with a small layer.
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
// Warp roles (448 threads):
//   warps 0..3   TMA producers of activation tiles (x for G, mid for D), stages
//                dealt round-robin: one warp completes about one bulk copy per
//                memory round trip, so several warps keep several in flight
//   warp 4       TMEM owner, single-thread MMA issuer (2 accumulators x 64 cols)
//   warps 5..12  weight decode into the swizzled B ring (16 weights per thread
//                per stage, two warps per scheduler), then tile epilogues
//                (each warp: one TMEM lane quarter, one column half)
//   warp 13      TMA producer of packed weights in 16 KB chunks (256 bytes x 64
//                rows, i.e. 4-16 K stages per copy) and of the E8M0 scales
// Pipeline barriers count one arrival per warp (after __syncwarp), not per thread.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {
namespace tok {

constexpr int kAProd = 4;          // activation producer warps 0..3 (stages round-robin)
constexpr int kMmaWarp = 4;
constexpr int kDec0 = 5;           // decode + epilogue warps 5..12
constexpr int kDecWarps = 8;
constexpr int kEpi = kDecWarps * 32;
constexpr int kRawWarp = 13;       // weight / scale producer
constexpr int kFThreads = 14 * 32;
constexpr int kFBK = 128;          // K per pipeline stage: two 64-wide 128-byte swizzle atoms
constexpr int kMaxStagesA = 4;     // activation ring depth (power of two: index math is masks)
constexpr int kStagesB = 2;        // decoded-weight ring: one slot per decode group
constexpr int kFBN = 64;           // B rows per tile (G: 32 gate + 32 up)
constexpr int kChunkRow = 256;     // packed weight bytes per row per TMA request (largest box extent)
constexpr int kChunks = 3;         // packed weight chunk ring

struct FusedParams {
    CUtensorMap tm_x;       // x [T][H] fp16, box {64, 128}, SW128
    CUtensorMap tm_mid;     // mid [T][I] fp16, box {64, 128}, SW128
    CUtensorMap tm_wg, tm_wu;   // raw [I][H*bits/8], box {raw_row, 32}
    CUtensorMap tm_wd;          // raw [H][I*bits/8], box {raw_row, 64}
    CUtensorMap tm_sg, tm_su;   // E8M0 [I][H/32], box {kbc_g, 32}
    CUtensorMap tm_sd;          // E8M0 [H][I/32], box {kbc_d, 64}
    __half *mid;
    void *out;              // fp32 or fp16 [T][H]
    float *ws;              // fp32 split partials [splits][T][H]
    uint32_t *sync;         // [0] finished G tiles, [1] finished CTAs, [2..] D tile arrivals (self-resetting)
    uint32_t *err;
    uint32_t T, H, I;
    uint32_t splits;        // K splits of the down projection
    uint32_t kbc_g, kbc_d;  // scale bytes per row per tile
    uint32_t n_gtiles, n_dtiles;
    uint32_t d_spin;        // 1: each CTA holds at most one down tile, its last (splits may wait for each other)
    unsigned long long *trace;  // optional: kTraceSlots per CTA (profiling aid)
};

// Trace slots per CTA (ns from %globaltimer for events, SM cycles for sums).
enum TraceSlot : int {
    TR_START = 0, TR_PROLOGUE = 1, TR_END = 2, TR_G_EPI_END = 3, TR_WAIT_END = 4, TR_D_EPI_END = 5, TR_SMID = 6,
    TR_RAWP_WAIT_EMPTY = 8, TR_AP_WAIT_EMPTY = 9, TR_AP_WAIT_COUNTER = 10, TR_MMA_WAIT_A = 11, TR_MMA_WAIT_B = 12,
    TR_MMA_WAIT_ACC = 13, TR_DEC_WAIT_RAW = 14, TR_DEC_WAIT_SLOT = 15, TR_DEC_WORK = 16, TR_EPI_G = 17,
    TR_DEC_WAIT_ACC = 18, TR_EPI_D = 19, TR_CYCLES = 20, TR_MMA_ISSUE = 21, TR_DEC_FIRST_RAW = 22, TR_DEC_FIRST_SC = 23, TR_MMA_FIRST_A = 24, TR_D_FENCED = 25, TR_D_COUNTED = 26, TR_D_CONVERTED = 27, TR_D_LAST = 28,
    TR_G_ACC = 29, TR_G_STORED = 30, TR_G_PUBLISHED = 31, TR_D_ACC = 7, TR_D_STORED = 56, TR_D_ACC_WAITED = 57, TR_MMA_STAGE = 32, TR_DEC_STAGE = 64,
    TR_AP_STAGE = 96, kTraceSlots = 128
};

// mbar_wait that, while a trace is being recorded, adds the cycles it spent to `acc`.
__device__ __forceinline__ bool mbar_wait_t(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *err,
                                            uint32_t site, unsigned long long &acc, bool timed)
{
    if (!timed) return mbar_wait(bar, parity, abort, err, site);
    const long long c0 = clock64();
    const bool ok = mbar_wait(bar, parity, abort, err, site);
    acc += (unsigned long long)(clock64() - c0);
    return ok;
}

__device__ __forceinline__ long long clk_if(bool timed) { return timed ? clock64() : 0; }

template <int W>
struct FusedCfg {
    static constexpr int kRawRow = kFBK * wfmt_bits(W) / 8;      // packed bytes per row per stage
    static constexpr uint32_t kSPC = kChunkRow / kRawRow;         // stages per weight chunk
    static constexpr uint32_t kChunkBytes = kFBN * kChunkRow;     // 16 KB
    static constexpr uint32_t kAAtom = kBM * 128;                 // 128 rows x 64 K fp16
    static constexpr uint32_t kBAtom = kFBN * 128;                // 64 rows x 64 K fp16
    static constexpr uint32_t kABytes = 2 * kAAtom;
    static constexpr uint32_t kBBytes = 2 * kBAtom;
    // layout: [B ring][weight chunks][scales][activation ring (stages_a)]
    static constexpr uint32_t kOffRaw = kStagesB * kBBytes;
    static constexpr uint32_t kOffScales = kOffRaw + kChunks * kChunkBytes;
    __host__ __device__ static uint32_t scale_slot(uint32_t kbc_max) { return kFBN * kbc_max; }
    __host__ __device__ static uint32_t off_a(uint32_t kbc_max)
    {
        const uint32_t sc = (W == W_MXFP4) ? 2 * scale_slot(kbc_max) : 0;
        return (kOffScales + sc + 1023u) & ~1023u;
    }
    static uint32_t smem_bytes(uint32_t kbc_max, uint32_t stages_a)
    {
        return 1024 + off_a(kbc_max) + stages_a * kABytes + 512;
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

// Named barrier over the 256 epilogue threads that also ORs a predicate:
// every participant gets the same answer, so no thread can skip a later
// barrier the others wait on.
__device__ __forceinline__ bool epi_bar_any(bool pred)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, 256, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void red_add_v4(float *p, float a, float b, float c, float d)
{
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
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
        ti.nk = p.H / kFBK;
    } else {
        const uint32_t d = t - p.n_gtiles, nj = p.H / kFBN;
        ti.is_g = false;
        ti.c0 = (d % nj) * kFBN;
        ti.kb = (d / nj) % p.splits;
        ti.m0 = (d / (nj * p.splits)) * kBM;
        ti.nk = p.I / p.splits / kFBK;
    }
    return ti;
}

// Counter of finished G tiles feeding down split kb of token tile mt.
__device__ __forceinline__ uint32_t *slice_counter(const FusedParams &p, uint32_t mt, uint32_t kb)
{
    const uint32_t n_mt = (p.T + kBM - 1) / kBM;
    return p.sync + 2 + (p.H / kFBN) * n_mt + mt * p.splits + kb;
}

template <int W, int EG, bool OUT_F16>
__global__ void __launch_bounds__(kFThreads, 1) mlp_fused_kernel(const __grid_constant__ FusedParams p)
{
    using Cfg = FusedCfg<W>;
    constexpr uint32_t SPC = Cfg::kSPC;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t kbc_max = p.kbc_g > p.kbc_d ? p.kbc_g : p.kbc_d;
    constexpr uint32_t SA = kMaxStagesA;   // compile-time: the ring index math stays shifts and masks
    uint8_t *sB = smem;
    uint8_t *sRaw = smem + Cfg::kOffRaw;
    uint8_t *sSc = smem + Cfg::kOffScales;
    uint8_t *sA = smem + Cfg::off_a(kbc_max);
    const uint32_t sc_slot = (W == W_MXFP4) ? Cfg::scale_slot(kbc_max) : 0;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sA + SA * Cfg::kABytes);
    uint64_t *ck_full = bars;                       // [kChunks] packed weight chunk landed
    uint64_t *ck_empty = ck_full + kChunks;         // [kChunks] chunk decoded
    // Stage s uses activation slot s % SA and decoded-weight slot s % 2. One
    // barrier pair per stage: full[s % SA] completes when the activation copy
    // landed AND the 4 warps of the decode group owning stage s arrived; the
    // MMA commits empty[s % SA]. A decode group reuses weight slot s % 2 after
    // waiting for stage s-2 to be committed on empty[(s-2) % SA].
    uint64_t *a_full = ck_empty + kChunks;          // [SA]
    uint64_t *a_empty = a_full + kMaxStagesA;       // [SA]
    uint64_t *sc_full = a_empty + kMaxStagesA;      // [2]
    uint64_t *sc_empty = sc_full + 2;               // [2]
    uint64_t *acc_full = sc_empty + 2;              // [2]
    uint64_t *acc_empty = acc_full + 2;             // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile uint32_t *s_last = tmem_slot + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntiles = p.n_gtiles + p.n_dtiles;
    unsigned long long *tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceSlots : nullptr;
    const long long clk0 = p.trace ? clock64() : 0;
    unsigned long long tw0 = 0, tw1 = 0, tw2 = 0, tw3 = 0;   // per-role accumulators (trace only)
    if (tr && threadIdx.x == 0) {
        tr[TR_START] = globaltimer_ns();
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        tr[TR_SMID] = smid;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < kChunks; ++s) {
            mbar_init(&ck_full[s], 1);
            mbar_init(&ck_empty[s], kDecWarps);
        }
        for (uint32_t s = 0; s < SA; ++s) {
            mbar_init(&a_full[s], 1 + kDecWarps);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sc_full[s], 1);
            mbar_init(&sc_empty[s], kDecWarps);
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kDecWarps);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kRawWarp && lane == 0) {
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
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tr && threadIdx.x == 0) tr[TR_PROLOGUE] = globaltimer_ns();
    // The next layer's kernel may start on SMs this grid leaves free; it waits
    // (griddepcontrol.wait) before it touches anything this kernel writes.
    pdl_launch_dependents();

    if (warp == kRawWarp) {
        // ------------------------------------------------ packed weight / scale producer
        if (lane == 0) {
            uint32_t gc = 0, ti_n = 0;
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
                const uint32_t byte0 = ti.kb * ti.nk * Cfg::kRawRow;   // this tile's K range within the row
                const uint32_t nck = (ti.nk + SPC - 1) / SPC;
                for (uint32_t c = 0; c < nck; ++c, ++gc) {
                    const uint32_t st = gc % kChunks, ph = (gc / kChunks) & 1u;
                    if (!mbar_wait_t(&ck_empty[st], ph ^ 1u, abort, p.err, 0x602, tw0, tr != nullptr)) break;
                    mbar_arrive_expect_tx(&ck_full[st], Cfg::kChunkBytes);
                    uint8_t *dst = sRaw + st * Cfg::kChunkBytes;
                    const int32_t kx = (int32_t)(byte0 + c * kChunkRow);
                    if (ti.is_g) {
                        tma_load_2d(dst, &p.tm_wg, kx, (int32_t)ti.c0, &ck_full[st]);
                        tma_load_2d(dst + 32 * kChunkRow, &p.tm_wu, kx, (int32_t)ti.c0, &ck_full[st]);
                    } else {
                        tma_load_2d(dst, &p.tm_wd, kx, (int32_t)ti.c0, &ck_full[st]);
                    }
                }
            }
            // no copies left in flight when the CTA exits
            for (uint32_t t = (gc > kChunks ? gc - kChunks : 0); t < gc; ++t)
                mbar_wait(&ck_full[t % kChunks], (t / kChunks) & 1u, nullptr, p.err, 0x603);
        }
    } else if (warp < kAProd) {
        // ------------------------------------------------ activation producers
        if (lane == 0) {
            pdl_wait_prior();   // activations and counters may come from the previous kernel
            uint32_t gs = 0;
            uint32_t waited_t = ~0u;
            for (uint32_t t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
                const TileInfo ti = tile_info(p, t);
                const CUtensorMap *tm = ti.is_g ? &p.tm_x : &p.tm_mid;
                const uint32_t kstage0 = ti.kb * ti.nk;
                bool ok = true;
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    if (gs % kAProd != (uint32_t)warp) continue;
                    if (!ti.is_g && waited_t != t) {
                        // mid is written by other CTAs' G tiles (generic stores); wait
                        // for all of them, then order those writes before our TMA reads
                        const long long cw = clk_if(tr);
                        // only the G tiles that write this split's K range of mid
                        if (!wait_counter(slice_counter(p, ti.m0 / kBM, ti.kb), p.I / p.splits / 32, abort, p.err,
                                          0x701)) { ok = false; break; }
                        if (tr) tw1 += (unsigned long long)(clock64() - cw);
                        if (tr && warp == 0) tr[TR_WAIT_END] = globaltimer_ns();
                        fence_proxy_async_global();
                        waited_t = t;
                    }
                    const uint32_t st = gs % SA, ph = (gs / SA) & 1u;
                    if (!mbar_wait_t(&a_empty[st], ph ^ 1u, abort, p.err, 0x702, tw0, tr != nullptr)) { ok = false; break; }
                    if (tr && gs < 32) tr[TR_AP_STAGE + gs] = (unsigned long long)(clock64() - clk0);
                    mbar_arrive_expect_tx(&a_full[st], Cfg::kABytes);
                    const int32_t kx = (int32_t)((kstage0 + s) * kFBK);
                    tma_load_2d(sA + st * Cfg::kABytes, tm, kx, (int32_t)ti.m0, &a_full[st]);
                    tma_load_2d(sA + st * Cfg::kABytes + Cfg::kAAtom, tm, kx + kBK, (int32_t)ti.m0, &a_full[st]);
                }
                if (!ok) break;
            }
            for (uint32_t t = (gs > SA ? gs - SA : 0); t < gs; ++t)
                if (t % kAProd == (uint32_t)warp) mbar_wait(&a_full[t % SA], (t / SA) & 1u, nullptr, p.err, 0x703);
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, kFBN);
            uint32_t gs = 0, ti_n = 0;
            for (uint32_t t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++ti_n) {
                const TileInfo ti = tile_info(p, t);
                const uint32_t acc = ti_n & 1u;
                if (!mbar_wait_t(&acc_empty[acc], ((ti_n >> 1) & 1u) ^ 1u, abort, p.err, 0x801, tw2, tr != nullptr)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * kFBN;
                uint32_t ra = mbar_test(&a_full[gs % SA], (gs / SA) & 1u);
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    const uint32_t sa = gs % SA, pa = (gs / SA) & 1u;
                    const uint32_t sbb = gs % kStagesB;
                    if (!ra && !mbar_wait_t(&a_full[sa], pa, abort, p.err, 0x802, tw0, tr != nullptr)) break;
                    if (tr && gs == 0) tr[TR_MMA_FIRST_A] = (unsigned long long)(clock64() - clk0);
                    // probe the next stage now; the answer is needed only after this
                    // stage's MMAs are issued
                    const uint32_t gn = gs + 1;
                    ra = (s + 1 < ti.nk) ? mbar_test(&a_full[gn % SA], (gn / SA) & 1u) : 0u;
                    const long long cis = clk_if(tr);
                    tc_fence_after();
#pragma unroll
                    for (uint32_t j = 0; j < 2; ++j) {
                        const uint64_t ad = smem_desc_sw128(sA + sa * Cfg::kABytes + j * Cfg::kAAtom);
                        const uint64_t bd = smem_desc_sw128(sB + sbb * Cfg::kBBytes + j * Cfg::kBAtom);
#pragma unroll
                        for (uint32_t k = 0; k < kBK / 16; ++k)
                            mma_f16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (s | j | k) != 0u);
                    }
                    mma_commit(&a_empty[sa]);
                    if (tr) tw3 += (unsigned long long)(clock64() - cis);
                    if (tr && gs < 24) tr[TR_MMA_STAGE + gs] = (unsigned long long)(clock64() - clk0);
                }
                mma_commit(&acc_full[acc]);
            }
        }
    } else {
        // ------------------------------------------------ decode + epilogue
        const uint32_t te = threadIdx.x - kDec0 * 32;   // 0..255
        const uint32_t quarter = warp & 3;             // TMEM lanes 32*quarter..+31
        const uint32_t colh = (warp - kDec0) >> 2;     // column half of the tile
        const uint32_t row = quarter * 32 + lane;
        // decode: all 8 warps share every stage; 32 weights per thread
        const uint32_t dr = te >> 2, dq = te & 3u;   // B row, K quarter of the 128-wide stage
        uint32_t gs = 0, gc = 0, ti_n = 0;
        for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++ti_n) {
            const TileInfo ti = tile_info(p, t);
            const uint32_t slot = ti_n & 1u;
            const uint32_t kbc = ti.is_g ? p.kbc_g : p.kbc_d;
            const uint8_t *scl = sSc + slot * sc_slot;
            if constexpr (W == W_MXFP4) mbar_wait(&sc_full[slot], (ti_n >> 1) & 1u, abort, p.err, 0x901);
            if (tr && te == 0 && ti_n == 0) tr[TR_DEC_FIRST_SC] = (unsigned long long)(clock64() - clk0);
            uint32_t cst = 0;
            for (uint32_t s = 0; s < ti.nk && !*abort; ++s, ++gs) {
                const uint32_t sc = s % SPC;
                if (sc == 0) {
                    cst = gc % kChunks;
                    if (!mbar_wait_t(&ck_full[cst], (gc / kChunks) & 1u, abort, p.err, 0x902, tw0, tr != nullptr)) break;
                    if (tr && te == 0 && gc == 0) tr[TR_DEC_FIRST_RAW] = (unsigned long long)(clock64() - clk0);
                }
                {
                    const uint32_t st = gs % kStagesB;
                    if (gs >= kStagesB) {   // stage gs-2 (same weight slot) consumed by the MMA
                        const uint32_t g3 = gs - kStagesB;
                        if (!mbar_wait_t(&a_empty[g3 % SA], (g3 / SA) & 1u, abort, p.err, 0x903, tw1, tr != nullptr)) break;
                    }
                    const long long cdec = clk_if(tr);
                    const uint8_t *raw = sRaw + cst * Cfg::kChunkBytes + dr * kChunkRow + sc * Cfg::kRawRow;
                    // this thread: row dr, K quarter dq = half (dq & 1) of swizzle atom dq >> 1
                    uint8_t *rowp = sB + st * Cfg::kBBytes + (dq >> 1) * Cfg::kBAtom + dr * 128;
                    uint32_t sb = 127u;
                    // G: rows 0..31 gate scales, 32..63 up scales, each kbc_g wide
                    if constexpr (W == W_MXFP4) sb = scl[dr * kbc + 4 * s + dq];
                    uint32_t o[16];
                    decode_chunk<W>(raw + dq * (Cfg::kRawRow / 4), sb, o);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t phys = (((dq & 1u) * 4 + q) ^ (dr & 7u)) * 16u;
                        *reinterpret_cast<uint4 *>(rowp + phys) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[gs % SA]);
                    if (tr) tw2 += (unsigned long long)(clock64() - cdec);
                    if (tr && te == 0 && gs < 32) tr[TR_DEC_STAGE + gs] = (unsigned long long)(clock64() - clk0);
                }
                if ((sc == SPC - 1) || (s + 1 == ti.nk)) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ck_empty[cst]);
                    ++gc;
                }
            }
            if constexpr (W == W_MXFP4) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&sc_empty[slot]);
            }

            // ---------------------------------------------- tile epilogue
            if (ti_n == 0) pdl_wait_prior();   // before the first write of mid / partials / out
            const uint32_t acc = ti_n & 1u;
            mbar_wait_t(&acc_full[acc], (ti_n >> 1) & 1u, abort, p.err, 0x904, tw3, tr != nullptr);
            const long long cepi = clk_if(tr);
            if (epi_bar_any(*abort != 0)) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((quarter * 32u) << 16) + acc * kFBN;
            const uint32_t m = ti.m0 + row;
            if (ti.is_g) {
                uint32_t g[16], u[16];
                tmem_ld_32x32b_x16(taddr + colh * 16, g);
                tmem_ld_32x32b_x16(taddr + 32 + colh * 16, u);
                tmem_ld_wait();
                if (tr && te == 0) tr[TR_G_ACC] = (unsigned long long)(clock64() - clk0);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                if (m < p.T) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.mid + (size_t)m * p.I + ti.c0 + colh * 16);
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        uint32_t w4[4];
#pragma unroll
                        for (int j2 = 0; j2 < 4; ++j2) {
                            const int e = 8 * i + 2 * j2;
                            w4[j2] = half2_bits(swiglu<EG>(__uint_as_float(g[e]), __uint_as_float(u[e])),
                                                swiglu<EG>(__uint_as_float(g[e + 1]), __uint_as_float(u[e + 1])));
                        }
                        dst[i] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
                if (tr && te == 0) tr[TR_G_STORED] = (unsigned long long)(clock64() - clk0);
                // publish: our generic stores ordered before other CTAs' TMA (async
                // proxy) reads; one release by one thread after the CTA barrier
                fence_proxy_async_global();
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (te == 0) {
                    __threadfence();
                    atomicAdd(slice_counter(p, ti.m0 / kBM, ti.c0 / (p.I / p.splits)), 1u);
                }
                if (tr && te == 0) {
                    tr[TR_G_PUBLISHED] = (unsigned long long)(clock64() - clk0);
                    tr[TR_G_EPI_END] = globaltimer_ns();
                    tr[TR_EPI_G] += (unsigned long long)(clock64() - cepi);
                }
            } else {
                // Down tile: store this split's fp32 partial tile (plain stores, no
                // atomics), count the split, then sum the splits into out.
                // partial tiles are stored tile-native: per split and output tile,
                // 16 column blocks of [128 rows][4 columns], so a warp's float4
                // stores cover 512 contiguous bytes
                const uint32_t n_mt = (p.T + kBM - 1) / kBM, tile_d = (ti.m0 / kBM) * (p.H / kFBN) + ti.c0 / kFBN;
                const size_t tile4 = (size_t)kBM * kFBN / 4, split4 = (size_t)n_mt * (p.H / kFBN) * tile4;
                float4 *part4 = reinterpret_cast<float4 *>(p.ws) + ti.kb * split4 + tile_d * tile4;
                uint32_t v[32];
                tmem_ld_32x32b_x32(taddr + colh * 32, v);
                tmem_ld_wait();
                if (tr && te == 0) tr[TR_D_ACC] = (unsigned long long)(clock64() - clk0);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    __stcg(part4 + (colh * 8 + i) * kBM + row,
                           make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                       __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
                if (tr && te == 0) {
                    tr[TR_EPI_D] += (unsigned long long)(clock64() - cepi);
                    tr[TR_D_STORED] = (unsigned long long)(clock64() - clk0);
                    tr[TR_D_ACC_WAITED] = (unsigned long long)(cepi - clk0);
                }
                __threadfence();
                asm volatile("bar.sync 1, 256;" ::: "memory");
                if (tr && te == 0) tr[TR_D_FENCED] = (unsigned long long)(clock64() - clk0);
                uint32_t *cnt = p.sync + 2 + tile_d;
                if (te == 0) {
                    const bool last = atomicAdd(cnt, 1u) == p.splits - 1;
                    if (last) __threadfence();   // the other splits' partials are visible to us
                    *s_last = last ? 1u : 0u;
                }
                asm volatile("bar.sync 1, 256;" ::: "memory");
                uint32_t r0 = 0, r1 = 0;   // rows of the tile this CTA sums
                if (p.d_spin) {
                    // Every split of this tile is resident and this is each CTA's last
                    // tile, so waiting cannot deadlock; each split then sums a
                    // 1/splits band of rows in parallel.
                    bool ok = true;
                    if (te == 0 && !*s_last) ok = wait_counter(cnt, p.splits, abort, p.err, 0x905);
                    if (epi_bar_any(!ok)) break;
                    r0 = ti.kb * kBM / p.splits;
                    r1 = (ti.kb + 1) * kBM / p.splits;
                } else if (*s_last) {
                    r1 = kBM;
                }
                if (tr && te == 0) { tr[TR_D_COUNTED] = (unsigned long long)(clock64() - clk0); tr[TR_D_LAST] = *s_last; }
                const float4 *tile0 = reinterpret_cast<const float4 *>(p.ws) + tile_d * tile4;
                const uint32_t nr = r1 - r0;
                for (uint32_t i = te; i < nr * (kFBN / 4); i += kEpi) {
                    const uint32_t c4 = i / nr, rw = r0 + i % nr, mm = ti.m0 + rw;
                    if (mm >= p.T) continue;
                    float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (uint32_t j0 = 0; j0 < p.splits; j0 += 8) {
                        // all eight loads in flight before the first add
                        float4 q[8];
#pragma unroll
                        for (uint32_t j = 0; j < 8; ++j)
                            q[j] = (j0 + j < p.splits) ? __ldcg(tile0 + (j0 + j) * split4 + c4 * kBM + rw)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (uint32_t j = 0; j < 8; ++j) {
                            acc4.x += q[j].x; acc4.y += q[j].y; acc4.z += q[j].z; acc4.w += q[j].w;
                        }
                    }
                    if constexpr (OUT_F16) {
                        *reinterpret_cast<uint2 *>(static_cast<__half *>(p.out) + (size_t)mm * p.H + ti.c0 + c4 * 4) =
                            make_uint2(half2_bits(acc4.x, acc4.y), half2_bits(acc4.z, acc4.w));
                    } else {
                        *reinterpret_cast<float4 *>(static_cast<float *>(p.out) + (size_t)mm * p.H + ti.c0 + c4 * 4) = acc4;
                    }
                }
                if (tr && te == 0) tr[TR_D_CONVERTED] = (unsigned long long)(clock64() - clk0);
                // reset the tile counter for the next launch once no split reads it
                if (p.d_spin) {
                    if (te == 0 && atomicAdd(cnt, 1u) == 2 * p.splits - 1) atomicExch(cnt, 0u);
                } else if (*s_last && te == 0) {
                    atomicExch(cnt, 0u);
                }
            }
        }
    }

    // ---------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
    // Every tile of this CTA is finished (no thread reads the grid counters any
    // more): count the CTA; the last one resets the counters for the next
    // launch on this stream.
    if (tr) {
        if (warp == kRawWarp && lane == 0) tr[TR_RAWP_WAIT_EMPTY] = tw0;
        if (warp == 0 && lane == 0) { tr[TR_AP_WAIT_EMPTY] = tw0; tr[TR_AP_WAIT_COUNTER] = tw1; }
        if (warp == kMmaWarp && lane == 0) { tr[TR_MMA_WAIT_A] = tw0; tr[TR_MMA_WAIT_B] = tw1; tr[TR_MMA_WAIT_ACC] = tw2; tr[TR_MMA_ISSUE] = tw3; }
        if (threadIdx.x == kDec0 * 32) {
            tr[TR_DEC_WAIT_RAW] = tw0; tr[TR_DEC_WAIT_SLOT] = tw1; tr[TR_DEC_WORK] = tw2; tr[TR_DEC_WAIT_ACC] = tw3;
            tr[TR_D_EPI_END] = globaltimer_ns();
        }
        if (threadIdx.x == 0) { tr[TR_END] = globaltimer_ns(); tr[TR_CYCLES] = (unsigned long long)(clock64() - clk0); }
    }
    if (threadIdx.x == 0 && atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
        const uint32_t n_mt = (p.T + kBM - 1) / kBM;
        for (uint32_t i = 0; i < n_mt * p.splits; ++i) atomicExch(slice_counter(p, i / p.splits, i % p.splits), 0u);
        atomicExch(p.sync + 1, 0u);
    }
}

}  // namespace tok
}  // namespace mpp41
