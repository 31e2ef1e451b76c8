// One MLP layer, down(swiglu(gate(x), up(x))), as ONE persistent kernel on
// the sm_100a tensor cores.
//
// The reference runs four dispatches per layer (gate GEMM, up GEMM, SwiGLU,
// down GEMM; encodeMXFP4FusedMLP main.swift:2033-2135, encodeMPPMLP
// 2636-2722). Here a cooperative grid of one CTA per SM walks two tile lists.
// The weights are the MMA's M side (128 rows per tile) and the tokens its N
// side (NT <= 128 per tile):
//
//   G tiles  64 channels x NT tokens: gate and up rows of the same channels
//            interleaved (row 2j = gate j, row 2j+1 = up j) so a lane pair holds
//            both operands of the SwiGLU; fp16 mid staged in shared memory and
//            stored row by row (L2)
//   D tiles  128 outputs x NT tokens x one K split of the down projection;
//            each split stores its fp32 partial tile, then the splits sum it
//            band by band (or the last arriving split sums all of it)
//
// Packed weights (MXFP4 E2M1 + E8M0, FP4, INT8/4/2, FP8) are decoded by eight
// warps straight into tensor memory, where tcgen05.mma reads its A operand
// (kind::f16, A from TMEM, B = activations in 128-byte-swizzled shared
// memory). Shared memory then only carries the activation stream and the
// packed bytes. D tiles decode their weights while the G tiles still run; only
// their activation (mid) loads wait, bounded, on a grid-wide count of finished
// G tiles. No TMA multicast is used anywhere.
//
// Warp roles (640 threads):
//   warps 0..1   TMA producers of activation stages (warp w: stages s, s % 2 == w)
//   warp 2       TMEM owner (512 columns), single-thread MMA issuer
//   warp 3       TMA producer of packed weight chunks (128 B x 128 rows) and
//                of E8M0 scale chunks (16 B x 128 rows)
//   warps 4..19  weight decode into the TMEM stage ring (lane quarter = warp%4,
//                K quarter = (warp-4)/4: 32 weights of one row per thread per
//                stage), then tile epilogues (lane quarter, token quarter)
// Pipeline barriers count one arrival per warp (after __syncwarp), not per thread.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {

constexpr int kAProd = 2;          // activation producer warps 0..1 (warp w: stages with gs % 2 == w)
constexpr int kMmaWarp = 2;
constexpr int kRawWarp = 3;        // weight / scale producer
constexpr int kDec0 = 4;           // decode + epilogue warps 4..19
constexpr int kDecWarps = 16;
constexpr int kEpi = kDecWarps * 32;
constexpr int kFThreads = 20 * 32;
constexpr int kWRows = 128;        // weight rows per tile (MMA M)
constexpr int kGCh = kWRows / 2;   // channels per G tile
constexpr int kFBK = 128;          // K per stage: two 64-wide swizzle atoms of fp16 activations
constexpr int kFStages = 4;         // stage ring depth (activation slot + TMEM weight slot), power of two
constexpr int kMaxNT = 128;        // tokens per tile (MMA N), at most
constexpr int kChunkRow = 128;     // packed bytes per row per weight chunk (one 128-byte swizzle row)
constexpr int kChunks = 3;         // weight chunk ring
constexpr uint32_t kChunkBytes = kWRows * kChunkRow;          // 16 KB
constexpr int kScRow = 16;         // MXFP4 scale bytes per row per scale chunk (512 K)
constexpr int kScChunks = 4;       // scale chunk ring
constexpr uint32_t kScBytes = kWRows * kScRow;                // 2 KB
constexpr uint32_t kStageBytes = kMaxNT * 2 * kFBK;           // activation slot (32 KB at NT = 128)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = kMaxNT;                         // fp32 columns per accumulator (2 of them)
constexpr uint32_t kACol0 = 2 * kAccCols;                     // weight stage slot i at kACol0 + 64 i
// shared memory layout (offsets from a 1024-aligned base)
constexpr uint32_t kOffRaw = kFStages * kStageBytes;
constexpr uint32_t kOffSc = kOffRaw + kChunks * kChunkBytes;
constexpr uint32_t kOffMid = kOffSc + kScChunks * kScBytes;
constexpr uint32_t kOffBar = kOffMid + kMaxNT * kGCh * 2;
constexpr uint32_t kFusedSmem = 1024 + kOffBar + 512;

struct FusedParams {
    CUtensorMap tm_x;           // x [T][H] fp16 as [H/64][T][64], box {64, NT, 2}, SW128
    CUtensorMap tm_mid;         // mid [T][I] fp16 as [I/64][T][64], box {64, NT, 2}, SW128
    CUtensorMap tm_wg, tm_wu;   // packed [I][H*bits/8], box {128, 64}, SW128
    CUtensorMap tm_wd;          // packed [H][I*bits/8], box {128, 128}, SW128
    CUtensorMap tm_sg, tm_su;   // E8M0 [I][H/32], box {16, 64}
    CUtensorMap tm_sd;          // E8M0 [H][I/32], box {16, 128}
    __half *mid;
    void *out;                  // fp32 or fp16 [T][H]
    float *ws;                  // splits > 1: fp32 split partials, per split and output tile NT/4 x [128][4]
    uint32_t *sync;             // [1] finished CTAs, [2..] D tile arrivals, then finished G tiles per
                                // (token tile, K split of the down projection); all self-resetting
    uint32_t *err;
    uint32_t T, H, I;
    uint32_t NT;                // tokens per tile, multiple of 16
    uint32_t splits;            // K splits of the down projection
    uint32_t n_gtiles, n_dtiles;
    uint32_t d_spin;            // 1: each CTA holds at most one down tile, its last (splits may wait for each other)
    uint32_t g_per_slice;       // G tiles that write one split's K range of mid (per token tile)
    unsigned long long *trace;  // optional: kTraceSlots per CTA (profiling aid)
};

// Trace slots per CTA (ns from %globaltimer for events, SM cycles otherwise).
enum TraceSlot : int {
    TR_START = 0, TR_PROLOGUE = 1, TR_END = 2, TR_G_EPI_END = 3, TR_WAIT_END = 4, TR_D_EPI_END = 5, TR_SMID = 6,
    TR_D_ACC = 7, TR_RAWP_WAIT_EMPTY = 8, TR_AP_WAIT_EMPTY = 9, TR_AP_WAIT_COUNTER = 10, TR_MMA_WAIT_A = 11, TR_G_COMPUTED = 12,
    TR_MMA_WAIT_ACC = 13, TR_DEC_WAIT_RAW = 14, TR_DEC_WAIT_SLOT = 15, TR_DEC_WORK = 16, TR_EPI_G = 17,
    TR_DEC_WAIT_ACC = 18, TR_EPI_D = 19, TR_CYCLES = 20, TR_MMA_ISSUE = 21, TR_DEC_FIRST_RAW = 22,
    TR_DEC_FIRST_SC = 23, TR_MMA_FIRST_A = 24, TR_D_FENCED = 25, TR_D_COUNTED = 26, TR_D_CONVERTED = 27,
    TR_D_LAST = 28, TR_G_ACC = 29, TR_G_STORED = 30, TR_G_PUBLISHED = 31, TR_MMA_STAGE = 32, TR_D_STORED = 56,
    TR_D_ACC_WAITED = 57, TR_DEC_WAIT_SC = 58, TR_DEC_STAGE = 64, TR_AP_STAGE = 96, TR_DEC_RAW_READY = 128,
    TR_DEC_START = 160, TR_MMA_WAIT_START = 192, TR_MMA_READY = 224, TR_WARP_DONE = 240,
    kTraceSlots = 256
};

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
        __nanosleep(32);
        if (ld_acquire_gpu(p) >= target) return true;
        if (abort && *abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            report_error(err, kErrTimeout, site);
            if (abort) *abort = 1;
            return false;
        }
    }
}

// Named barrier over the 512 epilogue threads that also ORs a predicate:
// every participant gets the same answer, so no thread can skip a later
// barrier the others wait on.
__device__ __forceinline__ bool epi_bar_any(bool pred)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, 512, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, A read from tensor memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 8 consecutive 32-bit TMEM columns; thread i reads lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t *r)
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr));
}

// 32 lanes x 4 consecutive 32-bit TMEM columns; thread i reads lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x4(uint32_t taddr, uint32_t *r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit TMEM columns; thread i writes lane (base+i).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit TMEM columns; thread i writes lane (base+i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- CTA pairs (tcgen05 cta_group::2): two CTAs of a 2-CTA cluster run one
// M = 256 MMA; each holds 128 weight rows in its tensor memory and half of the
// token tile in its shared memory, and the even CTA issues the MMAs. The
// barriers the MMA issuer waits on live in the even CTA; the odd CTA arrives on
// them through shared::cluster addresses.
__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *local, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cl(uint32_t caddr)
{
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cl(uint32_t caddr, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(caddr),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cl(uint32_t addr, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait with cluster-scope acquire (arrivals from the peer CTA), bounded the same way.
__device__ __forceinline__ bool mbar_wait_cl(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *err,
                                             uint32_t site)
{
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait_cl(addr, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cl(addr, parity)) return true;
        if ((it & 255u) == 0) {
            if (abort && *abort) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                report_error(err, kErrTimeout, site);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

// 3-D tiled load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const void *tmap, int32_t c0, int32_t c1, int32_t c2,
                                                 uint32_t bar_caddr)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(bar_caddr)
        : "memory");
}

__device__ __forceinline__ void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the mbarrier at `caddr` (either CTA of the pair) once all MMAs this
// thread issued before it complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t caddr)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(caddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

struct TileInfo {
    bool is_g;
    uint32_t m0;      // first token
    uint32_t c0;      // G: first channel; D: first output column
    uint32_t kb;      // D: split index
    uint32_t k0;      // first K element of the tile
    uint32_t nk;      // K stages
    uint32_t rot;     // the tile walks its K stages starting at stage rot (a multiple of 4)
    __device__ __forceinline__ uint32_t kstage(uint32_t s) const { return s + rot < nk ? s + rot : s + rot - nk; }
};

// Tile t of the list. With CTA pairs t indexes pair tiles (G: 128 channels,
// D: 256 outputs) and `half` (the CTA's rank in the pair) picks this CTA's
// 64 channels / 128 outputs; both CTAs of a pair walk the same K stages.
template <bool PAIR = false>
__device__ __forceinline__ TileInfo tile_info(const FusedParams &p, uint32_t t, uint32_t half = 0)
{
    TileInfo ti;
    constexpr uint32_t kGW = PAIR ? 2 * kGCh : kGCh, kDW = PAIR ? 2 * kWRows : kWRows;
    if (t < p.n_gtiles) {
        const uint32_t gch = p.I / kGW;
        ti.is_g = true;
        ti.c0 = (t % gch) * kGW + half * kGCh;
        ti.m0 = (t / gch) * p.NT;
        ti.kb = 0;
        ti.k0 = 0;
        ti.nk = p.H / kFBK;
    } else {
        const uint32_t d = t - p.n_gtiles, nh = p.H / kDW, ks = p.I / p.splits;
        ti.is_g = false;
        ti.c0 = (d % nh) * kDW + half * kWRows;
        ti.kb = (d / nh) % p.splits;
        ti.m0 = (d / (nh * p.splits)) * p.NT;
        ti.k0 = ti.kb * ks;
        ti.nk = ks / kFBK;
    }
    // Tiles that read the same activations start at different K stages, so
    // fewer CTAs request the same lines at once. Steps of 4 stages keep the
    // weight and scale chunks whole.
    ti.rot = (ti.nk % 4 == 0) ? (t % (ti.nk / 4)) * 4 : 0;
    return ti;
}

// Counter of finished G tiles feeding down split kb of token tile mt.
__device__ __forceinline__ uint32_t *slice_counter(const FusedParams &p, uint32_t mt, uint32_t kb)
{
    const uint32_t n_mt = (p.T + p.NT - 1) / p.NT;
    return p.sync + 2 + (p.H / kWRows) * n_mt + mt * p.splits + kb;
}

template <int W, int EG, bool OUT_F16, bool PAIR = false>
__global__ void __launch_bounds__(kFThreads, 1) mlp_fused_kernel(const __grid_constant__ FusedParams p)
{
    constexpr uint32_t RB = kFBK * wfmt_bits(W) / 8;   // packed bytes per row per stage
    constexpr uint32_t SPC = kChunkRow / RB;           // stages per weight chunk (1, 2 or 4)
    constexpr uint32_t SPS = 4;                        // stages per scale chunk (16 B = 512 K)
    constexpr uint32_t CB = chunk_bytes<W>();          // packed bytes per 32 weights
    static_assert(SPC >= 1 && SPC * RB == kChunkRow, "stage must divide the chunk");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sB = smem;
    uint8_t *sRaw = smem + kOffRaw;
    uint8_t *sSc = smem + kOffSc;
    __half *sMid = reinterpret_cast<__half *>(smem + kOffMid);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *ck_full = bars;                       // [kChunks] packed weight chunk landed
    uint64_t *ck_empty = ck_full + kChunks;         // [kChunks] chunk decoded
    uint64_t *sc_full = ck_empty + kChunks;         // [kScChunks] scale chunk landed
    uint64_t *sc_empty = sc_full + kScChunks;       // [kScChunks] scale chunk used
    // Stage s uses activation slot s % 4 and TMEM weight slot s % 4: full[s % 4]
    // completes when the activation copy landed AND all 8 decode warps stored
    // their weights; the MMA commits empty[s % 4], releasing both slots.
    uint64_t *st_full = sc_empty + kScChunks;       // [kFStages]
    uint64_t *st_empty = st_full + kFStages;         // [kFStages]
    uint64_t *acc_full = st_empty + kFStages;        // [2]
    uint64_t *acc_empty = acc_full + 2;             // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile uint32_t *s_last = tmem_slot + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntiles = p.n_gtiles + p.n_dtiles;
    const uint32_t NT = p.NT;
    // pairs: tile list walked per cluster; `half` is this CTA's rank in the pair
    const uint32_t half = PAIR ? cluster_rank() : 0u;
    const uint32_t t_first = PAIR ? blockIdx.x >> 1 : blockIdx.x, t_step = PAIR ? gridDim.x >> 1 : gridDim.x;
    const uint32_t NTc = PAIR ? NT / 2 : NT;   // tokens of the tile this CTA loads
    unsigned long long *tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceSlots : nullptr;
    const long long clk0 = p.trace ? clock64() : 0;
    unsigned long long tw0 = 0, tw1 = 0, tw2 = 0, tw3 = 0, tw4 = 0;   // per-role accumulators (trace only)
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
        for (int s = 0; s < kScChunks; ++s) {
            mbar_init(&sc_full[s], 1);
            mbar_init(&sc_empty[s], kDecWarps);
        }
        // pairs: the even CTA's st_full / acc_empty also count the odd CTA's arrivals
        constexpr uint32_t kSides = PAIR ? 2 : 1;
        for (int s = 0; s < kFStages; ++s) {
            mbar_init(&st_full[s], kSides * (1 + kDecWarps));
            mbar_init(&st_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kSides * kDecWarps);
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
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync_all();   // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tr && threadIdx.x == 0) tr[TR_PROLOGUE] = globaltimer_ns();
    // The next layer's kernel may start on SMs this grid leaves free: it loads
    // and decodes weights, and waits (griddepcontrol.wait) before it touches
    // anything this kernel writes. Weights and scales are never written here.
    pdl_launch_dependents();

    if (warp == kRawWarp) {
        // ------------------------------------------------ packed weight / scale producer
        // Copies are issued in stage order so both rings release in that order.
        if (lane == 0) {
            uint32_t gc = 0, gsc = 0;
            bool ok = true;
            for (uint32_t t = t_first; t < ntiles && ok && !*abort; t += t_step) {
                const TileInfo ti = tile_info<PAIR>(p, t, half);
                const int32_t row0 = (int32_t)ti.c0;
                for (uint32_t s = 0; s < ti.nk; ++s) {
                    if (W == W_MXFP4 && s % SPS == 0) {
                        const uint32_t sl = gsc % kScChunks;
                        if (!mbar_wait_t(&sc_empty[sl], ((gsc / kScChunks) & 1u) ^ 1u, abort, p.err, 0x601, tw0,
                                         tr != nullptr)) { ok = false; break; }
                        mbar_arrive_expect_tx(&sc_full[sl], kScBytes);
                        uint8_t *dst = sSc + sl * kScBytes;
                        const int32_t kx = (int32_t)((ti.k0 + ti.kstage(s) * kFBK) / 32);
                        if (ti.is_g) {
                            tma_load_2d(dst, &p.tm_sg, kx, row0, &sc_full[sl]);
                            tma_load_2d(dst + kGCh * kScRow, &p.tm_su, kx, row0, &sc_full[sl]);
                        } else {
                            tma_load_2d(dst, &p.tm_sd, kx, row0, &sc_full[sl]);
                        }
                        ++gsc;
                    }
                    if (s % SPC == 0) {
                        const uint32_t sl = gc % kChunks;
                        if (!mbar_wait_t(&ck_empty[sl], ((gc / kChunks) & 1u) ^ 1u, abort, p.err, 0x602, tw0,
                                         tr != nullptr)) { ok = false; break; }
                        mbar_arrive_expect_tx(&ck_full[sl], kChunkBytes);
                        uint8_t *dst = sRaw + sl * kChunkBytes;
                        const int32_t kx = (int32_t)(ti.k0 / kFBK * RB + ti.kstage(s) * RB);
                        if (ti.is_g) {
                            tma_load_2d(dst, &p.tm_wg, kx, row0, &ck_full[sl]);
                            tma_load_2d(dst + kGCh * kChunkRow, &p.tm_wu, kx, row0, &ck_full[sl]);
                        } else {
                            tma_load_2d(dst, &p.tm_wd, kx, row0, &ck_full[sl]);
                        }
                        ++gc;
                    }
                }
            }
            // no copies left in flight when the CTA exits
            for (uint32_t c = (gc > kChunks ? gc - kChunks : 0); c < gc; ++c)
                mbar_wait(&ck_full[c % kChunks], (c / kChunks) & 1u, nullptr, p.err, 0x603);
            for (uint32_t c = (gsc > kScChunks ? gsc - kScChunks : 0); c < gsc; ++c)
                mbar_wait(&sc_full[c % kScChunks], (c / kScChunks) & 1u, nullptr, p.err, 0x604);
        }
    } else if (warp < kAProd) {
        // ------------------------------------------------ activation producers
        // stage gs goes to warp gs % 2 and uses slot gs % 4
        if (lane == 0) {
            pdl_wait_prior();   // activations and counters may come from the previous kernel
            uint32_t gs = 0, last[2] = {0, 0}, waited_t = ~0u;
            bool ok = true, any[2] = {false, false};
            const uint32_t atom = NTc * 128;
            for (uint32_t t = t_first; t < ntiles && ok && !*abort; t += t_step) {
                const TileInfo ti = tile_info<PAIR>(p, t, half);
                const CUtensorMap *tm = ti.is_g ? &p.tm_x : &p.tm_mid;
                for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                    if ((gs & 1u) != (uint32_t)warp) continue;
                    if (!ti.is_g && waited_t != t) {
                        // mid is written by other CTAs' G tiles (generic stores); wait for
                        // the ones covering this split's K range, then order their writes
                        // before our TMA reads
                        const long long cw = clk_if(tr);
                        if (!wait_counter(slice_counter(p, ti.m0 / NT, ti.kb), p.g_per_slice, abort, p.err, 0x701)) {
                            ok = false;
                            break;
                        }
                        if (tr) tw1 += (unsigned long long)(clock64() - cw);
                        if (tr && warp == 0) tr[TR_WAIT_END] = globaltimer_ns();
                        fence_proxy_async_global();
                        waited_t = t;
                    }
                    const uint32_t sl = gs & (kFStages - 1), use = gs / kFStages;
                    if (!mbar_wait_t(&st_empty[sl], (use & 1u) ^ 1u, abort, p.err, 0x702, tw0, tr != nullptr)) {
                        ok = false;
                        break;
                    }
                    if (tr && gs < 32) tr[TR_AP_STAGE + gs] = (unsigned long long)(clock64() - clk0);
                    uint8_t *dst = sB + sl * kStageBytes;
                    const int32_t kx = (int32_t)(ti.k0 + ti.kstage(s) * kFBK);
                    if constexpr (PAIR) {
                        // this CTA's half of the token tile; completion counted in the even CTA
                        const uint32_t bar = cluster_addr(&st_full[sl], 0);
                        mbar_arrive_expect_tx_cl(bar, 2 * atom);
                        tma_load_3d_pair(dst, tm, 0, (int32_t)(ti.m0 + half * NTc), kx / 64, bar);
                    } else {
                        mbar_arrive_expect_tx(&st_full[sl], 2 * atom);
                        tma_load_3d(dst, tm, 0, (int32_t)ti.m0, kx / 64, &st_full[sl]);
                    }
                    last[sl >> 1] = gs;
                    any[sl >> 1] = true;
                }
            }
            // no copies left in flight when the CTA exits: the last use of each slot
            // (pairs: the MMAs that read it completed, which the issuer reports to both CTAs)
            for (int i = 0; i < 2; ++i)
                if (any[i]) {
                    if constexpr (PAIR)
                        mbar_wait(&st_empty[last[i] & (kFStages - 1)], (last[i] / kFStages) & 1u, nullptr, p.err, 0x703);
                    else
                        mbar_wait(&st_full[last[i] & (kFStages - 1)], (last[i] / kFStages) & 1u, nullptr, p.err, 0x703);
                }
        }
    } else if (warp == kMmaWarp) {
      if (!(PAIR && half != 0)) {   // pairs: the odd CTA's MMA warp only holds its TMEM allocation
        // ------------------------------------------------ MMA issuer
        // The whole warp runs the loop and makes every wait; one elected lane
        // issues (measured: ~70 vs 43 cycles per small-N MMA when one divergent
        // lane runs a loop with waits while its warp-mates wait elsewhere).
        // Pairs: the even CTA issues M = 256 MMAs over both CTAs' weight rows and
        // token halves, and reports completions to the barriers of both.
        const uint32_t idesc = idesc_f16_f32(PAIR ? 2 * kWRows : kWRows, (int)NT);
        const uint32_t atom = NTc * 128;
        auto wait_in = [&](uint64_t *bar, uint32_t parity, uint32_t site) -> bool {
            if constexpr (PAIR) return __all_sync(0xffffffffu, mbar_wait_cl(bar, parity, abort, p.err, site));
            else return warp_wait(bar, parity, abort, p.err, site);
        };
        auto commit = [&](uint64_t *bar) {
            if constexpr (PAIR) {
                mma_commit_pair(cluster_addr(bar, 0));
                mma_commit_pair(cluster_addr(bar, 1));
            } else {
                mma_commit(bar);
            }
        };
        uint32_t gs = 0, ti_n = 0;
        for (uint32_t t = t_first; t < ntiles && !__any_sync(0xffffffffu, *abort != 0); t += t_step, ++ti_n) {
            const TileInfo ti = tile_info<PAIR>(p, t, half);
            const uint32_t acc = ti_n & 1u;
            const long long cwa = clk_if(tr);
            if (!wait_in(&acc_empty[acc], ((ti_n >> 1) & 1u) ^ 1u, 0x801)) break;
            if (tr) tw2 += (unsigned long long)(clock64() - cwa);
            tc_fence_after();
            const uint32_t d_tmem = tmem + acc * kAccCols;
            bool ok = true;
            for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                const uint32_t sl = gs & (kFStages - 1);
                if (tr && lane == 0 && gs < 32) tr[TR_MMA_WAIT_START + gs] = (unsigned long long)(clock64() - clk0);
                const long long cws = clk_if(tr);
                if (!wait_in(&st_full[sl], (gs / kFStages) & 1u, 0x802)) {
                    ok = false;
                    break;
                }
                if (tr) tw0 += (unsigned long long)(clock64() - cws);
                if (tr && lane == 0 && gs == 0) tr[TR_MMA_FIRST_A] = (unsigned long long)(clock64() - clk0);
                if (tr && lane == 0 && gs < 16) tr[TR_MMA_READY + gs] = (unsigned long long)(clock64() - clk0);
                tc_fence_after();
                if (elect_one_sync()) {
                    const uint32_t a0 = tmem + kACol0 + sl * 64;
#pragma unroll
                    for (uint32_t j = 0; j < 2; ++j) {
                        const uint64_t bd = smem_desc_sw128(sB + sl * kStageBytes + j * atom);
#pragma unroll
                        for (uint32_t k = 0; k < 4; ++k) {
                            if constexpr (PAIR)
                                mma_f16_ts_pair(d_tmem, a0 + j * 32 + k * 8, bd + 2 * k, idesc, (s | j | k) != 0u);
                            else
                                mma_f16_ts(d_tmem, a0 + j * 32 + k * 8, bd + 2 * k, idesc, (s | j | k) != 0u);
                        }
                    }
                    commit(&st_empty[sl]);
                }
                __syncwarp();
                if (tr && lane == 0 && gs < 24) tr[TR_MMA_STAGE + gs] = (unsigned long long)(clock64() - clk0);
            }
            if (!ok) break;
            if (elect_one_sync()) commit(&acc_full[acc]);
            __syncwarp();
        }
      }
    } else {
        // ------------------------------------------------ decode + epilogue
        const uint32_t te = threadIdx.x - kDec0 * 32;   // 0..511
        const uint32_t quarter = warp & 3;             // TMEM lanes 32*quarter..+31
        const uint32_t kq = (warp - kDec0) >> 2;       // decode: K quarter of the stage; epilogue: token quarter
        const uint32_t r = quarter * 32 + lane;        // weight row of the tile = TMEM lane
        const uint32_t lane_base = (quarter * 32u) << 16;
        uint32_t gs = 0, gc = 0, gsc = 0, ti_n = 0;
        for (uint32_t t = t_first; t < ntiles; t += t_step, ++ti_n) {
            const TileInfo ti = tile_info<PAIR>(p, t, half);
            // packed row in the chunk: G rows interleave gate and up channels
            const uint32_t rr = ti.is_g ? ((r & 1u) ? kGCh + (r >> 1) : (r >> 1)) : r;
            bool ok = true;
            const uint32_t sw = rr & 7u;
            uint32_t cst = 0, scs = 0;
            for (uint32_t s = 0; s < ti.nk; ++s, ++gs) {
                const uint32_t sl = gs & (kFStages - 1);
                if (s % SPC == 0) {
                    cst = gc % kChunks;
                    if (!mbar_wait_t(&ck_full[cst], (gc / kChunks) & 1u, abort, p.err, 0x902, tw0, tr != nullptr)) {
                        ok = false;
                        break;
                    }
                    if (tr && te == 0 && gc == 0) tr[TR_DEC_FIRST_RAW] = (unsigned long long)(clock64() - clk0);
                    if (tr && te == 0 && gs < 32) tr[TR_DEC_RAW_READY + gs] = (unsigned long long)(clock64() - clk0);
                }
                if (W == W_MXFP4 && s % SPS == 0) {
                    scs = gsc % kScChunks;
                    if (!mbar_wait_t(&sc_full[scs], (gsc / kScChunks) & 1u, abort, p.err, 0x901, tw4, tr != nullptr)) {
                        ok = false;
                        break;
                    }
                }
                if (gs >= kFStages) {   // MMA of stage gs-4 (same TMEM slot) completed
                    if (!mbar_wait_t(&st_empty[sl], ((gs / kFStages) - 1u) & 1u, abort, p.err, 0x903, tw1,
                                     tr != nullptr)) { ok = false; break; }
                    tc_fence_after();
                }
                const long long cdec = clk_if(tr);
                if (tr && te == 0 && gs < 32) tr[TR_DEC_START + gs] = (unsigned long long)(cdec - clk0);
                const uint8_t *rowp = sRaw + cst * kChunkBytes + rr * kChunkRow;
                // this thread: 32 weights = RB/4 packed bytes of row rr
                const uint32_t off = (s % SPC) * RB + kq * CB;
                uint32_t w[8];
                if constexpr (CB == 8) {
                    const uint2 v = *reinterpret_cast<const uint2 *>(rowp + ((((off >> 4) ^ sw) << 4) | (off & 8u)));
                    w[0] = v.x; w[1] = v.y;
                } else {
#pragma unroll
                    for (int q = 0; q < (int)CB / 16; ++q) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(rowp + ((((off >> 4) + q) ^ sw) << 4));
                        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
                    }
                }
                uint32_t sb = 127u;
                if constexpr (W == W_MXFP4) sb = sSc[scs * kScBytes + rr * kScRow + (s % SPS) * 4 + kq];
                uint32_t words[16];
                decode_words<W>(w, sb, words);
                tmem_st_32x32b_x16(tmem + lane_base + kACol0 + sl * 64 + kq * 16, words);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR && half != 0) mbar_arrive_cl(cluster_addr(&st_full[sl], 0));
                    else mbar_arrive(&st_full[sl]);
                }
                if (tr) tw2 += (unsigned long long)(clock64() - cdec);
                if (tr && te == 0 && gs < 32) tr[TR_DEC_STAGE + gs] = (unsigned long long)(clock64() - clk0);
                if (tr && lane == 0 && gs == 2) tr[TR_WARP_DONE + (warp - kDec0)] = (unsigned long long)(clock64() - clk0);
                if (s % SPC == SPC - 1 || s + 1 == ti.nk) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ck_empty[cst]);
                    ++gc;
                }
                if (W == W_MXFP4 && (s % SPS == SPS - 1 || s + 1 == ti.nk)) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sc_empty[scs]);
                    ++gsc;
                }
            }


            // ---------------------------------------------- tile epilogue
            if (ti_n == 0) pdl_wait_prior();   // before the first write of mid / partials / out
            const uint32_t acc = ti_n & 1u;
            if (ok) mbar_wait_t(&acc_full[acc], (ti_n >> 1) & 1u, abort, p.err, 0x904, tw3, tr != nullptr);
            const long long cepi = clk_if(tr);
            if (epi_bar_any(*abort != 0)) break;
            tc_fence_after();
            const uint32_t ncol = NT / 4;                  // tokens of this thread: [kq*ncol, +ncol)
            const uint32_t taddr = tmem + lane_base + acc * kAccCols + kq * ncol;
            // accumulator columns in blocks of 32; the last block's loads release it
            const uint32_t j = r >> 1, is_up = lane & 1u;                // G: channel, gate/up
            const uint32_t h = ti.c0 + r, t0 = ti.m0 + kq * ncol;        // D: output column, first token
            // D: this split's partial tile, NT/4 blocks of [128 outputs][4 tokens]
            const uint32_t n_mt = (p.T + NT - 1) / NT, tile_d = (ti.m0 / NT) * (p.H / kWRows) + ti.c0 / kWRows;
            const size_t tile_floats = (size_t)NT * kWRows, split_floats = (size_t)n_mt * (p.H / kWRows) * tile_floats;
            float *part = p.ws + ti.kb * split_floats + tile_d * tile_floats;
            if (tr && te == 0) tr[ti.is_g ? TR_G_ACC : TR_D_ACC] = (unsigned long long)(clock64() - clk0);
            for (uint32_t cb = 0; cb < ncol; cb += 32) {
                uint32_t v[32];
#pragma unroll
                for (uint32_t c = 0; c < 32; c += 4)
                    if (cb + c < ncol) tmem_ld_32x32b_x4(taddr + cb + c, v + c);
                tmem_ld_wait();
                if (cb + 32 >= ncol) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (PAIR && half != 0) mbar_arrive_cl(cluster_addr(&acc_empty[acc], 0));
                        else mbar_arrive(&acc_empty[acc]);
                    }
                }
                if (ti.is_g) {
                    // lane pair (2j, 2j+1) = (gate, up) of channel j: the even lane
                    // finishes tokens 0..1 of each group of 4, the odd lane 2..3
#pragma unroll
                    for (uint32_t c = 0; c < 32; c += 4) {
                        if (cb + c < ncol) {
#pragma unroll
                            for (uint32_t i = 0; i < 2; ++i) {
                                // compile-time indices only: v stays in registers
                                const uint32_t mine = is_up ? v[c + 2 + i] : v[c + i];
                                const uint32_t send = is_up ? v[c + i] : v[c + 2 + i];   // what the partner needs
                                const uint32_t other = __shfl_xor_sync(0xffffffffu, send, 1);
                                const float g = __uint_as_float(is_up ? other : mine);
                                const float u = __uint_as_float(is_up ? mine : other);
                                sMid[(kq * ncol + cb + c + is_up * 2 + i) * kGCh + j] =
                                    __float2half_rn(swiglu<EG>(g, u));
                            }
                        }
                    }
                } else if (p.splits == 1) {
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i) {
                        if (cb + i < ncol && t0 + cb + i < p.T) {
                            const float f = __uint_as_float(v[i]);
                            if constexpr (OUT_F16)
                                static_cast<__half *>(p.out)[(size_t)(t0 + cb + i) * p.H + h] = __float2half_rn(f);
                            else
                                static_cast<float *>(p.out)[(size_t)(t0 + cb + i) * p.H + h] = f;
                        }
                    }
                } else {
                    // one float4 of 4 tokens per thread: a warp stores 512 contiguous bytes
#pragma unroll
                    for (uint32_t c = 0; c < 32; c += 4)
                        if (cb + c < ncol)
                            __stcg(reinterpret_cast<float4 *>(part) + ((kq * ncol + cb + c) / 4) * kWRows + r,
                                   make_float4(__uint_as_float(v[c]), __uint_as_float(v[c + 1]),
                                               __uint_as_float(v[c + 2]), __uint_as_float(v[c + 3])));
                }
            }
            if (ti.is_g) {
                if (tr && te == 0) tr[TR_G_COMPUTED] = (unsigned long long)(clock64() - clk0);
                epi_bar();
                // fp16 mid rows: NT x 128 bytes to mid[m0 + t][c0 .. c0 + 64)
                for (uint32_t i = te; i < NT * (kGCh / 8); i += kEpi) {
                    const uint32_t tt = i / (kGCh / 8), q = i % (kGCh / 8);
                    if (ti.m0 + tt < p.T)
                        *reinterpret_cast<uint4 *>(p.mid + (size_t)(ti.m0 + tt) * p.I + ti.c0 + q * 8) =
                            *reinterpret_cast<const uint4 *>(sMid + tt * kGCh + q * 8);
                }
                if (tr && te == 0) tr[TR_G_STORED] = (unsigned long long)(clock64() - clk0);
                // publish: our generic stores ordered before other CTAs' TMA (async
                // proxy) reads; one release by one thread after the CTA barrier
                fence_proxy_async_global();
                epi_bar();
                if (te == 0) {
                    __threadfence();
                    atomicAdd(slice_counter(p, ti.m0 / NT, ti.c0 / (p.I / p.splits)), 1u);
                }
                if (tr && te == 0) {
                    tr[TR_G_PUBLISHED] = (unsigned long long)(clock64() - clk0);
                    tr[TR_G_EPI_END] = globaltimer_ns();
                    tr[TR_EPI_G] += (unsigned long long)(clock64() - cepi);
                }
            } else {
                if (p.splits == 1) {
                    if (tr && te == 0) tr[TR_EPI_D] += (unsigned long long)(clock64() - cepi);
                    continue;
                }
                if (tr && te == 0) {
                    tr[TR_EPI_D] += (unsigned long long)(clock64() - cepi);
                    tr[TR_D_STORED] = (unsigned long long)(clock64() - clk0);
                    tr[TR_D_ACC_WAITED] = (unsigned long long)(cepi - clk0);
                }
                __threadfence();
                epi_bar();
                if (tr && te == 0) tr[TR_D_FENCED] = (unsigned long long)(clock64() - clk0);
                uint32_t *cnt = p.sync + 2 + tile_d;
                if (te == 0) {
                    const bool last = atomicAdd(cnt, 1u) == p.splits - 1;
                    if (last) __threadfence();   // the other splits' partials are visible to us
                    *s_last = last ? 1u : 0u;
                }
                epi_bar();
                const uint32_t nb = NT / 4;   // 4-token blocks of the tile
                uint32_t b0 = 0, b1 = 0;      // blocks this CTA sums
                if (p.d_spin) {
                    // every split of this tile is resident and this is each CTA's
                    // last tile, so waiting cannot deadlock; each split then sums a
                    // 1/splits band of token blocks
                    bool wok = true;
                    if (te == 0 && !*s_last) wok = wait_counter(cnt, p.splits, abort, p.err, 0x905);
                    if (epi_bar_any(!wok)) break;
                    b0 = ti.kb * nb / p.splits;
                    b1 = (ti.kb + 1) * nb / p.splits;
                } else if (*s_last) {
                    b1 = nb;
                }
                if (tr && te == 0) { tr[TR_D_COUNTED] = (unsigned long long)(clock64() - clk0); tr[TR_D_LAST] = *s_last; }
                const float4 *tile0 = reinterpret_cast<const float4 *>(p.ws + tile_d * tile_floats);
                for (uint32_t i = b0 * kWRows + te; i < b1 * kWRows; i += kEpi) {
                    const uint32_t blk = i / kWRows, hr = i % kWRows;
                    float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (uint32_t j0 = 0; j0 < p.splits; j0 += 8) {
                        // all eight loads in flight before the first add
                        float4 q[8];
#pragma unroll
                        for (uint32_t j = 0; j < 8; ++j)
                            q[j] = (j0 + j < p.splits) ? __ldcg(tile0 + (j0 + j) * (split_floats / 4) + i)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (uint32_t j = 0; j < 8; ++j) {
                            a4.x += q[j].x; a4.y += q[j].y; a4.z += q[j].z; a4.w += q[j].w;
                        }
                    }
                    const float f4[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                    for (uint32_t e = 0; e < 4; ++e) {
                        const uint32_t mm = ti.m0 + blk * 4 + e;
                        if (mm < p.T) {
                            if constexpr (OUT_F16)
                                static_cast<__half *>(p.out)[(size_t)mm * p.H + ti.c0 + hr] = __float2half_rn(f4[e]);
                            else
                                static_cast<float *>(p.out)[(size_t)mm * p.H + ti.c0 + hr] = f4[e];
                        }
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
    // pairs: neither CTA leaves while the other may still arrive on its barriers
    // or (the even CTA's MMAs) read its shared and tensor memory
    if constexpr (PAIR) cluster_sync_all();
    if (warp == kMmaWarp) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, kTmemCols);
        else tmem_dealloc(tmem, kTmemCols);
    }
    if (tr) {
        if (warp == kRawWarp && lane == 0) tr[TR_RAWP_WAIT_EMPTY] = tw0;
        if (warp == 0 && lane == 0) { tr[TR_AP_WAIT_EMPTY] = tw0; tr[TR_AP_WAIT_COUNTER] = tw1; }
        if (warp == kMmaWarp && lane == 0) { tr[TR_MMA_WAIT_A] = tw0; tr[TR_MMA_WAIT_ACC] = tw2; tr[TR_MMA_ISSUE] = tw3; }
        if (threadIdx.x == kDec0 * 32) {
            tr[TR_DEC_WAIT_RAW] = tw0; tr[TR_DEC_WAIT_SLOT] = tw1; tr[TR_DEC_WORK] = tw2; tr[TR_DEC_WAIT_ACC] = tw3;
            tr[TR_DEC_WAIT_SC] = tw4;
            tr[TR_D_EPI_END] = globaltimer_ns();
        }
        if (threadIdx.x == 0) { tr[TR_END] = globaltimer_ns(); tr[TR_CYCLES] = (unsigned long long)(clock64() - clk0); }
    }
    // Every tile of this CTA is finished (no thread reads the grid counters any
    // more): count the CTA; the last one resets the counters for the next
    // launch on this stream.
    if (threadIdx.x == 0 && atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
        const uint32_t n_mt = (p.T + NT - 1) / NT;
        for (uint32_t i = 0; i < n_mt * p.splits; ++i) atomicExch(slice_counter(p, i / p.splits, i % p.splits), 0u);
        atomicExch(p.sync + 1, 0u);
    }
}

}  // namespace mpp41
