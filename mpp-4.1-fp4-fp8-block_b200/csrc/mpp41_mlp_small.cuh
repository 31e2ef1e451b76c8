// One MLP layer, down(swiglu(gate(x), up(x))), as ONE kernel for small layers
// (at most 128 tokens, hidden <= 1024, 4-bit weights; BASELINE config 0 is
// T=128, H=1024, I=4096) on the sm_100a tensor cores.
//
// The reference runs four dispatches per layer (gate GEMM, up GEMM, SwiGLU,
// down GEMM; encodeMXFP4FusedMLP main.swift:2033-2135, encodeMPPMLP
// 2636-2722). Here every CTA of one co-resident grid runs one G tile and then
// one D tile:
//
//   G tile   64 channels x 64 tokens x all of H: gate and up rows of the
//            channels interleaved on the MMA's M side (TMEM lane 2j = gate j,
//            2j+1 = up j), decoded from the packed format straight into tensor
//            memory (the MMA's A operand); the 64-token x slice (128 KB at
//            H = 1024) is requested in full at kernel start. SwiGLU on the TMEM
//            accumulators, fp16 mid stored (it stays in L2), then a grid-wide
//            counter per (token half, K split of the down projection) is bumped.
//   D tile   128 outputs x 64 tokens x I/8 of K. The 8 K splits of an output
//            tile store their fp32 partials (coalesced, token-major) to a
//            workspace in L2, count themselves in, and each then sums a
//            1/8 band of the tile's rows over the 8 partials in split order.
//
// Why this shape (measured on B200, one CTA per SM):
//   - an SM ingests at most ~100-120 GB/s from L2 (TMA and plain loads share
//     it), so every CTA gets the same ingest: its 128 KB x slice, 64 KB of G
//     weights, a 64 KB mid slice and 32 KB of D weights;
//   - tcgen05.mma with M = 128 costs at least ~45 cycles per instruction below
//     N = 128, so 64-token tiles run at ~70 % of the tensor rate, which matches
//     the ingest rate;
//   - distributed shared memory moves only ~34 GB/s per SM and at most 15
//     8-CTA clusters are co-resident, so the K splits reduce through L2.
// The weights of both tiles are loaded and decoded while the previous layer
// finishes (programmatic dependent launch): only the x loads, the mid/out
// stores and the counters wait for it. No TMA multicast is used.
//
// Warp roles (608 threads):
//   warp 0       TMA producer of the activations (x slice, then mid split)
//   warp 1       TMA producer of packed weights (16 KB stages of 256 K x 128
//                rows, 4-slot shared-memory ring) and of all E8M0 scales
//   warp 2       TMEM owner (512 columns) and single-thread MMA issuer
//   warps 3..18  decode (lane quarter = warp % 4, K quarter = (warp-3)/4; 2
//                blocks of 32 weights of one row per stage) into a 3-slot TMEM
//                ring, then the two epilogues (token quarter = (warp-3)/4)
// Every wait is bounded; pipeline barriers count one arrival per warp.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {
namespace sl {

constexpr uint32_t kSplits = 8;      // K splits of the down projection
constexpr int kXWarp = 0, kWWarp = 1, kMmaWarp = 2, kDec0 = 3, kDecWarps = 16;
constexpr int kThreads = (kDec0 + kDecWarps) * 32;
constexpr int kEpi = kDecWarps * 32;
constexpr uint32_t kNT = 64;         // tokens per tile (MMA N)
constexpr uint32_t kRows = 128;      // weight rows per tile (MMA M)
constexpr uint32_t kGCh = 64;        // channels per G tile
constexpr uint32_t kXBytes = 128u << 10;   // activation region: the x slice (64 tokens x H <= 1024), later mid
constexpr uint32_t kWBytes = 64u << 10;    // packed-weight ring
constexpr uint32_t kMaxXSt = 8, kMaxMSt = 4, kMaxWSlots = 8, kMaxASlots = 6;   // barrier array sizes
constexpr uint32_t kAtom = kNT * 128;                    // 8 KB: 64 rows x 64 fp16 (one 128-byte swizzle atom)
constexpr uint32_t kScGRow = 32, kScDRow = 16;           // E8M0 bytes per row (H/32, I/8/32)
constexpr uint32_t kBand = kRows / kSplits;              // output rows each split sums (16)
// TMEM columns: G accumulator, D accumulator, then the operand ring
constexpr uint32_t kTmemCols = 512, kGAcc = 0, kDAcc = 64, kACol0 = 128;

// Per-format stage geometry. A stage covers the K whose packed bytes fill one
// 128-byte row (64 bytes for 2-bit weights): 256 K for 4-bit, 128 K for 8-bit
// and 256 K for 2-bit formats.
template <int W>
struct Fmt {
    static constexpr int kBits = wfmt_bits(W);
    static constexpr bool kMx = wfmt_mx(W);
    static constexpr uint32_t kRowB = kBits == 2 ? 64u : 128u;            // packed bytes per row per stage
    static constexpr uint32_t kSK = kRowB * 8u / (uint32_t)kBits;         // K per stage
    static constexpr bool kSw = kRowB == 128u;                            // 128-byte swizzled weight rows
    static constexpr uint32_t kWStage = kRows * kRowB;
    static constexpr uint32_t kWSlots = kWBytes / kWStage;
    static constexpr uint32_t kASlotCols = kSK / 2;                       // fp16 pairs per TMEM column
    static constexpr uint32_t kASlots =
        (kTmemCols - kACol0) / kASlotCols > kMaxASlots ? kMaxASlots : (kTmemCols - kACol0) / kASlotCols;
    static constexpr uint32_t kActStage = kNT * 2 * kSK;                  // x / mid bytes per stage
    static constexpr uint32_t kBlk = kSK / 128;                           // 32-weight blocks per decode thread
    static constexpr uint32_t kBlkB = 32u * (uint32_t)kBits / 8u;         // packed bytes per block
    static_assert(kWSlots <= kMaxWSlots && kASlots >= 2 && kBlk >= 1, "stage geometry");
};

// shared memory (offsets from a 1024-aligned base)
constexpr uint32_t kOffX = 0;
constexpr uint32_t kOffW = kOffX + kXBytes;
constexpr uint32_t kOffScG = kOffW + kWBytes;
constexpr uint32_t kOffScD = kOffScG + kRows * kScGRow;
constexpr uint32_t kOffMid = kOffScD + kRows * kScDRow;
constexpr uint32_t kOffBar = kOffMid + kNT * kGCh * 2;
constexpr uint32_t kSmem = 1024 + kOffBar + 256;
static_assert(kSmem <= 227u * 1024u, "shared memory");

struct Params {
    CUtensorMap tm_x;           // x [T][H] fp16 as [H/64][T][64], box {64, 64, kSK/64}, SW128
    CUtensorMap tm_mid;         // mid [T][I] fp16 as [I/64][T][64], box {64, 64, kSK/64}, SW128
    CUtensorMap tm_wg, tm_wu;   // packed [I][H*bits/8], box {kRowB, 64} (SW128 when kRowB = 128)
    CUtensorMap tm_wd;          // packed [H][I*bits/8], box {kRowB, 128}
    CUtensorMap tm_sg, tm_su;   // E8M0 [I][H/32], box {32, 64}
    CUtensorMap tm_sd;          // E8M0 [H][I/32], box {16, 128}
    __half *mid;
    const __half *rs_g, *rs_u, *rs_d;   // per-output-channel scales (row-scaled INT weights) or null
    void *out;                  // fp32 or fp16 [T][H]
    float *ws;                  // fp32 partials [n_h * H/128 tiles][8 splits][64 tokens][128 rows]
    uint32_t *sync;             // [0] finished CTAs, [1 + h*8 + s] finished G tiles,
                                // [1 + n_h*8 + tile] arrived D splits; self-resetting
    uint32_t *err;
    uint32_t T, H, I;
    uint32_t n_h;               // token halves (1 or 2)
    uint32_t n_g;               // G tiles ((I/64) x n_h); CTAs b < n_g run G tile b
    uint32_t n_d;               // D tiles ((H/128) x n_h x 8); CTAs b < n_d run D tile b
    uint32_t g_per_split;       // G tiles writing one K split of mid (per token half)
    unsigned long long *trace;  // optional: kTraceSlots per CTA (globaltimer ns)
};

enum TraceSlot : int {
    TR_START = 0, TR_W_LANDED = 1, TR_X_LANDED = 2, TR_G_DONE = 3, TR_G_PUB = 4, TR_CNT = 5, TR_D_DONE = 6,
    TR_RED = 7, TR_END = 8, TR_DEC_END = 9, TR_G_STORED = 10, TR_FENCED = 11, TR_D_STORED = 12, TR_D_ARRIVED = 13,
    TR_END_NS = 14,     // %globaltimer at the CTA's end
    TR_PDL_NS = 15,     // %globaltimer when griddepcontrol.wait returned (x producer)
    TR_PREV_END_NS = 63,// the previous launch's TR_END_NS of this CTA index
    TR_MMA_GO = 16,     // [8] stage i: operands ready, MMAs issued
    TR_DEC_GO = 24,     // [8] stage i: decoder passed its waits
    TR_DEC_DONE = 32,   // [8] stage i: decoded operand stored in TMEM
    TR_MMA_X = 40,      // [8] stage i: activation operand landed (seen by the MMA issuer)
    TR_MMA_ISSUED = 48, // [8] stage i: last MMA of the stage issued (slots 48..55)
    kTraceSlots = 64
};

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Release increment at GPU scope: the writes that happen before it (this
// thread's, and through the preceding CTA barrier the other threads') are
// visible to whoever acquires the new count.
__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier over the 512 decode/epilogue threads that also ORs a predicate, so
// every participant takes the same branch afterwards.
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

// Retiring a CTA: once its last counter wait has passed, one thread adds the
// CTA to the finished count (retire_begin, whose result is not needed until
// retire_end, so the round trip overlaps the CTA's remaining work); the last
// CTA of the grid then resets every counter for the next launch on the stream.
__device__ __forceinline__ uint32_t retire_begin(const Params &p) { return atomicAdd(p.sync, 1u); }

__device__ __forceinline__ void retire_end(const Params &p, uint32_t ticket, uint32_t n_m)
{
    if (ticket == gridDim.x - 1) {
        const uint32_t n = p.n_h * kSplits + p.n_h * n_m;
        for (uint32_t i = 0; i < n; ++i) atomicExch(p.sync + 1 + i, 0u);
        atomicExch(p.sync, 0u);
    }
}

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

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit TMEM columns; thread i reads lane (base+i).
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

template <int W, int EG, bool OUT_F16>
__global__ void __launch_bounds__(kThreads, 1) mlp_small_kernel(const __grid_constant__ Params p)
{
    using F = Fmt<W>;
    constexpr uint32_t kSK = F::kSK, kWSlots = F::kWSlots, kASlots = F::kASlots, kActStage = F::kActStage;
    constexpr uint32_t kWStage = F::kWStage, kASlotCols = F::kASlotCols, kRowB = F::kRowB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sX = smem + kOffX;
    uint8_t *sW = smem + kOffW;
    const uint8_t *sScG = smem + kOffScG;
    const uint8_t *sScD = smem + kOffScD;
    __half *sMid = reinterpret_cast<__half *>(smem + kOffMid);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *x_full = bars;                        // [kMaxXSt]
    uint64_t *m_full = x_full + kMaxXSt;            // [kMaxMSt]
    uint64_t *w_full = m_full + kMaxMSt;            // [kWSlots]
    uint64_t *w_empty = w_full + kMaxWSlots;        // [kWSlots] decode warps done with a slot
    uint64_t *a_full = w_empty + kMaxWSlots;        // [kASlots] decoded operand in TMEM
    uint64_t *a_empty = a_full + kMaxASlots;        // [kASlots] MMAs reading it completed
    uint64_t *sc_full = a_empty + kMaxASlots;
    uint64_t *g_done = sc_full + 1;                 // G accumulator complete (x no longer read)
    uint64_t *d_done = g_done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(d_done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_m = p.H / kRows;
    const uint32_t ds = blockIdx.x % kSplits;       // D tile: K split ds of output tile dt
    const uint32_t dt = blockIdx.x / kSplits;
    const uint32_t dm = dt % n_m, dh = dt / n_m;    // output rows dm*128.., token half dh
    const bool has_g = blockIdx.x < p.n_g;
    const uint32_t gch = p.I / kGCh;
    const uint32_t gw = blockIdx.x % gch, gh = blockIdx.x / gch;   // G tile: channels gw*64.., token half gh
    const uint32_t nG = has_g ? p.H / kSK : 0;      // G stages
    const bool has_d = blockIdx.x < p.n_d;
    const uint32_t KS = p.I / kSplits;              // K of one D split
    const uint32_t nD = has_d ? KS / kSK : 0;       // D stages
    uint32_t *g_cnt = p.sync + 1;                   // [n_h][8]
    uint32_t *d_cnt = p.sync + 1 + p.n_h * kSplits; // [n_h * n_m]
    unsigned long long *tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceSlots : nullptr;
    // trace: TR_START holds %globaltimer (ns), every other slot SM clock cycles
    // since the start (clock64 is cheap; a %globaltimer read is not)
    const long long clk0 = clock64();
    if (tr && threadIdx.x == 0) tr[TR_START] = globaltimer_ns();

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kMaxXSt; ++s) mbar_init(&x_full[s], 1);
        for (uint32_t s = 0; s < kMaxMSt; ++s) mbar_init(&m_full[s], 1);
        for (uint32_t s = 0; s < kWSlots; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], kDecWarps);
        }
        for (uint32_t s = 0; s < kASlots; ++s) {
            mbar_init(&a_full[s], kDecWarps);
            mbar_init(&a_empty[s], 1);
        }
        mbar_init(sc_full, 1);
        mbar_init(g_done, 1);
        mbar_init(d_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kWWarp && lane == 0) {
        tma_prefetch_desc(&p.tm_wg);
        tma_prefetch_desc(&p.tm_wu);
        tma_prefetch_desc(&p.tm_wd);
        if (F::kMx) {
            tma_prefetch_desc(&p.tm_sg);
            tma_prefetch_desc(&p.tm_su);
            tma_prefetch_desc(&p.tm_sd);
        }
    }
    if (warp == kXWarp && lane == 0) {
        tma_prefetch_desc(&p.tm_x);
        tma_prefetch_desc(&p.tm_mid);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    // The three role warps run converged; each copy and MMA is issued by one
    // elected lane, every wait is made by the whole warp.
    if (warp == kWWarp) {
        // ------------------------------------------------ packed weights and scales
        if (F::kMx && elect_one_sync()) {
            mbar_arrive_expect_tx(sc_full, (has_g ? kRows * kScGRow : 0u) + (has_d ? kRows * kScDRow : 0u));
            if (has_g) {
                tma_load_2d(smem + kOffScG, &p.tm_sg, 0, (int32_t)(gw * kGCh), sc_full);
                tma_load_2d(smem + kOffScG + kGCh * kScGRow, &p.tm_su, 0, (int32_t)(gw * kGCh), sc_full);
            }
            if (has_d)
                tma_load_2d(smem + kOffScD, &p.tm_sd, (int32_t)(ds * KS / 32), (int32_t)(dm * kRows), sc_full);
        }
        __syncwarp();
        const uint32_t n = nG + nD;
        bool ok = true;
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t sl = i % kWSlots;
            if (i >= kWSlots && !warp_wait(&w_empty[sl], ((i / kWSlots) - 1u) & 1u, abort, p.err, 0xC01)) {
                ok = false;
                break;
            }
            if (elect_one_sync()) {
                mbar_arrive_expect_tx(&w_full[sl], kWStage);
                uint8_t *dst = sW + sl * kWStage;
                if (i < nG) {
                    const int32_t kx = (int32_t)(i * kRowB);
                    tma_load_2d(dst, &p.tm_wg, kx, (int32_t)(gw * kGCh), &w_full[sl]);
                    tma_load_2d(dst + kGCh * kRowB, &p.tm_wu, kx, (int32_t)(gw * kGCh), &w_full[sl]);
                } else {
                    const int32_t kx = (int32_t)((ds * KS + (i - nG) * kSK) * F::kBits / 8);
                    tma_load_2d(dst, &p.tm_wd, kx, (int32_t)(dm * kRows), &w_full[sl]);
                }
            }
            __syncwarp();
        }
        // no copies in flight when the CTA exits
        if (ok)
            for (uint32_t i = (n > kWSlots ? n - kWSlots : 0); i < n; ++i)
                mbar_wait(&w_full[i % kWSlots], (i / kWSlots) & 1u, nullptr, p.err, 0xC02);
        if (F::kMx) mbar_wait(sc_full, 0, nullptr, p.err, 0xC03);
    } else if (warp == kXWarp) {
        // ------------------------------------------------ activations
        pdl_wait_prior();   // x and the counters come from / are reset by the previous kernel
        if (tr && lane == 0) {
            tr[TR_PREV_END_NS] = tr[TR_END_NS];
            tr[TR_PDL_NS] = globaltimer_ns();
        }
        if (elect_one_sync()) {
            for (uint32_t s = 0; s < nG; ++s) {
                mbar_arrive_expect_tx(&x_full[s], kActStage);
                tma_load_3d(sX + s * kActStage, &p.tm_x, 0, (int32_t)(gh * kNT), (int32_t)(s * kSK / 64), &x_full[s]);
            }
        }
        __syncwarp();
        bool ok = has_d;
        // mid goes where x was: wait until the G MMAs have read it
        if (ok && has_g) ok = warp_wait(g_done, 0, abort, p.err, 0xC11);
        if (ok) ok = __all_sync(0xffffffffu, wait_flag_ge(g_cnt + dh * kSplits + ds, p.g_per_split, kWaitLimitNs, abort, p.err, 0xC12));
        if (tr && lane == 0) tr[TR_CNT] = (unsigned long long)(clock64() - clk0);
        if (ok) {
            fence_proxy_async_global();   // the G tiles' generic mid stores before our TMA reads
            if (elect_one_sync()) {
                for (uint32_t s = 0; s < nD; ++s) {
                    mbar_arrive_expect_tx(&m_full[s], kActStage);
                    tma_load_3d(sX + s * kActStage, &p.tm_mid, 0, (int32_t)(dh * kNT),
                                (int32_t)((ds * KS + s * kSK) / 64), &m_full[s]);
                }
            }
            __syncwarp();
            for (uint32_t s = 0; s < nD; ++s) mbar_wait(&m_full[s], 0, nullptr, p.err, 0xC13);
        }
        for (uint32_t s = 0; s < nG; ++s) mbar_wait(&x_full[s], 0, nullptr, p.err, 0xC14);
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_f16_f32(kRows, kNT);
        bool ok = true;
        for (uint32_t i = 0; i < nG + nD; ++i) {
            const bool g = i < nG;
            const uint32_t s = g ? i : i - nG, sl = i % kASlots;
            if (!warp_wait(g ? &x_full[s] : &m_full[s], 0, abort, p.err, 0xC21)) { ok = false; break; }
            if (tr && lane == 0 && i < 8) tr[TR_MMA_X + i] = (unsigned long long)(clock64() - clk0);
            if (!warp_wait(&a_full[sl], (i / kASlots) & 1u, abort, p.err, 0xC22)) { ok = false; break; }
            if (tr && lane == 0 && i == 0) tr[TR_X_LANDED] = (unsigned long long)(clock64() - clk0);
            if (tr && lane == 0 && i < 8) tr[TR_MMA_GO + i] = (unsigned long long)(clock64() - clk0);
            tc_fence_after();
            if (elect_one_sync()) {
                const uint32_t d_tmem = tmem + (g ? kGAcc : kDAcc);
                const uint32_t a0 = tmem + kACol0 + sl * kASlotCols;
                const uint64_t b0 = smem_desc_sw128(sX + s * kActStage);
#pragma unroll
                for (uint32_t k = 0; k < kSK / 16; ++k)
                    mma_f16_ts(d_tmem, a0 + k * 8, b0 + (k / 4) * (kAtom >> 4) + 2 * (k % 4), idesc, (s | k) != 0u);
                mma_commit(&a_empty[sl]);
                if (g && i + 1 == nG) mma_commit(g_done);
            }
            __syncwarp();
            if (tr && lane == 0 && i < 8) tr[TR_MMA_ISSUED + i] = (unsigned long long)(clock64() - clk0);
        }
        if (ok && elect_one_sync()) mma_commit(d_done);
        __syncwarp();
    } else {
        // ------------------------------------------------ decode, then epilogues
        const uint32_t te = threadIdx.x - kDec0 * 32;   // 0..511
        const uint32_t q = warp & 3;                    // TMEM lanes 32q..32q+31
        const uint32_t kq = (warp - kDec0) >> 2;        // decode: K quarter of the stage; epilogue: token quarter
        const uint32_t r = q * 32 + lane;               // TMEM lane = weight row of the tile
        const uint32_t lane_base = (q * 32u) << 16;
        bool ok = true;
        if (F::kMx) ok = mbar_wait(sc_full, 0, abort, p.err, 0xC31);
        // ---------------------------------------------- G epilogue: SwiGLU -> fp16 mid
        // Runs once, inside the decode loop before the first D stage: the D
        // weights are decoded while other CTAs' G tiles finish (the D MMAs wait
        // for their mid anyway), so the mid of this tile is published first.
        bool g_epi_done = !has_g;
        auto g_epilogue = [&]() {
            g_epi_done = true;
            pdl_wait_prior();   // before the first write of mid
            const bool gok = ok && mbar_wait(g_done, 0, abort, p.err, 0xC41);
            if (!epi_bar_any(!gok || *abort)) {
                tc_fence_after();
                if (tr && te == 0) tr[TR_G_DONE] = (unsigned long long)(clock64() - clk0);
                uint32_t v[16];
                tmem_ld_x16(tmem + lane_base + kGAcc + kq * 16, v);
                tmem_ld_wait();
                if (p.rs_g) {   // per-output-channel scale of this lane's gate / up row
                    const float sc = __half2float(((r & 1u) ? p.rs_u : p.rs_g)[gw * kGCh + (r >> 1)]);
#pragma unroll
                    for (uint32_t t = 0; t < 16; ++t) v[t] = __float_as_uint(__uint_as_float(v[t]) * sc);
                }
                // lane pair (2j, 2j+1) = (gate, up) of channel j: the even lane
                // finishes tokens 0..7 of this warp's 16, the odd lane 8..15
                const uint32_t j = r >> 1, is_up = lane & 1u;
#pragma unroll
                for (uint32_t t = 0; t < 8; ++t) {
                    const uint32_t mine = is_up ? v[8 + t] : v[t];
                    const uint32_t send = is_up ? v[t] : v[8 + t];
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, send, 1);
                    const float gv = __uint_as_float(is_up ? other : mine);
                    const float uv = __uint_as_float(is_up ? mine : other);
                    sMid[(kq * 16 + is_up * 8 + t) * kGCh + j] = __float2half_rn(swiglu<EG>(gv, uv));
                }
                epi_bar_any(false);
                // 64 tokens x 128 bytes to mid[gh*64 + t][gw*64 ..)
                for (uint32_t idx = te; idx < kNT * (kGCh / 8); idx += kEpi) {
                    const uint32_t tl = idx / (kGCh / 8), c8 = idx % (kGCh / 8), tok = gh * kNT + tl;
                    if (tok < p.T)
                        *reinterpret_cast<uint4 *>(p.mid + (size_t)tok * p.I + gw * kGCh + c8 * 8) =
                            *reinterpret_cast<const uint4 *>(sMid + tl * kGCh + c8 * 8);
                }
                if (tr && te == 0) tr[TR_G_STORED] = (unsigned long long)(clock64() - clk0);
                // publish: generic stores ordered before other CTAs' TMA (async proxy)
                // reads, one release by one thread after the barrier
                fence_proxy_async_global();
                epi_bar_any(false);
                if (te == 0) {
                    red_release_add(g_cnt + gh * kSplits + gw / p.g_per_split, 1u);
                    if (tr) tr[TR_FENCED] = (unsigned long long)(clock64() - clk0);
                    if (tr) tr[TR_G_PUB] = (unsigned long long)(clock64() - clk0);
                }
            }
        };
        for (uint32_t i = 0; i < nG + nD && ok; ++i) {
            if (!g_epi_done && i == nG) g_epilogue();
            const bool g = i < nG;
            const uint32_t s = g ? i : i - nG, wsl = i % kWSlots, asl = i % kASlots;
            if (!mbar_wait(&w_full[wsl], (i / kWSlots) & 1u, abort, p.err, 0xC32)) { ok = false; break; }
            if (tr && i == 0 && te == 0) tr[TR_W_LANDED] = (unsigned long long)(clock64() - clk0);
            if (i >= kASlots) {   // MMAs of stage i-3 (same TMEM slot) completed
                if (!mbar_wait(&a_empty[asl], ((i / kASlots) - 1u) & 1u, abort, p.err, 0xC33)) { ok = false; break; }
                tc_fence_after();
            }
            if (tr && te == 0 && i < 8) tr[TR_DEC_GO + i] = (unsigned long long)(clock64() - clk0);
            // packed row of the slot: G rows interleave gate (even lanes) and up (odd lanes)
            const uint32_t rr = g ? ((r & 1u) ? kGCh + (r >> 1) : (r >> 1)) : r;
            const uint8_t *rowp = sW + wsl * kWStage + rr * kRowB;
            const uint8_t *scp = g ? sScG + rr * kScGRow + s * (kSK / 32) : sScD + rr * kScDRow + s * (kSK / 32);
            const uint32_t col = tmem + lane_base + kACol0 + asl * kASlotCols;
#pragma unroll
            for (uint32_t b = 0; b < F::kBlk; ++b) {
                const uint32_t blk = kq * F::kBlk + b;   // 32-weight block of the stage
                uint32_t wr[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
                if constexpr (F::kBits == 2) {
                    const uint2 v = *reinterpret_cast<const uint2 *>(rowp + blk * F::kBlkB);
                    wr[0] = v.x; wr[1] = v.y;
                } else {
#pragma unroll
                    for (uint32_t c = 0; c < F::kBlkB / 16; ++c) {
                        const uint32_t c16 = blk * (F::kBlkB / 16) + c;   // 16-byte chunk of the 128-byte row
                        const uint4 v = *reinterpret_cast<const uint4 *>(rowp + ((c16 ^ (rr & 7u)) << 4));
                        wr[4 * c] = v.x; wr[4 * c + 1] = v.y; wr[4 * c + 2] = v.z; wr[4 * c + 3] = v.w;
                    }
                }
                const uint32_t sb = F::kMx ? scp[blk] : 127u;
                uint32_t o[16];
                decode_words<W>(wr, sb, o);
                tmem_st_x16(col + blk * 16, o);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[asl]);
                mbar_arrive(&w_empty[wsl]);
            }
            if (tr && te == 0 && i < 8) tr[TR_DEC_DONE + i] = (unsigned long long)(clock64() - clk0);
        }
        if (tr && te == 0) tr[TR_DEC_END] = (unsigned long long)(clock64() - clk0);
        if (!g_epi_done) g_epilogue();
        pdl_wait_prior();   // before the first write of the workspace / out

        // ---------------------------------------------- D epilogue: split-K reduction through L2
        const bool dok = has_d && ok && mbar_wait(d_done, 0, abort, p.err, 0xC42);
        const bool dskip = epi_bar_any(!dok || *abort);
        uint32_t ticket = ~0u;                       // thread te == 0 only
        if (dskip && te == 0) ticket = retire_begin(p);   // no counter waits ahead
        if (!dskip) {
            tc_fence_after();
            if (tr && te == 0) tr[TR_D_DONE] = (unsigned long long)(clock64() - clk0);
            uint32_t v[16];
            tmem_ld_x16(tmem + lane_base + kDAcc + kq * 16, v);
            tmem_ld_wait();
            // partial tile, token-major: ws[dt][ds][token][row]; a warp stores
            // 128 contiguous bytes (32 rows) per token
            float *part = p.ws + ((size_t)dt * kSplits + ds) * (kNT * kRows);
#pragma unroll
            for (uint32_t t = 0; t < 16; ++t) __stcg(part + (kq * 16 + t) * kRows + r, __uint_as_float(v[t]));
            if (tr && te == 0) tr[TR_D_STORED] = (unsigned long long)(clock64() - clk0);
            epi_bar_any(false);
            bool aok = true;
            if (te == 0) {
                red_release_add(d_cnt + dt, 1u);
                if (tr) tr[TR_D_ARRIVED] = (unsigned long long)(clock64() - clk0);
                // all 8 splits of the tile are co-resident: waiting cannot deadlock
                aok = wait_flag_ge(d_cnt + dt, kSplits, kWaitLimitNs, abort, p.err, 0xC43);
                ticket = retire_begin(p);
            }
            if (!epi_bar_any(!aok)) {
                if (tr && te == 0) tr[TR_RED] = (unsigned long long)(clock64() - clk0);
                // this split sums rows ds*16 .. +16 of the tile over the 8 partials
                const uint32_t tok = te >> 3, r2 = ds * kBand + (te & 7u) * 2;
                const float *src = p.ws + (size_t)dt * kSplits * (kNT * kRows) + tok * kRows + r2;
                float2 a = make_float2(0.f, 0.f);
#pragma unroll
                for (uint32_t sp = 0; sp < kSplits; ++sp) {
                    const float2 b = __ldcg(reinterpret_cast<const float2 *>(src + sp * (kNT * kRows)));
                    a.x += b.x; a.y += b.y;
                }
                const uint32_t gtok = dh * kNT + tok, hcol = dm * kRows + r2;
                if (p.rs_d) {
                    a.x *= __half2float(p.rs_d[hcol]);
                    a.y *= __half2float(p.rs_d[hcol + 1]);
                }
                if (gtok < p.T) {
                    if constexpr (OUT_F16)
                        *reinterpret_cast<__half2 *>(static_cast<__half *>(p.out) + (size_t)gtok * p.H + hcol) =
                            __floats2half2_rn(a.x, a.y);
                    else
                        *reinterpret_cast<float2 *>(static_cast<float *>(p.out) + (size_t)gtok * p.H + hcol) = a;
                }
            }
        }
        if (te == 0) retire_end(p, ticket, n_m);
    }

    // ---------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (tr && threadIdx.x == 0) {
        tr[TR_END] = (unsigned long long)(clock64() - clk0);
        tr[TR_END_NS] = globaltimer_ns();
    }
}

}  // namespace sl
}  // namespace mpp41
