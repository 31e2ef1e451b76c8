// Decode-sized MLP layer (T <= 16 tokens, 4-bit weights: MXFP4, unscaled FP4,
// INT4) as ONE persistent weight-streaming kernel, one CTA per SM.
//
// With a handful of tokens the layer is a stream of packed weights (93.6 MB for
// the Llama-3-8B layer) and HBM only reaches its copy bandwidth with about
// 128 KB in flight per SM. So each CTA runs a deep shared-memory ring:
//   weight warp      streams the packed weights (TMA, 128-byte swizzle) and their
//                    E8M0 scales (cp.async, arriving on the same mbarrier) of every
//                    unit the CTA owns, gate/up units first and down units after
//                    them, without ever waiting for activations;
//   activation warp  streams the activations of each unit (TMA): x for gate/up
//                    units, and for down units the mid chunk it reads, once every
//                    gate/up group of that chunk is published grid-wide;
//   sync warp        publishes this CTA's finished gate/up groups (per 1024-channel
//                    mid chunk) and its down partial, and prefetches the partials
//                    the CTA must add; its gpu-scope fences stay off the math warps;
//   math warps       decode the weights straight into mma.sync A fragments
//                    (cvt.rn.f16x2.e2m1x2 for E2M1; (n ^ 8) - 8 INT4 exactly through
//                    fp16 arithmetic), multiply the activations (the N = 8 side, up
//                    to two token tiles) and keep fp32 sums.
// A unit is 16 KB of weights: 32 rows x 1024 K (gate/up: 16 gate + the same 16
// up channels; down: 32 output rows).
//
// Schedule. Gate/up groups (16 channels, all of K) are dealt round-robin: CTA b
// takes groups b, b + grid, b + 2*grid, ... whole, so the grid completes the mid
// chunk by chunk in order and the first down units find their chunk ready while
// other CTAs still run gate/up work. Down units (32 rows x 1024 K) are dealt in
// contiguous group-major ranges whose starts the host computes so that every CTA
// streams the same number of bytes over both phases. Within its range a CTA runs
// its last group first (low K chunks: the mid chunks published first) and its
// first group last. A down group whose units span several CTAs is finished by
// the CTA holding its last units, which adds the earlier parts' partials (each
// published when its CTA ran that group, at the start of its range) in CTA
// order: deterministic.
//
// MXFP4 math: each 32-wide K block is summed by the tensor core (exact E2M1 x
// fp16 products, fp32 accumulate) and scaled by 2^(s-127) into the fp32 sums,
// as the reference's W4A16 row (MXFP4Kernels.metal:138-173 decodes
// value * e8m0_to_float(scale) per element; the product is the same). K order
// inside a 32-block is permuted identically for weights and activations
// (lane t takes the block's bytes 4t..4t+3, i.e. k = 8t..8t+7).
//
// Every wait is bounded (mbarriers, counters); a wait that runs out records
// MPP41_ERR_TIMEOUT and the CTA winds down through the same barrier sequence,
// skipping work, and drains its copies in flight before exiting.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {
namespace gv {

// Warp roles for CW math warps in TEAMS teams. Team q takes the units n with
// n % TEAMS == q, so while one team waits for its next stage and loads it, the
// other keeps the tensor pipes busy (one team member per scheduler).
template <int CW, int TEAMS>
struct Roles {
    static constexpr int kPW = CW;             // weight producer warp
    static constexpr int kXW = CW + 1;         // activation producer warp
    static constexpr int kSW = CW + 2;         // sync warp: cross-CTA counts and partials
    static constexpr int kThreads = (CW + 3) * 32;
    static constexpr int kTW = CW / TEAMS;     // warps per team (each unit's consumers)
    static constexpr int kBPW = 32 / kTW;      // K blocks (of 32) per warp per unit
};

constexpr uint32_t kUnitK = 1024;         // K per unit
constexpr uint32_t kBox = 8192;           // one TMA box: 16 rows x 1024 K of 4-bit weights
constexpr uint32_t kWStage = 2 * kBox;    // two boxes per unit
constexpr uint32_t kSStage = 1024;        // E8M0 scales of a unit: [box][16 rows][32 B]
constexpr uint32_t kMaxTokens = 16;
constexpr uint32_t kMaxGrid = 148;
constexpr uint32_t kSlotFloats = 2 * kMaxTokens * 16;   // one partial: [box][token][row]
constexpr uint32_t kMaxParts = 4;     // partials of other CTAs one finishing CTA adds
constexpr uint32_t kMaxChunks = 32;   // mid chunks (I <= 32768): readiness kept in a bit mask
constexpr uint32_t kChunkGroups = 64; // gate/up groups (16 channels) per 1024-channel mid chunk
constexpr uint32_t kMaxStages = 16;
constexpr uint32_t kSmemLimit = 232448;   // 227 KB opt-in per block

struct Params {
    CUtensorMap tm_wg, tm_wu, tm_wd;   // packed rows viewed [K/256][rows][128 B], box {128, 16, 4}
    CUtensorMap tm_x, tm_mid;          // activations viewed [K/64][T][64 halves], box {64, T, 16}
    const uint8_t *sg, *su, *sd;       // E8M0 scales [rows][K/32] (MXFP4 only)
    __half *mid;                       // [T][I]
    void *out;                         // [T][H], fp16 or fp32
    float *ws;                         // one down partial slot per CTA
    // [0] retire ticket, [1, 1 + n_chunks) gate/up groups published per mid chunk,
    // then per down group the number of earlier parts published
    uint32_t *sync;
    uint32_t *err;
    uint32_t T, H, I;
    uint32_t n_gg, n_dg;               // gate/up groups (16 channels), down groups (32 rows)
    uint32_t nk_g, nk_d;               // units per group: ceil(H / 1024), ceil(I / 1024)
    uint32_t u_d;                      // down units
    uint32_t n_chunks;                 // mid chunks of 1024 channels (= nk_d)
    uint32_t stages, x_bytes;          // ring depth; activation bytes per unit (T x 2 KB)
    uint32_t sc16;                     // scale rows 16-byte aligned: 16-byte copies
    unsigned long long *trace;         // optional: kTraceSlots phase stamps per CTA (profiling)
    uint32_t d_start[kMaxGrid + 1];    // first down unit of each CTA; d_start[grid] = u_d
};

// Trace slots (per CTA; clock64 cycles since the CTA started unless noted).
enum : uint32_t {
    TR_START_NS = 0,     // %globaltimer at CTA start
    TR_W_G_ISSUED,       // weight warp issued its last gate/up unit
    TR_W_ALL_ISSUED,     // weight warp issued its last unit
    TR_C_G_DONE,         // math warps finished the gate/up units
    TR_C_G_PUB,          // sync warp published the last gate/up group
    TR_X_MID_READY,      // activation warp saw its first down unit's mid chunk
    TR_C_D_DONE,         // math warps finished the down units
    TR_C_END,
    TR_C_WAIT_G,         // math warp 0: cycles waiting for stages, gate/up phase
    TR_C_WAIT_D,         // ... down phase
    TR_W_WAIT,           // weight warp: cycles waiting for free stages
    TR_X_WAIT,           // activation warp: cycles waiting for free stages
    TR_C_WORK,           // math warp 0: cycles in the unit math
    TR_C_GROUP_END,      // math warp 0: cycles in group ends
    TR_END_NS,           // %globaltimer at the math warps' end (with TR_C_END: the SM clock)
    kTraceSlots = 16
};

// Shared-memory plan (offsets from a 1024-byte aligned base). Every region
// starts 16-byte aligned; ring stages are 1024-byte aligned for the swizzle.
struct Smem {
    uint32_t w, x, s, part, pbuf, bar, misc, total;
};
__host__ __device__ constexpr Smem smem_plan(uint32_t stages, uint32_t x_bytes, uint32_t nt, uint32_t cw)
{
    Smem m{};
    m.w = 0;
    m.x = m.w + stages * kWStage;
    m.s = m.x + stages * x_bytes;
    m.part = m.s + stages * kSStage;
    m.pbuf = m.part + cw * 2 * nt * 4 * 32 * 4;
    m.bar = m.pbuf + kMaxParts * kSlotFloats * 4;
    // mbarriers: wfull, xfull, empty [kMaxStages] each; partsbar, headbar
    m.misc = (m.bar + (3 * kMaxStages + 2) * 8 + 15) & ~15u;   // 16 zero bytes, abort flag, group count
    m.total = m.misc + 32;
    return m;
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// The mbarrier receives one arrival once this thread's earlier cp.async copies land.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int CW>
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory"); }

__device__ __forceinline__ void red_release_add_gpu(uint32_t *p, uint32_t v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global_gv() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_cta_shared(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta_shared(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// The 4 bytes of w (8 packed 4-bit weights) -> 4 fp16x2 words, byte i -> d[i].
// E2M1: the bytes are unpacked into 8-bit registers and converted by
// cvt.rn.f16x2.e2m1x2 (measured on B200: 2.56 conversions per clock per SM this
// way, 1.88 with a shift per byte). INT4: (n ^ 8) - 8 exactly through fp16
// arithmetic (n ^ 8 in the mantissa of 1024, minus 1032).
template <int W>
__device__ __forceinline__ void dec4(uint32_t w, uint32_t (&d)[4])
{
    if constexpr (W == W_I4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t byte = w >> (8 * i);
            const uint32_t h = 0x64006400u | ((byte & 0xFu) ^ 8u) | ((((byte >> 4) & 0xFu) ^ 8u) << 16);
            d[i] = hsub2_bits(h, 0x64086408u);
        }
    } else {
        asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\t"
            "mov.b32 {t0, t1, t2, t3}, %4;\n\t"
            "cvt.rn.f16x2.e2m1x2 %0, t0;\n\tcvt.rn.f16x2.e2m1x2 %1, t1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, t2;\n\tcvt.rn.f16x2.e2m1x2 %3, t3;\n\t}"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(w));
    }
}

// D += A x B (m16n8k16, fp16 in, fp32 accumulate); register-only, so the
// compiler may schedule it freely.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A x B with a zero accumulator.
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// Per-lane shared-memory offsets, fixed for the whole kernel (the warp's BPW K
// blocks of a unit are blocks warp*BPW .. warp*BPW+BPW-1 of its 32).
template <int NT, int BPW>
struct LaneOff {
    uint32_t w[BPW];       // weights of block b, row g, in box 0 (row g + 8: +1024; box 1: +kBox)
    uint32_t x[BPW][NT];   // activation granule of block b, token nt*8 + g (~0u past the last token)
    uint32_t s;            // scale bytes of row g in box 0 (row g + 8: +256; box 1: +512)
};

template <int NT, int BPW>
__device__ __forceinline__ LaneOff<NT, BPW> lane_offsets(uint32_t warp, uint32_t g, uint32_t t, uint32_t T)
{
    LaneOff<NT, BPW> o;
#pragma unroll
    for (int b = 0; b < BPW; ++b) {
        // weights: block bi is 16-byte granule j = bi%8 of 128-byte chunk c = bi/8 of its
        // row; line = c*16 + row, swizzled by row & 7 = g for rows g and g + 8
        const uint32_t bi = warp * BPW + b, c = bi >> 3, j = bi & 7u;
        o.w[b] = (c * 16 + g) * 128 + ((j ^ g) << 4) + 4 * t;
        // activations: 64-K row kb = bi/2, granule (bi&1)*4 + t, line kb*T + token
        const uint32_t kb = bi >> 1, gran = ((bi & 1u) << 2) | t;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint32_t tok = nt * 8 + g, line = kb * T + tok;
            o.x[b][nt] = tok < T ? line * 128 + ((gran ^ (line & 7u)) << 4) : ~0u;
        }
    }
    o.s = g * 32 + warp * BPW;
    return o;
}

// One unit's operands in registers: this warp's BPW K blocks of both 16-row
// boxes (packed weights, packed scale bytes) and the activations.
template <int NT, int BPW>
struct UnitRegs {
    uint4 xv[BPW][NT];
    uint32_t wr[2][BPW][2];
    uint32_t sc[2][2][(BPW + 3) / 4];   // E8M0 bytes of the warp's blocks, rows g, g + 8 (byte b%4 of word b/4)
};

// Shared memory -> registers (plain loads, ordered after the stage's mbarrier
// wait by its memory clobber).
template <int W, int NT, int BPW>
__device__ __forceinline__ void load_unit(UnitRegs<NT, BPW> &r, const uint8_t *wst, const uint8_t *xst,
                                          const uint8_t *sst, const uint8_t *zero16, const LaneOff<NT, BPW> &o)
{
#pragma unroll
    for (int b = 0; b < BPW; ++b)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            r.xv[b][nt] = *reinterpret_cast<const uint4 *>(o.x[b][nt] != ~0u ? xst + o.x[b][nt] : zero16);
#pragma unroll
    for (int bx = 0; bx < 2; ++bx) {
#pragma unroll
        for (int b = 0; b < BPW; ++b) {
            r.wr[bx][b][0] = *reinterpret_cast<const uint32_t *>(wst + bx * kBox + o.w[b]);
            r.wr[bx][b][1] = *reinterpret_cast<const uint32_t *>(wst + bx * kBox + o.w[b] + 1024);
        }
        if constexpr (W == W_MXFP4 && BPW >= 4) {
#pragma unroll
            for (int q = 0; q < BPW / 4; ++q) {
                r.sc[bx][0][q] = *reinterpret_cast<const uint32_t *>(sst + bx * 512 + o.s + 4 * q);
                r.sc[bx][1][q] = *reinterpret_cast<const uint32_t *>(sst + bx * 512 + o.s + 256 + 4 * q);
            }
        } else if constexpr (W == W_MXFP4) {
            r.sc[bx][0][0] = *reinterpret_cast<const uint16_t *>(sst + bx * 512 + o.s);
            r.sc[bx][1][0] = *reinterpret_cast<const uint16_t *>(sst + bx * 512 + o.s + 256);
        }
    }
}

// One unit's math, summed into acc[box][tile]. T1: one token, so only fragment
// elements 0 and 2 (column 2t, token 0 in lanes t = 0) matter.
template <int W, int NT, bool T1, int BPW>
__device__ __forceinline__ void compute_unit(const UnitRegs<NT, BPW> &r, float (&acc)[2][NT][4])
{
#pragma unroll
    for (int bx = 0; bx < 2; ++bx) {
#pragma unroll
        for (int b = 0; b < BPW; ++b) {
            uint32_t dl[4], dh[4];
            dec4<W>(r.wr[bx][b][0], dl);
            dec4<W>(r.wr[bx][b][1], dh);
            const uint32_t a0s0 = dl[0], a2s0 = dl[1], a0s1 = dl[2], a2s1 = dl[3];
            const uint32_t a1s0 = dh[0], a3s0 = dh[1], a1s1 = dh[2], a3s1 = dh[3];
            if constexpr (W == W_MXFP4) {
                // E8M0 byte b -> float bits byte << 23 (byte select, then an integer multiply)
                const float sl = __uint_as_float(__byte_perm(r.sc[bx][0][b / 4], 0u, 0x4440u | (b % 4)) * (1u << 23));
                const float sh = __uint_as_float(__byte_perm(r.sc[bx][1][b / 4], 0u, 0x4440u | (b % 4)) * (1u << 23));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float tmp[4];
                    mma16816_z(tmp, a0s0, a1s0, a2s0, a3s0, r.xv[b][nt].x, r.xv[b][nt].y);
                    mma16816(tmp, a0s1, a1s1, a2s1, a3s1, r.xv[b][nt].z, r.xv[b][nt].w);
                    acc[bx][nt][0] = fmaf(tmp[0], sl, acc[bx][nt][0]);
                    acc[bx][nt][2] = fmaf(tmp[2], sh, acc[bx][nt][2]);
                    if constexpr (!T1) {
                        acc[bx][nt][1] = fmaf(tmp[1], sl, acc[bx][nt][1]);
                        acc[bx][nt][3] = fmaf(tmp[3], sh, acc[bx][nt][3]);
                    }
                }
            } else {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    mma16816(acc[bx][nt], a0s0, a1s0, a2s0, a3s0, r.xv[b][nt].x, r.xv[b][nt].y);
                    mma16816(acc[bx][nt], a0s1, a1s1, a2s1, a3s1, r.xv[b][nt].z, r.xv[b][nt].w);
                }
            }
        }
    }
}

// A finished group sum: gate/up -> SwiGLU -> fp16 mid channel grp*16 + row;
// down -> output rows grp*32 + row and grp*32 + 16 + row.
template <int EG, bool OUT_F16>
__device__ __forceinline__ void finish_group(const Params &p, bool dphase, uint32_t grp, uint32_t row, uint32_t tok,
                                             float v0, float v1)
{
    if (tok >= p.T) return;
    if (!dphase) {
        p.mid[(size_t)tok * p.I + grp * 16 + row] = __float2half_rn(swiglu<EG>(v0, v1));
    } else {
        const size_t o0 = (size_t)tok * p.H + grp * 32 + row;
        if constexpr (OUT_F16) {
            static_cast<__half *>(p.out)[o0] = __float2half_rn(v0);
            static_cast<__half *>(p.out)[o0 + 16] = __float2half_rn(v1);
        } else {
            static_cast<float *>(p.out)[o0] = v0;
            static_cast<float *>(p.out)[o0 + 16] = v1;
        }
    }
}

// Order of a CTA's down units [d0, d1) (groups of nk units): first the units of
// its last group gB (K chunks from 0), then any whole groups between, then the
// units of its first group gA (its highest K chunks) last.
struct DownIter {
    uint32_t gA, gB, kA, kB, nk;   // kA: first chunk of gA here; kB: end chunk of gB here
    uint32_t seg, grp, kc, end;    // segment 0: gB; 1: whole groups; 2: gA
    __device__ __forceinline__ void start(uint32_t d0, uint32_t d1, uint32_t nk_)
    {
        nk = nk_;
        gA = d0 / nk;
        gB = (d1 - 1) / nk;
        kA = d0 % nk;
        kB = (d1 - 1) % nk + 1;
        if (gA == gB) {
            seg = 2; grp = gA; kc = kA; end = kB;
        } else {
            seg = 0; grp = gB; kc = 0; end = kB;
        }
    }
    // advance; true when the unit just left was the last of its group here
    __device__ __forceinline__ bool next()
    {
        if (++kc < end) return false;
        if (seg == 0 || (seg == 1 && grp + 1 >= gB)) {
            if (seg == 0 && gA + 1 < gB) {
                seg = 1; grp = gA + 1; kc = 0; end = nk;
            } else {
                seg = 2; grp = gA; kc = kA; end = nk;
            }
        } else if (seg == 1) {
            ++grp; kc = 0;
        } else {
            seg = 3;
        }
        return true;
    }
};

// The CTA (from `from` down) whose down range holds unit u.
__device__ __forceinline__ uint32_t down_owner_below(const Params &p, uint32_t u, uint32_t from)
{
    uint32_t c = from;
    while (c > 0 && p.d_start[c] > u) --c;
    return c;
}

// Workspace slot of CTA c's down partial: [box][token][row] fp32.
__device__ __forceinline__ float *ws_slot(const Params &p, uint32_t c) { return p.ws + (size_t)c * kSlotFloats; }

template <int W, int EG, bool OUT_F16, int NT, bool T1, int CW, int TEAMS>
__global__ void __launch_bounds__(Roles<CW, TEAMS>::kThreads, 1) gemv_layer_kernel(const __grid_constant__ Params p)
{
    using R = Roles<CW, TEAMS>;
    constexpr int kBPW = R::kBPW;
    constexpr bool SCALED = W == W_MXFP4;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *const gbase = smem_raw + (base - smem_u32(smem_raw));
    const Smem L = smem_plan(p.stages, p.x_bytes, NT, CW);
    uint64_t *wfull = reinterpret_cast<uint64_t *>(gbase + L.bar);
    uint64_t *xfull = wfull + kMaxStages;
    uint64_t *empty = xfull + kMaxStages;
    uint64_t *partsbar = empty + kMaxStages;   // earlier CTAs' down partials landed in pbuf
    uint64_t *headbar = partsbar + 1;          // this CTA's down partial is stored (ws)
    uint32_t *const zero16 = reinterpret_cast<uint32_t *>(gbase + L.misc);   // 16-byte aligned zeros
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + L.misc + 16);
    uint32_t *const g_stored = reinterpret_cast<uint32_t *>(gbase + L.misc + 20);   // gate/up groups stored
    float *part = reinterpret_cast<float *>(gbase + L.part);
    const float *pbuf = reinterpret_cast<const float *>(gbase + L.pbuf);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t grid = gridDim.x, cta = blockIdx.x;
    const long long clk0 = clock64();
    unsigned long long *const tr = p.trace ? p.trace + (size_t)cta * kTraceSlots : nullptr;
    if (tr && threadIdx.x == 0) tr[TR_START_NS] = globaltimer_ns();
    const uint32_t S = p.stages;
    uint32_t *const chunk_cnt = p.sync + 1;
    uint32_t *const d_cnt = chunk_cnt + p.n_chunks;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < S; ++i) {
            mbar_init(wfull + i, SCALED ? 33u : 1u);
            mbar_init(xfull + i, 1u);
            mbar_init(empty + i, R::kTW);
        }
        mbar_init(partsbar, 32u);
        mbar_init(headbar, 1u);
        *abort = 0;
        *g_stored = 0u;
        zero16[0] = zero16[1] = zero16[2] = zero16[3] = 0u;
        fence_mbar_init();
    }
    __syncthreads();

    // gate/up: groups cta, cta + grid, ... (whole); down: units [d0, d1)
    const uint32_t n_my = p.n_gg > cta ? (p.n_gg - cta + grid - 1) / grid : 0;
    const uint32_t d0 = p.d_start[cta], d1 = p.d_start[cta + 1];
    const uint32_t n_gu = n_my * p.nk_g, n_units = n_gu + (d1 - d0);
    const uint32_t nkd = p.nk_d;
    // down groups shared with other CTAs: the last one continues past d1 (this CTA
    // publishes a partial); the first one began before d0 and ends here (finished here)
    const bool d_pub = d1 > d0 && ((d1 - 1) / nkd) * nkd + nkd > d1;
    const uint32_t d_pub_grp = d1 > d0 ? (d1 - 1) / nkd : 0;
    const bool d_fin = d1 > d0 && (d0 / nkd) * nkd < d0 && (d0 / nkd) * nkd + nkd <= d1;
    const uint32_t d_fin_grp = d0 / nkd;
    const uint32_t d_fin_lo = d_fin ? down_owner_below(p, d_fin_grp * nkd, cta) : cta;

    if (warp == R::kPW) {
        // ---------------------------------------------------------- weights + scales
        // packed weights and scales are inputs that no earlier kernel writes:
        // they stream before griddepcontrol.wait
        if (elect_one_sync()) {
            tma_prefetch_desc(&p.tm_wg);
            tma_prefetch_desc(&p.tm_wu);
            tma_prefetch_desc(&p.tm_wd);
        }
        __syncwarp();
        uint32_t issued = 0;
        long long wwait = 0;
        // stage s used for the (par+1)-th time; group / K chunk of the unit (no divisions in the loop)
        uint32_t s = 0, par = 0, grp = cta, kc = 0;
        DownIter it;
        bool dphase = false;
        for (uint32_t n = 0; n < n_units; ++n) {
            if (!dphase && n == n_gu) {
                dphase = true;
                it.start(d0, d1, nkd);
                if (tr && lane == 0) tr[TR_W_G_ISSUED] = clock64() - clk0;
            }
            if (dphase) {
                grp = it.grp;
                kc = it.kc;
            }
            const long long tw = clock64();
            if (n >= S && !warp_wait(empty + s, par ^ 1u, abort, p.err, 0xE01)) break;
            wwait += clock64() - tw;
            const uint32_t K = dphase ? p.I : p.H;
            if (elect_one_sync()) {
                mbar_arrive_expect_tx(wfull + s, kWStage);
                uint8_t *dst = gbase + L.w + s * kWStage;
                if (dphase) {
                    tma_load_3d(dst, &p.tm_wd, 0, (int)(grp * 32), (int)(kc * 4), wfull + s);
                    tma_load_3d(dst + kBox, &p.tm_wd, 0, (int)(grp * 32 + 16), (int)(kc * 4), wfull + s);
                } else {
                    tma_load_3d(dst, &p.tm_wg, 0, (int)(grp * 16), (int)(kc * 4), wfull + s);
                    tma_load_3d(dst + kBox, &p.tm_wu, 0, (int)(grp * 16), (int)(kc * 4), wfull + s);
                }
            }
            if constexpr (SCALED) {
                // [box][16 rows][32 bytes]: bytes kc*32 .. +32 of each row's K/32 scale bytes
                const uint32_t rowb = K / 32, kbyte = kc * 32, sdst = base + L.s + s * kSStage;
                if (p.sc16) {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const uint32_t idx = lane + 32 * i, bx = idx >> 5, row = (idx >> 1) & 15u, q = idx & 1u;
                        const uint8_t *src = dphase ? p.sd + (size_t)(grp * 32 + bx * 16 + row) * rowb
                                                    : (bx ? p.su : p.sg) + (size_t)(grp * 16 + row) * rowb;
                        if (kbyte + q * 16 < rowb) cp_async16(sdst + bx * 512 + row * 32 + q * 16, src + kbyte + q * 16);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t idx = lane + 32 * i, bx = idx >> 7, row = (idx >> 3) & 15u, q = idx & 7u;
                        const uint8_t *src = dphase ? p.sd + (size_t)(grp * 32 + bx * 16 + row) * rowb
                                                    : (bx ? p.su : p.sg) + (size_t)(grp * 16 + row) * rowb;
                        if (kbyte + q * 4 < rowb) cp_async4(sdst + bx * 512 + row * 32 + q * 4, src + kbyte + q * 4);
                    }
                }
                cp_async_arrive_noinc(wfull + s);
            }
            issued = n + 1;
            if (dphase) {
                it.next();
            } else if (++kc == p.nk_g) {
                kc = 0;
                grp += grid;
            }
            if (++s == S) { s = 0; par ^= 1u; }
        }
        if (tr && lane == 0) {
            tr[TR_W_ALL_ISSUED] = clock64() - clk0;
            tr[TR_W_WAIT] = wwait;
        }
        if constexpr (SCALED) cp_async_wait_all();
        // drain: every issued stage has landed before the CTA may exit (on the
        // normal path these phases completed long ago and the waits return at once)
        if (elect_one_sync()) {
            for (uint32_t n = issued > S ? issued - S : 0; n < issued; ++n)
                mbar_wait(wfull + n % S, (n / S) & 1u, nullptr, p.err, 0xE02);
        }
        __syncwarp();
    } else if (warp == R::kXW) {
        // ---------------------------------------------------------- activations
        pdl_wait_prior();
        if (elect_one_sync()) {
            tma_prefetch_desc(&p.tm_x);
            tma_prefetch_desc(&p.tm_mid);
        }
        __syncwarp();
        uint32_t issued = 0, ready = 0;   // ready: bit c = mid chunk c published grid-wide
        long long xwait = 0;
        uint32_t s = 0, par = 0, kc = 0;
        DownIter it;
        bool dphase = false;
        for (uint32_t n = 0; n < n_units; ++n) {
            if (!dphase && n == n_gu) {
                dphase = true;
                it.start(d0, d1, nkd);
            }
            if (dphase) kc = it.kc;
            if (dphase && !((ready >> kc) & 1u)) {
                // every gate/up group of mid chunk kc is published (other CTAs publish
                // theirs independently of this CTA's progress: no deadlock)
                const uint32_t need = min(kChunkGroups, p.n_gg - kc * kChunkGroups);
                uint32_t ok = 1;
                if (elect_one_sync()) ok = wait_flag_ge(chunk_cnt + kc, need, kWaitLimitNs, abort, p.err, 0xE04);
                if (!__all_sync(0xffffffffu, ok)) break;
                if (tr && lane == 0 && !ready) tr[TR_X_MID_READY] = clock64() - clk0;
                if (!ready) pdl_launch_dependents();
                ready |= 1u << kc;
                fence_proxy_async_global_gv();   // the mid's generic stores before our TMA reads
            }
            const long long tw = clock64();
            if (n >= S && !warp_wait(empty + s, par ^ 1u, abort, p.err, 0xE03)) break;
            xwait += clock64() - tw;
            if (elect_one_sync()) {
                mbar_arrive_expect_tx(xfull + s, p.x_bytes);
                tma_load_3d(gbase + L.x + s * p.x_bytes, dphase ? &p.tm_mid : &p.tm_x, 0, 0, (int)(kc * 16),
                            xfull + s);
            }
            __syncwarp();
            issued = n + 1;
            if (dphase) it.next();
            else if (++kc == p.nk_g) kc = 0;
            if (++s == S) { s = 0; par ^= 1u; }
        }
        if (d1 == d0) pdl_launch_dependents();   // no down units: signal here
        if (tr && lane == 0) tr[TR_X_WAIT] = xwait;
        if (elect_one_sync()) {
            for (uint32_t n = issued > S ? issued - S : 0; n < issued; ++n)
                mbar_wait(xfull + n % S, (n / S) & 1u, nullptr, p.err, 0xE05);
        }
        __syncwarp();
    } else if (warp == R::kSW) {
        // ---------------------------------------------------------- cross-CTA sync
        // Publishing takes a gpu-scope fence, which waits out the memory system's
        // queue under the weight stream: it runs here, off the math warps' path.
        pdl_wait_prior();
        bool ok = true;
        // gate/up groups as the math warps store them: one fence per batch, then one
        // count per group on its mid chunk
        for (uint32_t published = 0; ok && published < n_my;) {
            uint32_t stored = 0;
            if (lane == 0) {
                const uint64_t t0 = globaltimer_ns();
                while ((stored = ld_acquire_cta_shared(g_stored)) <= published) {
                    if (*abort) break;
                    if (globaltimer_ns() - t0 > kWaitLimitNs) {
                        report_error(p.err, kErrTimeout, 0xE0C);
                        *abort = 1;
                        break;
                    }
                    __nanosleep(64);
                }
                if (stored > published && !*abort) {
                    __threadfence();
                    for (uint32_t j = published; j < stored; ++j)
                        red_release_add_gpu(chunk_cnt + (cta + j * grid) / kChunkGroups, 1u);
                }
            }
            stored = __shfl_sync(0xffffffffu, stored, 0);
            ok = !*abort && stored > published;
            published = stored;
        }
        if (tr && lane == 0) tr[TR_C_G_PUB] = clock64() - clk0;
        // the down group continuing past d1: publish this CTA's partial
        if (ok && d_pub) {
            ok = warp_wait(headbar, 0, abort, p.err, 0xE0D);
            if (ok && elect_one_sync()) {
                __threadfence();
                red_release_add_gpu(d_cnt + d_pub_grp, 1u);
            }
            __syncwarp();
        }
        // the down group finished here: wait until every earlier part is published,
        // then copy their partials to pbuf in CTA order
        if (ok && d_fin) {
            uint32_t parts = 0;
            for (uint32_t c = d_fin_lo; c < cta; ++c) parts += p.d_start[c + 1] > p.d_start[c];
            uint32_t w = 1;
            if (elect_one_sync()) w = wait_flag_ge(d_cnt + d_fin_grp, parts, kWaitLimitNs, abort, p.err, 0xE09);
            if (__all_sync(0xffffffffu, w)) {
                uint32_t i = 0;
                for (uint32_t c = d_fin_lo; c < cta; ++c) {
                    if (p.d_start[c + 1] == p.d_start[c]) continue;
                    if (i >= kMaxParts) {   // the host sizes the grid so that this cannot happen
                        report_error(p.err, kErrBounds, 0xE0B);
                        break;
                    }
                    const float *src = ws_slot(p, c);
                    const uint32_t dst = base + L.pbuf + i * kSlotFloats * 4;
#pragma unroll
                    for (int q = 0; q < (int)(kSlotFloats * 4 / 16 / 32); ++q)
                        cp_async16(dst + (lane + 32 * q) * 16, src + (lane + 32 * q) * 4);
                    ++i;
                }
            }
        }
        cp_async_arrive_noinc(partsbar);
        cp_async_wait_all();
    } else {
        // ---------------------------------------------------------- math warps
        pdl_wait_prior();
        const uint32_t g = lane >> 2, t = lane & 3u;
        const uint32_t ctid = threadIdx.x;   // 0 .. CW*32-1
        const uint32_t team = warp / R::kTW, wt = warp % R::kTW;   // team, warp within the team
        const LaneOff<NT, kBPW> lo = lane_offsets<NT, kBPW>(wt, g, t, p.T);
        // element e = ctid < NT*128 of a group's sums: tile nt = e >> 7, fragment i, lane l;
        // row (l>>2) + 8*(i>>1), token nt*8 + 2*(l&3) + (i&1)
        const bool mine = ctid < (uint32_t)NT * 128;
        const uint32_t el = ctid & 31u, ei = (ctid >> 5) & 3u, ent = ctid >> 7;
        const uint32_t row = (el >> 2) + 8 * (ei >> 1), tok = ent * 8 + 2 * (el & 3u) + (ei & 1u);
        float acc[2][NT][4];
        uint32_t s = 0, par = 0;   // ring stage and its use parity, carried across the phases
        long long cwait = 0, cwork = 0, cgroup = 0;
        auto zero_acc = [&]() {
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
        };
        // one unit: wait for its stage, load it into registers, multiply, release the
        // stage (units of the other team only advance the stage counter)
        uint32_t n_at = 0;
        auto unit = [&](uint32_t kc, uint32_t K) {
            const bool my = (n_at++ % TEAMS) == team;
            if (!my) {
                if (++s == S) { s = 0; par ^= 1u; }
                return;
            }
            const long long tw = clock64();
            bool ok = !*abort;
            ok = ok && warp_wait(wfull + s, par, abort, p.err, 0xE06);
            ok = ok && warp_wait(xfull + s, par, abort, p.err, 0xE07);
            const long long tc = clock64();
            cwait += tc - tw;
            if (ok && kc * kUnitK + wt * kBPW * 32 < K) {
                UnitRegs<NT, kBPW> r;
                load_unit<W, NT, kBPW>(r, gbase + L.w + s * kWStage, gbase + L.x + s * p.x_bytes,
                                       gbase + L.s + s * kSStage, reinterpret_cast<const uint8_t *>(zero16), lo);
                compute_unit<W, NT, T1, kBPW>(r, acc);
            }
            cwork += clock64() - tc;
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + s);
            if (++s == S) { s = 0; par ^= 1u; }
        };
        // group end: the warps' sums in warp order -> (v0, v1) of element ctid
        auto group_sums = [&](float &v0, float &v1) {
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) part[(((warp * 2 + a) * NT + nt) * 4 + i) * 32 + lane] = acc[a][nt][i];
            consumer_bar<CW>();
            v0 = v1 = 0.f;
            if (mine) {
                for (int w = 0; w < CW; ++w) {
                    v0 += part[(((w * 2 + 0) * NT + ent) * 4 + ei) * 32 + el];
                    v1 += part[(((w * 2 + 1) * NT + ent) * 4 + ei) * 32 + el];
                }
            }
        };
        uint32_t j = 0, kcg = 0;   // gate/up: group index of this CTA, K chunk
        DownIter it;
        zero_acc();
        for (uint32_t n = 0; n < n_units; ++n) {
            const bool dphase = n >= n_gu;
            if (dphase && n == n_gu) it.start(d0, d1, nkd);
            const uint32_t ugrp = dphase ? it.grp : cta + j * grid;
            unit(dphase ? it.kc : kcg, dphase ? p.I : p.H);
            bool group_end;
            if (dphase) {
                group_end = it.next();
            } else {
                group_end = ++kcg == p.nk_g;
                if (group_end) { kcg = 0; ++j; }
            }
            if (group_end) {
                const long long tge = clock64();
                float v0, v1;
                group_sums(v0, v1);
                zero_acc();
                const bool live = !*abort;
                if (!dphase) {
                    // gate/up group (whole here): SwiGLU -> mid, published by the sync warp
                    if (mine && live) {
                        finish_group<EG, OUT_F16>(p, false, ugrp, row, tok, v0, v1);
                        fence_proxy_async_global_gv();   // the mid is read by other CTAs' TMA
                    }
                    consumer_bar<CW>();   // mid stored (and part[] free again)
                    if (ctid == 0) st_release_cta_shared(g_stored, j);
                    if (tr && ctid == 0 && j == n_my) {
                        tr[TR_C_G_DONE] = clock64() - clk0;
                        tr[TR_C_WAIT_G] = cwait;
                    }
                } else if (d_pub && ugrp == d_pub_grp) {
                    // continues in later CTAs: store the partial for its finishing CTA
                    if (mine && live) {
                        float *ws = ws_slot(p, cta);
                        __stcg(ws + tok * 16 + row, v0);
                        __stcg(ws + (kMaxTokens + tok) * 16 + row, v1);
                    }
                    consumer_bar<CW>();
                    if (ctid == 0) mbar_arrive(headbar);   // the sync warp publishes it
                } else {
                    if (d_fin && ugrp == d_fin_grp) {
                        // finished here: earlier parts' partials (CTA order), then this one's
                        const bool got = warp_wait(partsbar, 0, abort, p.err, 0xE0A);
                        if (got && mine) {
                            float e0 = 0.f, e1 = 0.f;
                            uint32_t i = 0;
                            for (uint32_t c = d_fin_lo; c < cta; ++c) {
                                if (p.d_start[c + 1] == p.d_start[c]) continue;
                                e0 += pbuf[i * kSlotFloats + tok * 16 + row];
                                e1 += pbuf[i * kSlotFloats + (kMaxTokens + tok) * 16 + row];
                                ++i;
                            }
                            v0 = e0 + v0;
                            v1 = e1 + v1;
                        }
                        if (ctid == 0) d_cnt[ugrp] = 0u;   // every part has arrived: the count is free again
                    }
                    if (mine && live) finish_group<EG, OUT_F16>(p, true, ugrp, row, tok, v0, v1);
                    consumer_bar<CW>();   // part[] is rewritten at the next group end
                }
                cgroup += clock64() - tge;
            }
        }
        if (tr && ctid == 0) {
            tr[TR_C_D_DONE] = clock64() - clk0;
            tr[TR_C_WAIT_D] = cwait - (n_my ? (long long)tr[TR_C_WAIT_G] : 0);
            tr[TR_C_END] = clock64() - clk0;
            tr[TR_C_WORK] = cwork;
            tr[TR_C_GROUP_END] = cgroup;
            tr[TR_END_NS] = globaltimer_ns();
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // the last CTA to finish resets the chunk counts (every CTA has passed its waits)
        __threadfence();
        const uint32_t tk = atomicAdd(p.sync, 1u);
        if (tk == grid - 1) {
            for (uint32_t c = 0; c < p.n_chunks; ++c) atomicExch(chunk_cnt + c, 0u);
            atomicExch(p.sync, 0u);
        }
    }
}

}  // namespace gv
}  // namespace mpp41
