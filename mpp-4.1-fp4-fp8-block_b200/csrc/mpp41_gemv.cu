// Decode-sized MLP layer (T <= 32 tokens) with 4-bit weights (MXFP4, unscaled
// FP4 or INT4), the W4A16 math of the fused layer -- exact E2M1 x fp16 products, fp32
// sums, SwiGLU on the fp32 gate/up sums, fp16 mid -- as two weight-streaming
// kernels (gate/up + SwiGLU, then down). With so few tokens the layer is a
// stream of 4-bit weights; decoding them into shared or tensor memory for
// tcgen05 costs more than the stream itself, so here the packed bytes go from
// global memory straight into registers, are expanded with
// cvt.rn.f16x2.e2m1x2 into the A fragments of mma.sync.m16n8k16 (fp32
// accumulate), and the tokens are the N = 8 side (up to four N tiles).
//
// Per warp: 16 weight rows, staged chunk by chunk in shared memory; per 32-wide K block (one E8M0 scale per row) two
// MMAs sum into a fresh fragment that is then scaled by the block scale and
// added to the running fp32 sums (scale 2^(s-127) built as s << 23: byte 0
// gives 0 and 255 infinity, as the reference's e8m0_to_float,
// MXFP4Kernels.metal:26-29). K order inside a block is permuted the same way
// for weights and activations (lane t of a row group takes the block's bytes
// 4t..4t+3, i.e. k = 8t..8t+7), which leaves every block sum unchanged. The
// warps of a CTA split K (strided over 128-wide chunks) and add their partial
// sums through shared memory in warp order.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"
#include "mpp41_gemv.cuh"

#include <cstring>

namespace mpp41 {
namespace gemv {

constexpr int kGateWarps = 8;    // K split of the gate/up kernel (16 channels per CTA)
constexpr int kDownWarps = 16;   // K split of the down kernel (16 output rows per CTA)

__device__ __forceinline__ uint32_t e2m1x2_to_h2(uint32_t byte)
{
    uint32_t h2;
    asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h2) : "r"(byte));
    return h2;
}

// Two packed 4-bit weights (one byte, low nibble = even k) -> half2, exactly:
// E2M1 by the hardware conversion; INT4 (two's complement, the reference's
// (n ^ 8) - 8) by placing n ^ 8 in the mantissa of 1024 and subtracting 1032.
template <int W>
__device__ __forceinline__ uint32_t dec2(uint32_t byte)
{
    if constexpr (W == W_I4) {
        const uint32_t h = 0x64006400u | ((byte & 0xFu) ^ 8u) | ((((byte >> 4) & 0xFu) ^ 8u) << 16);
        const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&h), __halves2half2(__ushort_as_half(0x6408),
                                                                                        __ushort_as_half(0x6408)));
        return *reinterpret_cast<const uint32_t *>(&r);
    } else {
        return e2m1x2_to_h2(byte);
    }
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float e8m0(uint32_t s) { return __uint_as_float(s << 23); }

// Weight staging: each warp copies its 16 rows x 64 bytes (one 128-wide K
// chunk) of each weight matrix into shared memory with 16-byte cp.async
// (full sectors), kStage - 1 chunks ahead. Rows are 80 bytes apart, so the
// fragment reads (lane g, t: row g, bytes 16b + 4t) hit 32 distinct banks.
constexpr int kStage = 2;   // 2, 3 and 4 measured within 10 %; 2 was fastest
constexpr uint32_t kRowPitch = 80;
constexpr uint32_t kMatBytes = 16 * kRowPitch;   // one 16-row chunk of one matrix

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Lane l copies segments l and l + 32 of the chunk: row = seg / 4, 16 bytes at
// (seg % 4) * 16 of the chunk's 64 bytes in that row.
__device__ __forceinline__ void stage_chunk(uint8_t *dst, const uint8_t *w, uint32_t K, uint32_t r0, uint32_t ch,
                                            uint32_t lane)
{
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t seg = lane + 32 * i, row = seg >> 2, part = seg & 3;
        cp_async16(dst + row * kRowPitch + part * 16, w + (size_t)(r0 + row) * (K / 2) + (size_t)ch * 64 + part * 16);
    }
}

// One 32-wide K block of one 16-row weight group against NT token tiles:
// wg = this lane's 4 bytes of row g, wg8 = of row g + 8; x[nt] = the lane's 8
// activations (k = 8t..8t+7) of token nt*8 + g; the block sums go to tmp.
template <int W, int NT>
__device__ __forceinline__ void block_mma(uint32_t wg, uint32_t wg8, const uint4 (&x)[NT], float (&tmp)[NT][4])
{
    const uint32_t a0s0 = dec2<W>(wg & 0xFFu), a2s0 = dec2<W>((wg >> 8) & 0xFFu);
    const uint32_t a1s0 = dec2<W>(wg8 & 0xFFu), a3s0 = dec2<W>((wg8 >> 8) & 0xFFu);
    const uint32_t a0s1 = dec2<W>((wg >> 16) & 0xFFu), a2s1 = dec2<W>(wg >> 24);
    const uint32_t a1s1 = dec2<W>((wg8 >> 16) & 0xFFu), a3s1 = dec2<W>(wg8 >> 24);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        tmp[nt][0] = tmp[nt][1] = tmp[nt][2] = tmp[nt][3] = 0.0f;
        mma16816(tmp[nt], a0s0, a1s0, a2s0, a3s0, x[nt].x, x[nt].y);
        mma16816(tmp[nt], a0s1, a1s1, a2s1, a3s1, x[nt].z, x[nt].w);
    }
}

// Activations of token n, k = 8t..8t+7 of block kb (zeros past the last token).
__device__ __forceinline__ uint4 load_x(const __half *x, uint32_t T, uint32_t K, uint32_t n, uint32_t kb, uint32_t t)
{
    if (n >= T) return make_uint4(0, 0, 0, 0);
    return __ldg(reinterpret_cast<const uint4 *>(x + (size_t)n * K + (size_t)kb * 32 + 8 * t));
}

// Scales of 4 consecutive blocks of row r.
template <bool SCALED>
__device__ __forceinline__ uint32_t load_s4(const uint8_t *s, uint32_t K, uint32_t r, uint32_t kb4)
{
    if constexpr (!SCALED) return 0x7F7F7F7Fu;   // 2^0 for every block
    return __ldg(reinterpret_cast<const uint32_t *>(s + (size_t)r * (K / 32) + (size_t)kb4 * 4));
}

// ---------------------------------------------------------------- gate/up + SwiGLU
// CTA: 16 channels [c0, c0+16) of gate and up, kGateWarps warps splitting K = H.
template <int W, int EG, int NT>
__global__ void __launch_bounds__(kGateWarps * 32) gate_up_kernel(const __half *__restrict__ x, const uint8_t *__restrict__ wg,
                                                                  const uint8_t *__restrict__ wu, const uint8_t *__restrict__ sg,
                                                                  const uint8_t *__restrict__ su, __half *__restrict__ mid,
                                                                  uint32_t T, uint32_t H, uint32_t I)
{
    constexpr bool SCALED = W == W_MXFP4;
    extern __shared__ __align__(16) uint8_t wsm[];   // weight ring, then (aliased) the partial sums
    float(*part)[2][NT][4][32] = reinterpret_cast<float(*)[2][NT][4][32]>(wsm);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t c0 = blockIdx.x * 16;
    float ag[NT][4] = {}, au[NT][4] = {};
    const uint32_t chunks = H / 128;
    uint8_t *ring = wsm + warp * (kStage * 2 * kMatBytes);   // [stage][gate, up]
    // prologue: the first kStage - 1 chunks of this warp in flight
    uint32_t issued = warp;
#pragma unroll
    for (int st = 0; st < kStage - 1; ++st) {
        if (issued < chunks) {
            stage_chunk(ring + st * 2 * kMatBytes, wg, H, c0, issued, lane);
            stage_chunk(ring + st * 2 * kMatBytes + kMatBytes, wu, H, c0, issued, lane);
        }
        cp_commit();
        issued += kGateWarps;
    }
    // scales and activations are loaded into registers a chunk ahead (one token tile)
    uint32_t nsg4 = 0, nsg48 = 0, nsu4 = 0, nsu48 = 0;
    uint4 nxv[4][NT];
    auto fetch = [&](uint32_t c) {
        nsg4 = load_s4<SCALED>(sg, H, c0 + g, c);
        nsg48 = load_s4<SCALED>(sg, H, c0 + g + 8, c);
        nsu4 = load_s4<SCALED>(su, H, c0 + g, c);
        nsu48 = load_s4<SCALED>(su, H, c0 + g + 8, c);
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) nxv[b][nt] = load_x(x, T, H, nt * 8 + g, c * 4 + b, t);
    };
    // one token tile: prefetch one chunk ahead; two tiles would need too many registers
    constexpr bool kAhead = NT == 1;
    if (kAhead && warp < chunks) fetch(warp);
    uint32_t slot = 0;
    for (uint32_t ch = warp; ch < chunks; ch += kGateWarps) {
        if constexpr (!kAhead) fetch(ch);
        {   // keep kStage - 1 chunks in flight
            const uint32_t fill = (slot + kStage - 1) % kStage;
            if (issued < chunks) {
                stage_chunk(ring + fill * 2 * kMatBytes, wg, H, c0, issued, lane);
                stage_chunk(ring + fill * 2 * kMatBytes + kMatBytes, wu, H, c0, issued, lane);
            }
            cp_commit();
            issued += kGateWarps;
        }
        const uint32_t sg4 = nsg4, sg48 = nsg48, su4 = nsu4, su48 = nsu48;
        uint4 xv[4][NT];
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xv[b][nt] = nxv[b][nt];
        if (kAhead && ch + kGateWarps < chunks) fetch(ch + kGateWarps);
        cp_wait<kStage - 1>();
        __syncwarp();
        const uint8_t *cg = ring + slot * 2 * kMatBytes, *cu = cg + kMatBytes;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            float tmp[NT][4];
            const uint32_t off = b * 16 + 4 * t;
            const uint32_t wgr = *reinterpret_cast<const uint32_t *>(cg + g * kRowPitch + off);
            const uint32_t wgr8 = *reinterpret_cast<const uint32_t *>(cg + (g + 8) * kRowPitch + off);
            const uint32_t wur = *reinterpret_cast<const uint32_t *>(cu + g * kRowPitch + off);
            const uint32_t wur8 = *reinterpret_cast<const uint32_t *>(cu + (g + 8) * kRowPitch + off);
            const float s0 = e8m0((sg4 >> (8 * b)) & 0xFFu), s8 = e8m0((sg48 >> (8 * b)) & 0xFFu);
            block_mma<W, NT>(wgr, wgr8, xv[b], tmp);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                ag[nt][0] = fmaf(tmp[nt][0], s0, ag[nt][0]);
                ag[nt][1] = fmaf(tmp[nt][1], s0, ag[nt][1]);
                ag[nt][2] = fmaf(tmp[nt][2], s8, ag[nt][2]);
                ag[nt][3] = fmaf(tmp[nt][3], s8, ag[nt][3]);
            }
            const float u0 = e8m0((su4 >> (8 * b)) & 0xFFu), u8 = e8m0((su48 >> (8 * b)) & 0xFFu);
            block_mma<W, NT>(wur, wur8, xv[b], tmp);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                au[nt][0] = fmaf(tmp[nt][0], u0, au[nt][0]);
                au[nt][1] = fmaf(tmp[nt][1], u0, au[nt][1]);
                au[nt][2] = fmaf(tmp[nt][2], u8, au[nt][2]);
                au[nt][3] = fmaf(tmp[nt][3], u8, au[nt][3]);
            }
        }
        __syncwarp();   // the slot is refilled next iteration
        slot = (slot + 1) % kStage;
    }
    cp_wait<0>();
    __syncthreads();   // every warp is done with the ring the partial sums reuse
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            part[warp][0][nt][i][lane] = ag[nt][i];
            part[warp][1][nt][i][lane] = au[nt][i];
        }
    __syncthreads();
    // thread -> (fragment element i, lane l, tile nt): sum the warps in order, SwiGLU, store
    for (uint32_t e = threadIdx.x; e < NT * 4 * 32; e += blockDim.x) {
        const uint32_t l = e & 31, i = (e >> 5) & 3, nt = e >> 7;
        float gs = 0.0f, us = 0.0f;
        for (int w = 0; w < kGateWarps; ++w) {
            gs += part[w][0][nt][i][l];
            us += part[w][1][nt][i][l];
        }
        // fragment element i of lane l: row (l>>2) + 8*(i>>1), token 2*(l&3) + (i&1)
        const uint32_t ch = c0 + (l >> 2) + 8 * (i >> 1), tok = nt * 8 + 2 * (l & 3) + (i & 1);
        if (tok < T && ch < I) mid[(size_t)tok * I + ch] = __float2half_rn(swiglu<EG>(gs, us));
    }
}

// ---------------------------------------------------------------- down
// CTA: 16 output columns [h0, h0+16), kDownWarps warps splitting K = I.
template <int W, bool OUT_F16, int NT>
__global__ void __launch_bounds__(kDownWarps * 32) down_kernel(const __half *__restrict__ mid, const uint8_t *__restrict__ wd,
                                                               const uint8_t *__restrict__ sd, void *__restrict__ out,
                                                               uint32_t T, uint32_t H, uint32_t I)
{
    constexpr bool SCALED = W == W_MXFP4;
    extern __shared__ __align__(16) uint8_t wsm[];
    float(*part)[NT][4][32] = reinterpret_cast<float(*)[NT][4][32]>(wsm);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t h0 = blockIdx.x * 16;
    float acc[NT][4] = {};
    const uint32_t chunks = I / 128;
    uint8_t *ring = wsm + warp * (kStage * kMatBytes);
    uint32_t issued = warp;
#pragma unroll
    for (int st = 0; st < kStage - 1; ++st) {
        if (issued < chunks) stage_chunk(ring + st * kMatBytes, wd, I, h0, issued, lane);
        cp_commit();
        issued += kDownWarps;
    }
    uint32_t ns4 = 0, ns48 = 0;
    uint4 nxv[4][NT];
    auto fetch = [&](uint32_t c) {
        ns4 = load_s4<SCALED>(sd, I, h0 + g, c);
        ns48 = load_s4<SCALED>(sd, I, h0 + g + 8, c);
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) nxv[b][nt] = load_x(mid, T, I, nt * 8 + g, c * 4 + b, t);
    };
    // one token tile: prefetch one chunk ahead; two tiles would need too many registers
    constexpr bool kAhead = NT == 1;
    if (kAhead && warp < chunks) fetch(warp);
    uint32_t slot = 0;
    for (uint32_t ch = warp; ch < chunks; ch += kDownWarps) {
        if constexpr (!kAhead) fetch(ch);
        {
            const uint32_t fill = (slot + kStage - 1) % kStage;
            if (issued < chunks) stage_chunk(ring + fill * kMatBytes, wd, I, h0, issued, lane);
            cp_commit();
            issued += kDownWarps;
        }
        const uint32_t s4 = ns4, s48 = ns48;
        uint4 xv[4][NT];
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xv[b][nt] = nxv[b][nt];
        if (kAhead && ch + kDownWarps < chunks) fetch(ch + kDownWarps);
        cp_wait<kStage - 1>();
        __syncwarp();
        const uint8_t *cw = ring + slot * kMatBytes;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            float tmp[NT][4];
            const uint32_t off = b * 16 + 4 * t;
            const uint32_t wr = *reinterpret_cast<const uint32_t *>(cw + g * kRowPitch + off);
            const uint32_t wr8 = *reinterpret_cast<const uint32_t *>(cw + (g + 8) * kRowPitch + off);
            const float s0 = e8m0((s4 >> (8 * b)) & 0xFFu), s8 = e8m0((s48 >> (8 * b)) & 0xFFu);
            block_mma<W, NT>(wr, wr8, xv[b], tmp);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[nt][0] = fmaf(tmp[nt][0], s0, acc[nt][0]);
                acc[nt][1] = fmaf(tmp[nt][1], s0, acc[nt][1]);
                acc[nt][2] = fmaf(tmp[nt][2], s8, acc[nt][2]);
                acc[nt][3] = fmaf(tmp[nt][3], s8, acc[nt][3]);
            }
        }
        __syncwarp();
        slot = (slot + 1) % kStage;
    }
    cp_wait<0>();
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) part[warp][nt][i][lane] = acc[nt][i];
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < NT * 4 * 32; e += blockDim.x) {
        const uint32_t l = e & 31, i = (e >> 5) & 3, nt = e >> 7;
        float s = 0.0f;
        for (int w = 0; w < kDownWarps; ++w) s += part[w][nt][i][l];
        const uint32_t h = h0 + (l >> 2) + 8 * (i >> 1), tok = nt * 8 + 2 * (l & 3) + (i & 1);
        if (tok < T && h < H) {
            if constexpr (OUT_F16) static_cast<__half *>(out)[(size_t)tok * H + h] = __float2half_rn(s);
            else static_cast<float *>(out)[(size_t)tok * H + h] = s;
        }
    }
}

constexpr uint32_t gate_smem(int NT)
{
    const uint32_t ring = kGateWarps * kStage * 2 * kMatBytes, part = kGateWarps * 2 * NT * 4 * 32 * 4;
    return ring > part ? ring : part;
}
constexpr uint32_t down_smem(int NT)
{
    const uint32_t ring = kDownWarps * kStage * kMatBytes, part = kDownWarps * NT * 4 * 32 * 4;
    return ring > part ? ring : part;
}

template <typename K>
bool allow_smem(K kern, uint32_t bytes)
{
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

template <int W, int EG, int NT>
int launch_nt(const FusedLaunch &L, cudaStream_t st)
{
    static const bool ok = allow_smem(gate_up_kernel<W, EG, NT>, gate_smem(NT)) &&
                           allow_smem(down_kernel<W, true, NT>, down_smem(NT)) &&
                           allow_smem(down_kernel<W, false, NT>, down_smem(NT));
    if (!ok) return 2;
    gate_up_kernel<W, EG, NT><<<L.I / 16, kGateWarps * 32, gate_smem(NT), st>>>(
        static_cast<const __half *>(L.x), static_cast<const uint8_t *>(L.wg), static_cast<const uint8_t *>(L.wu), L.sg,
        L.su, static_cast<__half *>(L.mid), L.T, L.H, L.I);
    if (L.out_f16)
        down_kernel<W, true, NT><<<L.H / 16, kDownWarps * 32, down_smem(NT), st>>>(
            static_cast<const __half *>(L.mid), static_cast<const uint8_t *>(L.wd), L.sd, L.out, L.T, L.H, L.I);
    else
        down_kernel<W, false, NT><<<L.H / 16, kDownWarps * 32, down_smem(NT), st>>>(
            static_cast<const __half *>(L.mid), static_cast<const uint8_t *>(L.wd), L.sd, L.out, L.T, L.H, L.I);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

template <int W, int EG>
int launch_eg(const FusedLaunch &L, cudaStream_t st)
{
    if (L.T <= 8) return launch_nt<W, EG, 1>(L, st);
    if (L.T <= 16) return launch_nt<W, EG, 2>(L, st);
    return launch_nt<W, EG, 4>(L, st);
}

template <int W>
int launch_s(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    switch (L.gate_epi) {
    case EPI_SWIGLU_PLAIN: return launch_eg<W, EPI_SWIGLU_PLAIN>(L, st);
    case EPI_SWIGLU_HALF: return launch_eg<W, EPI_SWIGLU_HALF>(L, st);
    case EPI_SWIGLU_HALF_H: return launch_eg<W, EPI_SWIGLU_HALF_H>(L, st);
    default: *why = "SwiGLU variant"; return 1;
    }
}

}  // namespace gemv


// ---------------------------------------------------------------- persistent streaming kernel
namespace gv {

bool covers(uint32_t T, uint32_t H, uint32_t I, int wfmt)
{
    // below 8M weights per matrix the launch's fixed costs (ring fill, one grid-wide
    // hand-off) outweigh the streaming: such layers keep the register-fed kernels
    // (BASELINE config 0 at T=1, 1024 x 4096: 7.1 us there, 12.1 us here)
    return T >= 1 && T <= kMaxTokens && (wfmt == W_MXFP4 || wfmt == W_FP4 || wfmt == W_I4) && H % 256 == 0 &&
           I % 256 == 0 && I <= kMaxChunks * kUnitK && (uint64_t)H * I >= (8ull << 20);
}

size_t ws_bytes() { return (size_t)kMaxGrid * kSlotFloats * sizeof(float); }

// retire ticket, one count per 1024-channel mid chunk, one per down group
size_t sync_words(uint32_t H, uint32_t I) { return 1 + (size_t)(I + kUnitK - 1) / kUnitK + (size_t)H / 32; }

// Down-unit starts per CTA: gate/up groups go round-robin (CTA b has
// nk_g * ceil((n_gg - b) / grid) units), and the down ranges are cut so that
// every CTA's gate/up + down total is as even as the round-robin allows
// (ds[b] = ideal cumulative total minus gate/up cumulative, kept monotone).
static void down_starts(uint32_t n_gg, uint32_t nk_g, uint32_t u_d, uint32_t grid, uint32_t *ds)
{
    const uint64_t W = (uint64_t)n_gg * nk_g + u_d;
    uint64_t cg = 0;
    ds[0] = 0;
    for (uint32_t b = 1; b < grid; ++b) {
        cg += (uint64_t)nk_g * (n_gg > b - 1 ? (n_gg - (b - 1) + grid - 1) / grid : 0);
        const int64_t ideal = (int64_t)((uint64_t)b * W / grid) - (int64_t)cg;
        int64_t v = ideal < (int64_t)ds[b - 1] ? (int64_t)ds[b - 1] : ideal;
        if (v > (int64_t)u_d) v = u_d;
        ds[b] = (uint32_t)v;
    }
    ds[grid] = u_d;
}

// Most partials of other CTAs that one down group's finishing CTA adds (the CTA
// holding a group's last units finishes it from the earlier parts).
static uint32_t max_other_parts(const uint32_t *ds, uint32_t grid, uint32_t nk)
{
    uint32_t most = 0;
    for (uint32_t b = 0; b < grid; ++b) {
        const uint32_t d0 = ds[b], d1 = ds[b + 1];
        if (d0 >= d1) continue;
        const uint32_t g0u = (d0 / nk) * nk;
        if (!(g0u < d0 && g0u + nk <= d1)) continue;   // not finishing a group that began earlier
        uint32_t n = 0;
        for (uint32_t c = b; c-- > 0 && ds[c + 1] > g0u;) n += ds[c + 1] > ds[c];
        if (n > most) most = n;
    }
    return most;
}

template <int W, int EG, bool F16, int NT, bool T1, int CW, int TEAMS>
static int launch_t(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    Params p;
    memset(&p, 0, sizeof(p));
    p.T = L.T; p.H = L.H; p.I = L.I;
    p.n_gg = L.I / 16;
    p.n_dg = L.H / 32;
    p.nk_g = (L.H + kUnitK - 1) / kUnitK;
    p.nk_d = (L.I + kUnitK - 1) / kUnitK;
    p.u_d = p.n_dg * p.nk_d;
    p.n_chunks = p.nk_d;
    p.x_bytes = L.T * 2048;
    const uint32_t fixed = smem_plan(0, 0, NT, CW).total + 1024;   // + base alignment
    uint32_t stages = (kSmemLimit - fixed) / (kWStage + kSStage + p.x_bytes);
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) { *why = "ring of fewer than 2 stages"; return 1; }
    p.stages = stages;
    const uint32_t smem = smem_plan(stages, p.x_bytes, NT, CW).total + 1024;
    if (!L.ws || !L.sync) { *why = "workspace"; return 1; }
    bool ok = make_map_rows128(&p.tm_wg, L.wg, L.H / 2, L.I, 16, 4) &&
              make_map_rows128(&p.tm_wu, L.wu, L.H / 2, L.I, 16, 4) &&
              make_map_rows128(&p.tm_wd, L.wd, L.I / 2, L.H, 16, 4) &&
              make_map_kblocks(&p.tm_x, L.x, L.H, L.T, L.T, 16) &&
              make_map_kblocks(&p.tm_mid, L.mid, L.I, L.T, L.T, 16);
    if (!ok) { *why = "tensor maps (16-byte aligned bases needed)"; return 1; }
    if (W == W_MXFP4) {
        if (!L.sg || !L.su || !L.sd) { *why = "MXFP4 scales"; return 1; }
        const uintptr_t a = reinterpret_cast<uintptr_t>(L.sg) | reinterpret_cast<uintptr_t>(L.su) |
                            reinterpret_cast<uintptr_t>(L.sd);
        if (a & 3u) { *why = "scale planes need 4-byte aligned bases"; return 1; }
        p.sc16 = (a & 15u) == 0 && (L.H / 32) % 16 == 0 && (L.I / 32) % 16 == 0;
        p.sg = L.sg; p.su = L.su; p.sd = L.sd;
    }
    p.mid = static_cast<__half *>(L.mid);
    p.out = L.out;
    p.ws = L.ws;
    p.sync = L.sync;
    p.err = L.err;
    p.trace = L.trace;

    auto kern = gemv_layer_kernel<W, EG, F16, NT, T1, CW, TEAMS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    // every CTA must be resident at once (down units wait for gate/up groups of
    // other CTAs): one CTA per SM, at most one per SM of the device
    static thread_local int checked_dev = -1, sms = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (checked_dev != dev) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        checked_dev = dev;
    }
    uint32_t grid = (uint32_t)sms < kMaxGrid ? (uint32_t)sms : kMaxGrid;
    const uint32_t work = p.n_gg > p.u_d ? p.n_gg : p.u_d;
    if (grid > work) grid = work;
    // a finishing CTA holds at most kMaxParts other partials in shared memory
    for (;; --grid) {
        down_starts(p.n_gg, p.nk_g, p.u_d, grid, p.d_start);
        if (grid == 1 || max_other_parts(p.d_start, grid, p.nk_d) <= kMaxParts) break;
    }

    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Roles<CW, TEAMS>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // programmatic stream serialization: the weight stream starts while the
    // previous kernel finishes; activations and scratch wait for it
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    return 0;
}

template <int W, int EG, bool F16>
static int launch_nt(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (L.T == 1) return launch_t<W, EG, F16, 1, true, 8, 2>(L, st, why);
    return L.T <= 8 ? launch_t<W, EG, F16, 1, false, 8, 2>(L, st, why) : launch_t<W, EG, F16, 2, false, 8, 1>(L, st, why);
}

template <int W>
static int launch_w(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    switch (L.gate_epi) {
    case EPI_SWIGLU_PLAIN:
        return L.out_f16 ? launch_nt<W, EPI_SWIGLU_PLAIN, true>(L, st, why) : launch_nt<W, EPI_SWIGLU_PLAIN, false>(L, st, why);
    case EPI_SWIGLU_HALF:
        return L.out_f16 ? launch_nt<W, EPI_SWIGLU_HALF, true>(L, st, why) : launch_nt<W, EPI_SWIGLU_HALF, false>(L, st, why);
    case EPI_SWIGLU_HALF_H:
        return L.out_f16 ? launch_nt<W, EPI_SWIGLU_HALF_H, true>(L, st, why)
                         : launch_nt<W, EPI_SWIGLU_HALF_H, false>(L, st, why);
    default: *why = "SwiGLU variant"; return 1;
    }
}

int launch(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (!covers(L.T, L.H, L.I, L.wfmt)) { *why = "shape or format"; return 1; }
    switch (L.wfmt) {
    case W_MXFP4: return launch_w<W_MXFP4>(L, st, why);
    case W_FP4: return launch_w<W_FP4>(L, st, why);
    default: return launch_w<W_I4>(L, st, why);
    }
}

}  // namespace gv

// four token tiles of 8; on the Llama-3-8B layer T = 17..32 run 80-89 us here
// against about 100 us on the weight-major tcgen05 kernel
constexpr uint32_t kGemvMaxTokens = 32;

bool gemv_covers(uint32_t T, uint32_t H, uint32_t I, int wfmt)
{
    return T >= 1 && T <= kGemvMaxTokens && (wfmt == W_MXFP4 || wfmt == W_FP4 || wfmt == W_I4) && H % 128 == 0 &&
           I % 128 == 0;
}

int launch_gemv_layer(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (!gemv_covers(L.T, L.H, L.I, L.wfmt)) { *why = "shape or format"; return 1; }
    const int rc = L.wfmt == W_MXFP4 ? gemv::launch_s<W_MXFP4>(L, st, why)
                   : L.wfmt == W_FP4 ? gemv::launch_s<W_FP4>(L, st, why)
                                     : gemv::launch_s<W_I4>(L, st, why);
    if (rc == 2) *why = cudaGetErrorString(cudaGetLastError());
    return rc;
}

}  // namespace mpp41
