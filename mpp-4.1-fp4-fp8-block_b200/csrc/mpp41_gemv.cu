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
