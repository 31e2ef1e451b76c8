// Mixture-of-experts layer around the FP4 grouped GEMM (
// router softmax -> top-k -> renormalise, token permutation, grouped expert
// MLP, weighted combine; no counterpart in the single-layer reference).
//
// Data flow for T tokens, E experts, top-k, R = T * k assignments:
//   route:    logits [T][E] fp32 -> ids [T][k] int32, weights [T][k] fp32
//   permute:  counts[E], offsets[E+1], row tiles {expert, row0, row_end},
//             perm_src[R] (row -> assignment t*k+j), inv[R] (assignment -> row);
//             rows are grouped by expert, and within an expert keep
//             assignment order, so the layout is deterministic
//   gather:   quantized x rows (MXFP4 bytes + scales) into expert order
//   experts:  grouped gate/up GEMM (SwiGLU + MXFP4 re-quantization epilogue),
//             grouped down GEMM -> y [R][H] fp32
//   combine:  out[t] = shared(t) + sum_j weights[t][j] * y[inv[t*k+j]], in slot order
// All of it is integer/byte work bound by memory except the two GEMMs.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace moe {

constexpr uint32_t kMaxExperts = 512;   // 16 logits per lane in the router
constexpr uint32_t kMaxTopK = 16;

// One warp per token. Top-k by repeated warp arg-max (ties to the lower
// expert id); weights = softmax over the chosen logits, which equals the
// full softmax renormalised over the top k (the full denominator cancels).
__global__ void route_kernel(const float *__restrict__ logits, uint32_t T, uint32_t E, uint32_t k,
                             int32_t *__restrict__ ids, float *__restrict__ weights)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= T) return;
    const uint32_t per = E / 32;
    float v[kMaxExperts / 32];
#pragma unroll
    for (uint32_t j = 0; j < kMaxExperts / 32; ++j)
        v[j] = j < per ? logits[(size_t)t * E + lane + 32 * j] : -INFINITY;
    uint32_t taken = 0;
    float best_v[kMaxTopK];
    int32_t best_i[kMaxTopK];
#pragma unroll 1
    for (uint32_t s = 0; s < k; ++s) {
        float bv = -INFINITY;
        int32_t bi = 0x7fffffff;
#pragma unroll
        for (uint32_t j = 0; j < kMaxExperts / 32; ++j) {
            const int32_t idx = (int32_t)(lane + 32 * j);
            if (j < per && !(taken >> j & 1u) && (v[j] > bv || (v[j] == bv && idx < bi))) {
                bv = v[j];
                bi = idx;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((uint32_t)bi % 32 == lane) taken |= 1u << ((uint32_t)bi / 32);
        best_v[s & (kMaxTopK - 1)] = bv;
        best_i[s & (kMaxTopK - 1)] = bi;
    }
    if (lane == 0) {
        float sum = 0.0f;
        for (uint32_t s = 0; s < k; ++s) sum += expf(best_v[s] - best_v[0]);
        for (uint32_t s = 0; s < k; ++s) {
            ids[(size_t)t * k + s] = best_i[s];
            weights[(size_t)t * k + s] = expf(best_v[s] - best_v[0]) / sum;
        }
    }
}

__global__ void count_kernel(const int32_t *__restrict__ ids, uint32_t n, uint32_t E, uint32_t *__restrict__ counts,
                             uint32_t *err)
{
    for (uint32_t a = blockIdx.x * blockDim.x + threadIdx.x; a < n; a += gridDim.x * blockDim.x) {
        const int32_t e = ids[a];
        if (e < 0 || (uint32_t)e >= E) {
            report_error(err, kErrBounds, 0xE01);
            continue;
        }
        atomicAdd(&counts[e], 1u);
    }
}

// One thread: exclusive offsets and the row-tile table (E is small).
__global__ void scan_kernel(const uint32_t *__restrict__ counts, uint32_t E, uint32_t bm, uint32_t *__restrict__ offsets,
                            uint4 *__restrict__ tiles, uint32_t *__restrict__ n_tiles)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    uint32_t off = 0, nt = 0;
    for (uint32_t e = 0; e < E; ++e) {
        offsets[e] = off;
        const uint32_t n = counts[e];
        for (uint32_t r = 0; r < n; r += bm) tiles[nt++] = make_uint4(e, off + r, off + n, 0u);
        off += n;
    }
    offsets[E] = off;
    *n_tiles = nt;
}

// One CTA per expert: a stable block-wide compaction of the assignments that
// chose it, in assignment order.
__global__ void scatter_kernel(const int32_t *__restrict__ ids, uint32_t n, const uint32_t *__restrict__ offsets,
                               uint32_t *__restrict__ perm_src, uint32_t *__restrict__ inv)
{
    __shared__ uint32_t warp_tot[32];
    __shared__ uint32_t base;
    const int32_t e = (int32_t)blockIdx.x;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (threadIdx.x == 0) base = offsets[e];
    __syncthreads();
    for (uint32_t a0 = 0; a0 < n; a0 += blockDim.x) {
        const uint32_t a = a0 + threadIdx.x;
        const bool hit = a < n && ids[a] == e;
        const uint32_t bal = __ballot_sync(0xffffffffu, hit);
        if (lane == 0) warp_tot[warp] = __popc(bal);
        __syncthreads();
        uint32_t before = 0, total = 0;
        for (uint32_t w = 0; w < nw; ++w) {
            before += w < warp ? warp_tot[w] : 0u;
            total += warp_tot[w];
        }
        if (hit) {
            const uint32_t row = base + before + __popc(bal & ((1u << lane) - 1u));
            perm_src[row] = a;
            inv[a] = row;
        }
        __syncthreads();
        if (threadIdx.x == 0) base += total;
        __syncthreads();
    }
}

// dst row r = src row (perm_src[r] / k); one warp per row, 16-byte units.
__global__ void gather_rows_kernel(const uint8_t *__restrict__ src, uint32_t row_bytes, const uint32_t *__restrict__ perm_src,
                                   uint32_t k, const uint32_t *__restrict__ n_rows, uint8_t *__restrict__ dst)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t R = *n_rows;
    for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += (gridDim.x * blockDim.x) >> 5) {
        const uint4 *s = reinterpret_cast<const uint4 *>(src + (size_t)(perm_src[r] / k) * row_bytes);
        uint4 *d = reinterpret_cast<uint4 *>(dst + (size_t)r * row_bytes);
        for (uint32_t i = lane; i < row_bytes / 16; i += 32) d[i] = s[i];
    }
}

// One CTA per token; float4 columns. Slots are summed in order 0..k-1 after
// the shared expert's row, each as one fp32 fma.
__global__ void combine_kernel(const float *__restrict__ y, const uint32_t *__restrict__ inv,
                               const float *__restrict__ w, uint32_t k, uint32_t H, const float *__restrict__ shared_y,
                               void *__restrict__ out, int out_f16)
{
    const uint32_t t = blockIdx.x;
    for (uint32_t c = threadIdx.x; c < H / 4; c += blockDim.x) {
        float4 acc = shared_y ? reinterpret_cast<const float4 *>(shared_y + (size_t)t * H)[c] : make_float4(0, 0, 0, 0);
        for (uint32_t j = 0; j < k; ++j) {
            const float wt = w[(size_t)t * k + j];
            const float4 v = reinterpret_cast<const float4 *>(y + (size_t)inv[(size_t)t * k + j] * H)[c];
            acc.x = fmaf(wt, v.x, acc.x);
            acc.y = fmaf(wt, v.y, acc.y);
            acc.z = fmaf(wt, v.z, acc.z);
            acc.w = fmaf(wt, v.w, acc.w);
        }
        if (out_f16) {
            __half2 *o = reinterpret_cast<__half2 *>(static_cast<__half *>(out) + (size_t)t * H + 4 * c);
            o[0] = __floats2half2_rn(acc.x, acc.y);
            o[1] = __floats2half2_rn(acc.z, acc.w);
        } else {
            reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)t * H)[c] = acc;
        }
    }
}

// Expert parallel: from every rank's per-expert counts allc[P][E], the
// segments {row in the receive buffer (source-major), row in the grouped
// buffer (expert-major), rows} of (source s, local expert le) at [s * El + le],
// and the row-tile table of the grouped buffer. One thread: P * El is small.
__global__ void ep_plan_kernel(const uint32_t *__restrict__ allc, uint32_t P, uint32_t E, uint32_t rank, uint32_t bm,
                               uint4 *__restrict__ segs, uint4 *__restrict__ tiles, uint32_t *__restrict__ n_tiles)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint32_t El = E / P;
    uint32_t base = 0;
    for (uint32_t s = 0; s < P; ++s)
        for (uint32_t le = 0; le < El; ++le) {
            const uint32_t n = allc[(size_t)s * E + (size_t)rank * El + le];
            segs[s * El + le] = make_uint4(base, 0u, n, 0u);
            base += n;
        }
    uint32_t off = 0, nt = 0;
    for (uint32_t le = 0; le < El; ++le) {
        const uint32_t start = off;
        for (uint32_t s = 0; s < P; ++s) {
            segs[s * El + le].y = off;
            off += segs[s * El + le].z;
        }
        for (uint32_t r = start; r < off; r += bm) tiles[nt++] = make_uint4(le, r, off, 0u);
    }
    *n_tiles = nt;
}

// One CTA per segment: a contiguous copy of rows * row_bytes bytes between
// the receive layout and the grouped layout (either direction).
__global__ void segments_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, uint32_t row_bytes,
                                const uint4 *__restrict__ segs, bool to_recv)
{
    const uint4 sg = segs[blockIdx.x];
    const size_t from = (size_t)(to_recv ? sg.y : sg.x) * row_bytes, to = (size_t)(to_recv ? sg.x : sg.y) * row_bytes;
    const size_t n16 = (size_t)sg.z * row_bytes / 16;
    const uint4 *s = reinterpret_cast<const uint4 *>(src + from);
    uint4 *d = reinterpret_cast<uint4 *>(dst + to);
    for (size_t i = threadIdx.x; i < n16; i += blockDim.x) d[i] = s[i];
}

}  // namespace moe

static unsigned grid_cap(size_t work, unsigned block, unsigned cap)
{
    const size_t g = (work + block - 1) / block;
    return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

cudaError_t launch_moe_route(const float *logits, uint32_t T, uint32_t E, uint32_t k, int32_t *ids, float *weights,
                             cudaStream_t st)
{
    if (!T) return cudaSuccess;
    moe::route_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, T, E, k, ids, weights);
    return cudaGetLastError();
}

cudaError_t launch_moe_permute(const int32_t *ids, uint32_t n, uint32_t E, uint32_t bm, uint32_t *counts,
                               uint32_t *offsets, uint4 *tiles, uint32_t *n_tiles, uint32_t *perm_src, uint32_t *inv,
                               uint32_t *err, cudaStream_t st)
{
    cudaError_t e = cudaMemsetAsync(counts, 0, E * sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    if (n) moe::count_kernel<<<grid_cap(n, 256, 148 * 4), 256, 0, st>>>(ids, n, E, counts, err);
    moe::scan_kernel<<<1, 32, 0, st>>>(counts, E, bm, offsets, tiles, n_tiles);
    if (n) moe::scatter_kernel<<<E, 512, 0, st>>>(ids, n, offsets, perm_src, inv);
    return cudaGetLastError();
}

cudaError_t launch_moe_gather(const void *src, uint32_t row_bytes, const uint32_t *perm_src, uint32_t k,
                              const uint32_t *n_rows, uint32_t max_rows, void *dst, cudaStream_t st)
{
    if (!max_rows) return cudaSuccess;
    moe::gather_rows_kernel<<<grid_cap((size_t)max_rows * 32, 256, 148 * 8), 256, 0, st>>>(
        static_cast<const uint8_t *>(src), row_bytes, perm_src, k, n_rows, static_cast<uint8_t *>(dst));
    return cudaGetLastError();
}

cudaError_t launch_moe_ep_plan(const uint32_t *allc, uint32_t P, uint32_t E, uint32_t rank, uint32_t bm, uint4 *segs,
                               uint4 *tiles, uint32_t *n_tiles, cudaStream_t st)
{
    moe::ep_plan_kernel<<<1, 32, 0, st>>>(allc, P, E, rank, bm, segs, tiles, n_tiles);
    return cudaGetLastError();
}

cudaError_t launch_moe_segments(const void *src, void *dst, uint32_t row_bytes, const uint4 *segs, uint32_t nsegs,
                                bool to_recv, cudaStream_t st)
{
    if (!nsegs) return cudaSuccess;
    moe::segments_kernel<<<nsegs, 256, 0, st>>>(static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst),
                                                row_bytes, segs, to_recv);
    return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float *y, const uint32_t *inv, const float *w, uint32_t T, uint32_t k, uint32_t H,
                               const float *shared_y, void *out, bool out_f16, cudaStream_t st)
{
    if (!T) return cudaSuccess;
    moe::combine_kernel<<<T, 256, 0, st>>>(y, inv, w, k, H, shared_y, out, out_f16 ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace mpp41
