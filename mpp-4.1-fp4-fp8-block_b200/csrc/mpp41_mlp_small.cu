// Host side of the small-layer MLP kernel (mpp41_mlp_small.cuh): shape check,
// tensor maps, co-residency check and the launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "mpp41_internal.h"
#include "mpp41_mlp_small.cuh"

namespace mpp41 {
namespace sl {

template <int W>
static bool covers_t(uint32_t T, uint32_t H, uint32_t I)
{
    using F = Fmt<W>;
    if (T == 0 || T > 2 * kNT) return false;
    if (H % F::kSK || (uint64_t)kNT * H * 2 > kXBytes) return false;
    const uint32_t ks = I / kSplits;
    if (I % (kSplits * F::kSK) || ks / F::kSK > kMaxMSt || H / F::kSK > kMaxXSt) return false;
    // the E8M0 rows staged per tile are exactly H/32 and I/8/32 bytes
    if (F::kMx && (H / 32 != kScGRow || ks / 32 != kScDRow)) return false;
    return true;
}

bool covers(uint32_t T, uint32_t H, uint32_t I, int wfmt)
{
    switch (wfmt) {
    case W_MXFP4: return covers_t<W_MXFP4>(T, H, I);
    case W_FP4: return covers_t<W_FP4>(T, H, I);
    case W_I4: return covers_t<W_I4>(T, H, I);
    case W_I8: return covers_t<W_I8>(T, H, I);
    case W_I2: return covers_t<W_I2>(T, H, I);
    case W_E4M3: return covers_t<W_E4M3>(T, H, I);
    case W_E5M2: return covers_t<W_E5M2>(T, H, I);
    case W_E4M3_MX: return covers_t<W_E4M3_MX>(T, H, I);
    case W_E5M2_MX: return covers_t<W_E5M2_MX>(T, H, I);
    default: return false;   // fp16 weights are not packed
    }
}

size_t sync_words(uint32_t T, uint32_t H)
{
    const size_t n_h = (T + kNT - 1) / kNT;
    return 1 + n_h * kSplits + n_h * (H / kRows);
}

size_t ws_bytes(uint32_t T, uint32_t H)
{
    const size_t n_h = (T + kNT - 1) / kNT;
    return n_h * (H / kRows) * kSplits * kNT * kRows * sizeof(float);
}

template <int W, int EG, bool F16>
static int launch_t(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    Params p;
    memset(&p, 0, sizeof(p));
    p.T = L.T; p.H = L.H; p.I = L.I;
    p.n_h = (L.T + kNT - 1) / kNT;
    p.n_g = (L.I / kGCh) * p.n_h;
    p.g_per_split = (L.I / kGCh) / kSplits;
    p.n_d = (L.H / kRows) * p.n_h * kSplits;
    // at most one G tile and one D tile per CTA
    const uint32_t grid = p.n_g > p.n_d ? p.n_g : p.n_d;
    if (!L.ws) { *why = "workspace"; return 1; }
    using F = Fmt<W>;
    const uint64_t rawH = (uint64_t)L.H * F::kBits / 8, rawI = (uint64_t)L.I * F::kBits / 8;
    const CUtensorMapSwizzle wsw = F::kSw ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    bool ok = make_map_kblocks(&p.tm_x, L.x, L.H, L.T, kNT, F::kSK / 64) &&
              make_map_kblocks(&p.tm_mid, L.mid, L.I, L.T, kNT, F::kSK / 64) &&
              make_map(&p.tm_wg, L.wg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawH, L.I, F::kRowB, kGCh, wsw) &&
              make_map(&p.tm_wu, L.wu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawH, L.I, F::kRowB, kGCh, wsw) &&
              make_map(&p.tm_wd, L.wd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawI, L.H, F::kRowB, kRows, wsw);
    if (ok && F::kMx)
        ok = make_map(&p.tm_sg, L.sg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.H / 32, L.I, kScGRow, kGCh, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_su, L.su, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.H / 32, L.I, kScGRow, kGCh, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_sd, L.sd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.I / 32, L.H, kScDRow, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (L.row_scales) {
        if (W != W_I8 && W != W_I4 && W != W_I2) { *why = "per-row scales need INT8/INT4/INT2 weights"; return 1; }
        if (!L.sg || !L.su || !L.sd) { *why = "per-row scales need gate, up and down scale vectors"; return 1; }
        p.rs_g = reinterpret_cast<const __half *>(L.sg);
        p.rs_u = reinterpret_cast<const __half *>(L.su);
        p.rs_d = reinterpret_cast<const __half *>(L.sd);
    }
    if (!ok) { *why = "tensor maps (16-byte aligned bases and row pitches needed)"; return 1; }
    p.mid = static_cast<__half *>(L.mid);
    p.out = L.out;
    p.ws = L.ws;
    p.sync = L.sync;
    p.err = L.err;
    p.trace = L.trace;

    auto kern = mlp_small_kernel<W, EG, F16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }

    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    // The D tiles wait on counters bumped by other CTAs' G tiles, and the K
    // splits of an output tile wait for each other: every CTA of the grid must
    // be resident at once (one per SM: shared memory and all of tensor memory).
    static thread_local int checked_dev = -1, checked_ctas = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (checked_dev != dev) {
        int per_sm = 0, sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, kSmem);
        if (e != cudaSuccess) { cudaGetLastError(); per_sm = 0; }
        checked_dev = dev;
        checked_ctas = per_sm * sms;
    }
    if ((uint32_t)checked_ctas < grid) {
        static thread_local char msg[96];
        snprintf(msg, sizeof(msg), "%d co-resident CTAs, %u needed", checked_ctas, grid);
        *why = msg;
        return 1;
    }
    // Programmatic stream serialization: the grid may launch while the previous
    // kernel finishes; it only loads and decodes weights until griddepcontrol.wait.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    return 0;
}

template <int W>
static int launch_w(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (L.out_f16) {
        switch (L.gate_epi) {
        case EPI_SWIGLU_HALF: return launch_t<W, EPI_SWIGLU_HALF, true>(L, st, why);
        case EPI_SWIGLU_HALF_H: return launch_t<W, EPI_SWIGLU_HALF_H, true>(L, st, why);
        case EPI_SWIGLU_PLAIN: return launch_t<W, EPI_SWIGLU_PLAIN, true>(L, st, why);
        }
    } else {
        switch (L.gate_epi) {
        case EPI_SWIGLU_HALF: return launch_t<W, EPI_SWIGLU_HALF, false>(L, st, why);
        case EPI_SWIGLU_HALF_H: return launch_t<W, EPI_SWIGLU_HALF_H, false>(L, st, why);
        case EPI_SWIGLU_PLAIN: return launch_t<W, EPI_SWIGLU_PLAIN, false>(L, st, why);
        }
    }
    *why = "epilogue";
    return 1;
}

int launch(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (!covers(L.T, L.H, L.I, L.wfmt)) { *why = "shape or format not covered by the small-layer kernel"; return 1; }
    switch (L.wfmt) {
    case W_FP4: return launch_w<W_FP4>(L, st, why);
    case W_I4: return launch_w<W_I4>(L, st, why);
    case W_MXFP4: return launch_w<W_MXFP4>(L, st, why);
    case W_I8: return launch_w<W_I8>(L, st, why);
    case W_I2: return launch_w<W_I2>(L, st, why);
    case W_E4M3: return launch_w<W_E4M3>(L, st, why);
    case W_E5M2: return launch_w<W_E5M2>(L, st, why);
    case W_E4M3_MX: return launch_w<W_E4M3_MX>(L, st, why);
    case W_E5M2_MX: return launch_w<W_E5M2_MX>(L, st, why);
    default: *why = "weight format not covered by the small-layer kernel"; return 1;
    }
}

}  // namespace sl
}  // namespace mpp41
