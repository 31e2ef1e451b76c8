// Host side of the token-major persistent MLP kernel: tensor maps, cooperative
// launch (all CTAs co-resident, one per SM), template dispatch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "mpp41_internal.h"
#include "mpp41_mlp_tok.cuh"

namespace mpp41 {
namespace tok {

size_t sync_words(uint32_t T, uint32_t H, uint32_t splits)
{
    const size_t n_mt = (T + kBM - 1) / kBM;
    return 2 + (size_t)(H / kFBN) * n_mt + splits * n_mt;
}

size_t ws_bytes(uint32_t T, uint32_t H, uint32_t splits) { return (size_t)splits * ((T + kBM - 1) / kBM) * kBM * H * 4; }

// Enough CTAs to cover the SMs; each split keeps >= 256 of K; the fp16 output
// always reduces through the workspace (at least 2 splits).
uint32_t splits(uint32_t T, uint32_t H, uint32_t I, bool out_f16)
{
    const uint32_t tiles = (H / kFBN) * ((T + kBM - 1) / kBM);
    uint32_t s = 1;
    while (tiles * s * 2 <= 160 && (I % (kFBK * s * 2)) == 0 && I / (s * 2) >= 256) s *= 2;
    return (out_f16 && s == 1) ? 2 : s;
}

template <int W, int EG, bool F16>
static int launch_ft(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    using Cfg = FusedCfg<W>;
    FusedParams p;
    memset(&p, 0, sizeof(p));
    p.T = L.T; p.H = L.H; p.I = L.I; p.splits = L.splits;
    p.kbc_g = L.H / 32;
    p.kbc_d = L.I / L.splits / 32;
    if (W == W_MXFP4 && (p.kbc_g % 16 || p.kbc_g > 256 || p.kbc_d % 16 || p.kbc_d > 256)) {
        *why = "scale tiles need (H/32) and (I/splits/32) multiples of 16 and at most 256";
        return 1;
    }
    p.n_gtiles = (L.I / 32) * ((L.T + kBM - 1) / kBM);
    p.n_dtiles = (L.H / kFBN) * L.splits * ((L.T + kBM - 1) / kBM);
    const uint32_t kbc_max = p.kbc_g > p.kbc_d ? p.kbc_g : p.kbc_d;
    const uint32_t smem = Cfg::smem_bytes(kbc_max, kMaxStagesA);
    if (smem > 227u * 1024u) { *why = "shared memory"; return 1; }
    const uint64_t rawH = (uint64_t)L.H * wfmt_bits(W) / 8, rawI = (uint64_t)L.I * wfmt_bits(W) / 8;
    if (rawH < (uint64_t)kChunkRow || rawI < (uint64_t)kChunkRow) { *why = "packed rows shorter than one chunk"; return 1; }
    bool ok = make_map(&p.tm_x, L.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.H, L.T, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map(&p.tm_mid, L.mid, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.I, L.T, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map(&p.tm_wg, L.wg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawH, L.I, kChunkRow, 32, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              make_map(&p.tm_wu, L.wu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawH, L.I, kChunkRow, 32, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              make_map(&p.tm_wd, L.wd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawI, L.H, kChunkRow, kFBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (ok && W == W_MXFP4)
        ok = make_map(&p.tm_sg, L.sg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.H / 32, L.I, p.kbc_g, 32, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_su, L.su, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.H / 32, L.I, p.kbc_g, 32, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_sd, L.sd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.I / 32, L.H, p.kbc_d, kFBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) { *why = "tensor maps (16-byte aligned bases and row pitches needed)"; return 1; }
    p.mid = static_cast<__half *>(L.mid);
    p.out = L.out;
    p.ws = L.ws;
    p.sync = L.sync;
    p.err = L.err;
    p.trace = L.trace;

    auto kern = mlp_fused_kernel<W, EG, F16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFThreads, smem);
    if (e != cudaSuccess || per_sm < 1) { cudaGetLastError(); *why = "occupancy"; return 2; }
    const uint32_t ntiles = p.n_gtiles + p.n_dtiles;
    uint32_t grid = (uint32_t)(sms * per_sm);
    if (grid > ntiles) grid = ntiles;
    // tiles go to CTAs round-robin, down tiles last: with no more down tiles
    // than CTAs each CTA holds at most one and it is its final tile
    p.d_spin = p.n_dtiles <= grid ? 1u : 0u;

    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    // Programmatic stream serialization: the grid may launch while the previous
    // kernel finishes; its grid-wide waits all follow griddepcontrol.wait, when
    // every CTA (at most one per SM) can be resident.
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    return 0;
}

template <int W>
static int launch_fw(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (L.out_f16) {
        switch (L.gate_epi) {
        case EPI_SWIGLU_HALF: return launch_ft<W, EPI_SWIGLU_HALF, true>(L, st, why);
        case EPI_SWIGLU_HALF_H: return launch_ft<W, EPI_SWIGLU_HALF_H, true>(L, st, why);
        case EPI_SWIGLU_PLAIN: return launch_ft<W, EPI_SWIGLU_PLAIN, true>(L, st, why);
        }
    } else {
        switch (L.gate_epi) {
        case EPI_SWIGLU_HALF: return launch_ft<W, EPI_SWIGLU_HALF, false>(L, st, why);
        case EPI_SWIGLU_HALF_H: return launch_ft<W, EPI_SWIGLU_HALF_H, false>(L, st, why);
        case EPI_SWIGLU_PLAIN: return launch_ft<W, EPI_SWIGLU_PLAIN, false>(L, st, why);
        }
    }
    *why = "epilogue";
    return 1;
}

int launch(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (L.H % kFBN || L.H % kFBK || L.I % (kFBK * L.splits) || L.I % 32) { *why = "shape"; return 1; }
    switch (L.wfmt) {
    case W_I8: return launch_fw<W_I8>(L, st, why);
    case W_I4: return launch_fw<W_I4>(L, st, why);
    case W_I2: return launch_fw<W_I2>(L, st, why);
    case W_FP4: return launch_fw<W_FP4>(L, st, why);
    case W_E4M3: return launch_fw<W_E4M3>(L, st, why);
    case W_E5M2: return launch_fw<W_E5M2>(L, st, why);
    case W_MXFP4: return launch_fw<W_MXFP4>(L, st, why);
    default: *why = "weight format not covered by the fused kernel"; return 1;
    }
}

}  // namespace tok
}  // namespace mpp41
