// Host side of the block-scaled FP4 (kind::mxf4 / kind::mxf4nvf4) GEMM: tensor maps, shape
// checks and the launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mpp41_internal.h"
#include "mpp41_mxf4_gemm.cuh"
#include "mpp41_mxf4_persist.cuh"

namespace mpp41 {

int launch_mxf4_gemm(const MxLaunch &L, cudaStream_t st, const char **why)
{
    using namespace mxf4;
    // scale rows of K/32 (MXFP4) or K/16 (NVFP4) bytes must be whole 16-byte units
    if (L.K % (L.nv ? 256 : 512)) { *why = L.nv ? "K must be a multiple of 256" : "K must be a multiple of 512"; return 1; }
    if (L.nv && (!L.ts_a || !L.ts_b0 || !L.ts_b1)) { *why = "NVFP4 needs the tensor scales"; return 1; }
    if (L.N % 32) { *why = "N must be a multiple of 32"; return 1; }
    const bool swiglu = L.epi == EPI_SWIGLU_MX || L.epi == EPI_SWIGLU_F16;
    if (swiglu && L.N % 128) { *why = "intermediate must be a multiple of 128"; return 1; }
    if (!swiglu && L.b0 != L.b1) { *why = "two B matrices only with the SwiGLU epilogues"; return 1; }
    if (L.epi != EPI_SWIGLU_MX && L.ldc % (L.epi == EPI_F32 ? 4 : 8)) { *why = "ldc must keep 16-byte rows"; return 1; }
    // Weight-streaming launches (grouped, or at most 128 rows) run the
    // persistent 128 x 128 kernel; larger ones the 128 x 256 tile kernel, one
    // CTA per tile. The B rows of column tile t: SwiGLU epilogues take BN/2
    // gate rows (b0) and BN/2 up rows (b1) at t * BN/2; otherwise b0 == b1 is
    // one matrix and the tile's two halves start at t * BN and t * BN + BN/2.
    const bool persistent = L.tiles || L.M <= 128;
    const int BN = persistent ? 128 : 256;
    Params p;
    memset(&p, 0, sizeof(p));
    p.out = L.out;
    p.out_scales = L.out_scales;
    p.M = L.M; p.N = L.N; p.K = L.K; p.ldc = L.ldc;
    p.b0_row0 = 0;
    p.b1_row0 = swiglu ? 0u : (uint32_t)BN / 2;
    p.b_row_step = swiglu ? (uint32_t)BN / 2 : (uint32_t)BN;
    p.ts_a = L.ts_a; p.ts_b0 = L.ts_b0; p.ts_b1 = L.ts_b1;
    p.amax_out = L.amax_out;
    p.tiles = L.tiles; p.n_tiles = L.n_tiles; p.b_expert_rows = L.b_expert_rows;
    p.err = L.err;
    const uint32_t sf_cols = L.K / (L.nv ? 16 : 32), half = (uint32_t)BN / 2;
    const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const bool ok = make_map(&p.tm_a, L.a, u8, 1, L.K / 2, L.M, 128, kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_b0, L.b0, u8, 1, L.K / 2, L.b_rows, 128, half, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_b1, L.b1, u8, 1, L.K / 2, L.b_rows, 128, half, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_sa, L.sa, u8, 1, sf_cols, L.M, kSfRow, kBM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                    make_map(&p.tm_sb0, L.sb0, u8, 1, sf_cols, L.b_rows, kSfRow, half, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                    make_map(&p.tm_sb1, L.sb1, u8, 1, sf_cols, L.b_rows, kSfRow, half, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) { *why = "tensor maps (16-byte aligned bases needed)"; return 1; }
    void (*kern)(Params) = nullptr;
    uint32_t smem = 0;
#define MXF4_PICK(EPI, NVF)                                                                          \
    if (persistent) { kern = mxf4_persist_kernel<EPI, NVF>; smem = kPSmem; }                         \
    else { kern = mxf4_gemm_kernel<EPI, NVF, 256>; smem = Tile<256>::kSmem; }
    switch (L.epi * 2 + (L.nv ? 1 : 0)) {
    case EPI_F32 * 2: MXF4_PICK(EPI_F32, false) break;
    case EPI_F16 * 2: MXF4_PICK(EPI_F16, false) break;
    case EPI_SWIGLU_MX * 2: MXF4_PICK(EPI_SWIGLU_MX, false) break;
    case EPI_SWIGLU_F16 * 2: MXF4_PICK(EPI_SWIGLU_F16, false) break;
    case EPI_F32 * 2 + 1: MXF4_PICK(EPI_F32, true) break;
    case EPI_F16 * 2 + 1: MXF4_PICK(EPI_F16, true) break;
    case EPI_SWIGLU_F16 * 2 + 1: MXF4_PICK(EPI_SWIGLU_F16, true) break;
    default: *why = "unsupported epilogue for this format"; return 1;
    }
#undef MXF4_PICK
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    const uint32_t cols = swiglu ? half : (uint32_t)BN;
    p.col_tiles = (L.N + cols - 1) / cols;
    if (persistent) {
        static int sms = 0;
        if (!sms && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0) != cudaSuccess) sms = 148;
        // grouped: L.max_tiles row tiles at most (the table's bound); the kernel reads the count
        const uint64_t bound = (uint64_t)(L.tiles ? L.max_tiles : (L.M + kBM - 1) / kBM) * p.col_tiles;
        if (!bound) return 0;
        const uint32_t grid = (uint32_t)(bound < (uint64_t)sms ? bound : (uint64_t)sms);
        kern<<<grid, kPThreads, smem, st>>>(p);
    } else {
        const dim3 grid(p.col_tiles, (L.M + kBM - 1) / kBM);
        if (!grid.y) return 0;
        kern<<<grid, kThreads, smem, st>>>(p);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) { *why = cudaGetErrorString(e); return 2; }
    return 0;
}

}  // namespace mpp41
