// Host side of the block-scaled FP4 (kind::mxf4 / kind::mxf4nvf4) GEMM: tensor maps, shape
// checks and the launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mpp41_internal.h"
#include "mpp41_mxf4_gemm.cuh"

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
    if (L.epi != EPI_SWIGLU_MX && L.ldc % (L.epi == EPI_F32 ? 4 : 8)) { *why = "ldc must keep 16-byte rows"; return 1; }
    Params p;
    memset(&p, 0, sizeof(p));
    p.out = L.out;
    p.out_scales = L.out_scales;
    p.M = L.M; p.N = L.N; p.K = L.K; p.ldc = L.ldc;
    p.b0_row0 = L.b0_row0; p.b1_row0 = L.b1_row0; p.b_row_step = L.b_row_step;
    p.ts_a = L.ts_a; p.ts_b0 = L.ts_b0; p.ts_b1 = L.ts_b1;
    p.amax_out = L.amax_out;
    p.tiles = L.tiles; p.n_tiles = L.n_tiles; p.b_expert_rows = L.b_expert_rows;
    p.err = L.err;
    const uint32_t sf_cols = L.K / (L.nv ? 16 : 32);
    const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const bool ok = make_map(&p.tm_a, L.a, u8, 1, L.K / 2, L.M, 128, kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_b0, L.b0, u8, 1, L.K / 2, L.b_rows, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_b1, L.b1, u8, 1, L.K / 2, L.b_rows, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&p.tm_sa, L.sa, u8, 1, sf_cols, L.M, kSfRow, kBM, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                    make_map(&p.tm_sb0, L.sb0, u8, 1, sf_cols, L.b_rows, kSfRow, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                    make_map(&p.tm_sb1, L.sb1, u8, 1, sf_cols, L.b_rows, kSfRow, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) { *why = "tensor maps (16-byte aligned bases needed)"; return 1; }
    void (*kern)(Params);
    switch (L.epi * 2 + (L.nv ? 1 : 0)) {
    case EPI_F32 * 2: kern = mxf4_gemm_kernel<EPI_F32, false>; break;
    case EPI_F16 * 2: kern = mxf4_gemm_kernel<EPI_F16, false>; break;
    case EPI_SWIGLU_MX * 2: kern = mxf4_gemm_kernel<EPI_SWIGLU_MX, false>; break;
    case EPI_SWIGLU_F16 * 2: kern = mxf4_gemm_kernel<EPI_SWIGLU_F16, false>; break;
    case EPI_F32 * 2 + 1: kern = mxf4_gemm_kernel<EPI_F32, true>; break;
    case EPI_F16 * 2 + 1: kern = mxf4_gemm_kernel<EPI_F16, true>; break;
    case EPI_SWIGLU_F16 * 2 + 1: kern = mxf4_gemm_kernel<EPI_SWIGLU_F16, true>; break;
    default: *why = "unsupported epilogue for this format"; return 1;
    }
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    const uint32_t cols = swiglu ? 128 : kBN;
    // grouped: L.max_tiles row tiles at most (the table's bound), L.M = all rows
    const dim3 grid((L.N + cols - 1) / cols, L.tiles ? L.max_tiles : (L.M + kBM - 1) / kBM);
    if (!grid.y) return 0;
    kern<<<grid, kThreads, kSmem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) { *why = cudaGetErrorString(e); return 2; }
    return 0;
}

}  // namespace mpp41
