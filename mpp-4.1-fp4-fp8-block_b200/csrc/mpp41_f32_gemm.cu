// Host side of the fp32-activation (kind::tf32, split-A) GEMM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mpp41_f32_gemm.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace f32 {

template <int W, bool ATOMIC>
static int launch_t(const F32Launch &L, cudaStream_t st, const char **why)
{
    using Cf = Cfg<W>;
    const uint32_t splits = ATOMIC ? L.splits : 1;
    if (!splits || L.K % (kBK * splits)) { *why = "K must be a multiple of 32 x splits"; return 1; }
    if (L.N % 32) { *why = "N must be a multiple of 32"; return 1; }
    Params p;
    memset(&p, 0, sizeof(p));
    p.out = L.out;
    p.M = L.M; p.N = L.N; p.K = L.K; p.ldc = L.ldc;
    p.k_per_split = L.K / splits;
    p.err = L.err;
    const bool ok =
        make_map(&p.tm_a, L.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.K, L.M, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
        make_map(&p.tm_b, L.b, W == W_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                 W == W_F16 ? 2 : 1, L.K, L.N, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) { *why = "tensor maps (16-byte aligned bases and row pitches needed)"; return 1; }
    auto kern = f32_gemm_kernel<W, ATOMIC>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::kSmem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    const dim3 grid((L.N + kBN - 1) / kBN, (L.M + kBM - 1) / kBM, splits);
    kern<<<grid, kThreads, Cf::kSmem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) { *why = cudaGetErrorString(e); return 2; }
    return 0;
}

}  // namespace f32

int launch_f32_gemm(const F32Launch &L, cudaStream_t st, const char **why)
{
    const bool atomic = L.splits > 1;
    switch (L.wfmt) {
    case W_F16: return atomic ? f32::launch_t<W_F16, true>(L, st, why) : f32::launch_t<W_F16, false>(L, st, why);
    case W_I8: return atomic ? f32::launch_t<W_I8, true>(L, st, why) : f32::launch_t<W_I8, false>(L, st, why);
    default: *why = "fp32-activation GEMM takes half or INT8 weights"; return 1;
    }
}

}  // namespace mpp41
