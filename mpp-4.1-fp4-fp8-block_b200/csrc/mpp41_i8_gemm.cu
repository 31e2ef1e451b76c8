// Host side of the integer (kind::i8) GEMM: tensor maps, grid, template dispatch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "mpp41_i8_gemm.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace i8 {

template <int W, int E>
static int launch_t(const I8Launch &L, cudaStream_t st, const char **why)
{
    using Cf = Cfg<W>;
    constexpr bool kPair = (E == I8_SWIGLU || E == I8_DQ_SWIGLU);
    const uint32_t splits = (E == I8_ATOMIC) ? L.splits : 1;
    if (!splits || L.K % (kBK * splits)) { *why = "K must be a multiple of 128 x splits"; return 1; }
    if (L.N % (kPair ? kBN / 2 : 32)) { *why = "N must be a multiple of 32 (64 for the gate/up pair)"; return 1; }
    Params p;
    memset(&p, 0, sizeof(p));
    p.out = L.out;
    p.row_scale = L.row_scale; p.col_scale0 = L.col_scale0; p.col_scale1 = L.col_scale1;
    if ((E == I8_DQ || E == I8_DQ_SWIGLU) && (!L.row_scale || !L.col_scale0 || (kPair && !L.col_scale1))) {
        *why = "scaled epilogues need the row and column scales";
        return 1;
    }
    p.M = L.M; p.N = L.N; p.K = L.K; p.ldc = L.ldc;
    p.k_per_split = L.K / splits;
    p.err = L.err;
    const uint32_t rows = kPair ? kBN / 2 : kBN;
    bool ok = make_map(&p.tm_a, L.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.K, L.M, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    const void *bs[2] = {L.b0, L.b1};
    CUtensorMap *maps[2] = {&p.tm_b0, &p.tm_b1};
    for (int i = 0; i < (kPair ? 2 : 1) && ok; ++i) {
        if (Cf::kDirect)
            ok = make_map(maps[i], bs[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.K, L.N, kBK, rows, CU_TENSOR_MAP_SWIZZLE_128B);
        else
            ok = make_map(maps[i], bs[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.K * wfmt_bits(W) / 8, L.N,
                          Cf::kRawRow, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (!ok) { *why = "tensor maps (16-byte aligned bases and row pitches needed)"; return 1; }
    auto kern = i8_gemm_kernel<W, E>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::kSmem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    const dim3 grid((L.N + rows - 1) / rows, (L.M + kBM - 1) / kBM, splits);
    kern<<<grid, kThreads, Cf::kSmem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) { *why = cudaGetErrorString(e); return 2; }
    return 0;
}

template <int W>
static int launch_w(const I8Launch &L, cudaStream_t st, const char **why)
{
    switch (L.epi) {
    case I8_STORE: return launch_t<W, I8_STORE>(L, st, why);
    case I8_ATOMIC: return launch_t<W, I8_ATOMIC>(L, st, why);
    case I8_SWIGLU: return launch_t<W, I8_SWIGLU>(L, st, why);
    case I8_DQ_SWIGLU: return launch_t<W, I8_DQ_SWIGLU>(L, st, why);
    case I8_DQ: return launch_t<W, I8_DQ>(L, st, why);
    }
    *why = "epilogue";
    return 1;
}

}  // namespace i8

int launch_i8_gemm(const I8Launch &L, cudaStream_t st, const char **why)
{
    switch (L.wfmt) {
    case W_I8: return i8::launch_w<W_I8>(L, st, why);
    case W_I4: return i8::launch_w<W_I4>(L, st, why);
    case W_I2: return i8::launch_w<W_I2>(L, st, why);
    default: *why = "int8-activation GEMM takes INT8, INT4 or INT2 weights"; return 1;
    }
}

}  // namespace mpp41
