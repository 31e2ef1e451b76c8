// Host side of the quantized-weight tensor-core GEMM: TMA descriptor
// encoding, template dispatch over (weight format, epilogue) and launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

static bool make_map_encode(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint32_t elem, uint64_t cols,
                            uint64_t rows, uint32_t bc, uint32_t br, CUtensorMapSwizzle sw);

// 2D row-major tensor [rows][cols] of `elem`-byte elements, tile box {bc, br}.
bool make_map(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint32_t elem, uint64_t cols,
                     uint64_t rows, uint32_t bc, uint32_t br, CUtensorMapSwizzle sw)
{
    // a plane of an active weight handle: its map is encoded once and reused
    WeightMapCache *cache = active_cache_for(base);
    const uint64_t key[8] = {1, reinterpret_cast<uintptr_t>(base), (uint64_t)dt, elem, cols, rows,
                             (uint64_t)bc | ((uint64_t)br << 32), (uint64_t)sw};
    if (cache && cache_find(cache, key, m)) return true;
    const bool ok = make_map_encode(m, base, dt, elem, cols, rows, bc, br, sw);
    if (ok && cache) cache_put(cache, key, *m);
    return ok;
}

static bool make_map_encode(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint32_t elem, uint64_t cols,
                            uint64_t rows, uint32_t bc, uint32_t br, CUtensorMapSwizzle sw)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    if ((cols * elem) % 16 != 0) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * elem};
    const cuuint32_t box[2] = {bc, br};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_kblocks(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t br, uint32_t nblk)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || cols % 64 != 0) return false;
    const cuuint64_t dims[3] = {64, rows, cols / 64};
    const cuuint64_t strides[2] = {cols * 2, 128};
    const cuuint32_t box[3] = {64, br, nblk};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_rows128(CUtensorMap *m, const void *base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows,
                      uint32_t box_chunks)
{
    WeightMapCache *cache = active_cache_for(base);
    const uint64_t key[8] = {2, reinterpret_cast<uintptr_t>(base), row_bytes, rows, box_rows, box_chunks, 0, 0};
    if (cache && cache_find(cache, key, m)) return true;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || row_bytes % 128 != 0) return false;
    const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
    const cuuint64_t strides[2] = {row_bytes, 128};
    const cuuint32_t box[3] = {128, box_rows, box_chunks};
    const cuuint32_t es[3] = {1, 1, 1};
    const bool ok = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    if (ok && cache) cache_put(cache, key, *m);
    return ok;
}

template <int W, int BN, int E>
static int launch_t(const WqLaunch &L, cudaStream_t st, const char **why)
{
    using Cfg = WqCfg<W, BN, E>;
    WqGemmParams p;
    memset(&p, 0, sizeof(p));
    const uint32_t splits = (E == EPI_ATOMIC_F32 || E == EPI_SPLITK_F16) ? (L.splits ? L.splits : 1) : 1;
    if (E == EPI_SPLITK_F16 && (!L.ws || !L.tile_count)) { *why = "split-K fp16 output needs a workspace"; return 1; }
    if (L.K % (kBK * splits) != 0) { *why = "K must be a multiple of 64 * split"; return 1; }
    if (L.N % Cfg::kCols != 0) { *why = "N must be a multiple of the CTA column tile"; return 1; }
    const uint32_t kps = L.K / splits;
    if (!make_map(&p.tmap_a, L.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.K, L.M, kBK, kBM,
                  CU_TENSOR_MAP_SWIZZLE_128B)) {
        *why = "activation tensor map (needs 16-byte aligned base, K % 8 == 0)";
        return 1;
    }
    const uint32_t rows_box = Cfg::kPair ? BN / 2 : BN;
    const void *bs[2] = {L.b0, L.b1};
    CUtensorMap *maps[2] = {&p.tmap_b0, &p.tmap_b1};
    for (int i = 0; i < (Cfg::kPair ? 2 : 1); ++i) {
        bool ok;
        if (Cfg::kDirect)
            ok = make_map(maps[i], bs[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.K, L.N, kBK, rows_box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
        else
            ok = make_map(maps[i], bs[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.K * wfmt_bits(W) / 8, L.N,
                          Cfg::kRawRow, rows_box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (!ok) { *why = "weight tensor map (needs 16-byte aligned base and row pitch)"; return 1; }
    }
    p.scales0 = L.s0;
    p.scales1 = L.s1;
    p.out = L.out;
    p.M = L.M; p.N = L.N; p.K = L.K;
    p.k_per_split = kps;
    p.ldc = L.ldc;
    p.err = L.err;
    p.ws = L.ws;
    p.tile_count = L.tile_count;
    p.zero = static_cast<float4 *>(L.zero);
    p.zero_vec4 = (uint32_t)(L.zero_bytes / 16);
    if (L.zero && ((reinterpret_cast<uintptr_t>(L.zero) & 15u) || (L.zero_bytes & 15u))) {
        *why = "buffer to clear must be 16-byte aligned and sized";
        return 1;
    }
    const uint32_t smem = Cfg::smem_bytes(kps);
    if (smem > 227u * 1024u) { *why = "K range per CTA too large for shared memory"; return 1; }
    // opt in to the dynamic shared memory this launch needs (idempotent, cheap)
    cudaError_t e = cudaFuncSetAttribute(wq_gemm_kernel<W, BN, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *why = cudaGetErrorString(e);
        return 2;
    }
    const dim3 grid(L.N / Cfg::kCols, (L.M + kBM - 1) / kBM, splits);
    wq_gemm_kernel<W, BN, E><<<grid, kThreads, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) { *why = cudaGetErrorString(e); return 2; }
    return 0;
}

template <int W>
static int launch_w(const WqLaunch &L, cudaStream_t st, const char **why)
{
    switch (L.epi) {
    case EPI_STORE_F32: return launch_t<W, 64, EPI_STORE_F32>(L, st, why);
    case EPI_STORE_F16: return launch_t<W, 64, EPI_STORE_F16>(L, st, why);
    case EPI_ATOMIC_F32: return launch_t<W, 64, EPI_ATOMIC_F32>(L, st, why);
    case EPI_SWIGLU_FLOAT: return launch_t<W, 64, EPI_SWIGLU_FLOAT>(L, st, why);
    case EPI_SWIGLU_HALF: return launch_t<W, 64, EPI_SWIGLU_HALF>(L, st, why);
    case EPI_SWIGLU_HALF_H: return launch_t<W, 64, EPI_SWIGLU_HALF_H>(L, st, why);
    case EPI_SWIGLU_PLAIN: return launch_t<W, 64, EPI_SWIGLU_PLAIN>(L, st, why);
    case EPI_SPLITK_F16: return launch_t<W, 64, EPI_SPLITK_F16>(L, st, why);
    default: *why = "unknown epilogue"; return 1;
    }
}

int launch_wq_gemm(const WqLaunch &L, cudaStream_t st, const char **why)
{
    switch (L.wfmt) {
    case W_F16: return launch_w<W_F16>(L, st, why);
    case W_I8: return launch_w<W_I8>(L, st, why);
    case W_I4: return launch_w<W_I4>(L, st, why);
    case W_I2: return launch_w<W_I2>(L, st, why);
    case W_FP4: return launch_w<W_FP4>(L, st, why);
    case W_E4M3: return launch_w<W_E4M3>(L, st, why);
    case W_E5M2: return launch_w<W_E5M2>(L, st, why);
    case W_MXFP4: return launch_w<W_MXFP4>(L, st, why);
    default: *why = "unknown weight format"; return 1;
    }
}

}  // namespace mpp41
