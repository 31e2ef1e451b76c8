// Host side of the persistent fused MLP kernel: tensor maps, cooperative
// launch (all CTAs co-resident, one per SM), template dispatch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "mpp41_internal.h"
#include "mpp41_mlp_fused.cuh"

namespace mpp41 {

uint32_t fused_splits(uint32_t T, uint32_t H, uint32_t I);

static uint32_t fused_nt(uint32_t T) { return T >= (uint32_t)kMaxNT ? (uint32_t)kMaxNT : (T + 15u) & ~15u; }

size_t fused_sync_words(uint32_t T, uint32_t H, uint32_t I)
{
    const uint32_t nt = fused_nt(T), n_mt = (T + nt - 1) / nt;
    return 2 + (size_t)(H / kWRows) * n_mt + (size_t)fused_splits(T, H, I) * n_mt;
}

size_t fused_ws_bytes(uint32_t T, uint32_t H, uint32_t splits)
{
    const uint32_t nt = fused_nt(T);
    return splits > 1 ? (size_t)splits * ((T + nt - 1) / nt) * nt * H * 4 : 0;
}

// K splits of the down projection. Tiles are dealt round-robin to at most
// kAssumedSMs CTAs; each tile costs its K stages plus a fixed overhead (more
// for split tiles, which reduce through the workspace). The split count with
// the smallest busiest-CTA cost wins (fewest splits on ties). Depends on the
// shape only, so the scratch size can be computed without a device.
uint32_t fused_splits(uint32_t T, uint32_t H, uint32_t I)
{
    constexpr uint32_t kAssumedSMs = 148, kTileCost = 6, kSplitCost = 2;
    const uint32_t nt = fused_nt(T), mt = (T + nt - 1) / nt;
    const uint32_t n_g = (I / kGCh) * mt, g_cost = H / kFBK + kTileCost, nh = H / kWRows;
    uint32_t best = 1;
    uint64_t best_cost = ~0ull;
    for (uint32_t s = 1; s <= 32; s *= 2) {
        if (I % (s * kFBK)) break;
        if (s > 1 && (I / s) % 512) break;   // split starts on a 16-byte scale boundary
        const uint32_t n_d = nh * s * mt, d_cost = I / s / kFBK + kTileCost + (s > 1 ? kSplitCost : 0);
        const uint32_t n = n_g + n_d, grid = n < kAssumedSMs ? n : kAssumedSMs;
        uint64_t worst = 0;
        for (uint32_t b = 0; b < grid; ++b) {
            uint64_t c = 0;
            for (uint32_t t = b; t < n; t += grid) c += t < n_g ? g_cost : d_cost;
            if (c > worst) worst = c;
        }
        if (worst < best_cost) { best_cost = worst; best = s; }
    }
    return best;
}

LayerPlan plan_layer(uint32_t T, uint32_t H, uint32_t I, bool out_f16, int wfmt)
{
    constexpr uint32_t kAssumedSMs = 148;
    LayerPlan pl{};
    // Decode-sized layers with 4-bit weights: one persistent weight-streaming kernel.
    if (gv::covers(T, H, I, wfmt)) {
        pl.gemv = true;
        pl.splits = 1;
        pl.ws_bytes = gv::ws_bytes();
        pl.sync_words = gv::sync_words(H, I);
        return pl;
    }
    // Small layers with 4-bit weights: every CTA runs one
    // G and one D tile; the down projection's 8 K splits reduce through L2.
    if (T > 32 && sl::covers(T, H, I, wfmt)) {
        pl.small = true;
        pl.splits = 8;
        pl.ws_bytes = sl::ws_bytes(T, H);
        pl.sync_words = sl::sync_words(T, H);
        return pl;
    }
    // The weight-major kernel gives each CTA one tile: with fewer G tiles than
    // half the SMs (one 128-token tile of a small layer) each phase would
    // leave most SMs idle, so such layers use the token-major kernel, whose
    // CTAs all take a G tile and then a D tile.
    pl.token_major = T > 64 && T <= 128 && H % 64 == 0 && I % 256 == 0 && (I / kGCh) * 2 < kAssumedSMs;
    if (pl.token_major) {
        pl.splits = tok::splits(T, H, I, out_f16);
        pl.ws_bytes = tok::ws_bytes(T, H, pl.splits);
        pl.sync_words = tok::sync_words(T, H, pl.splits);
    } else {
        pl.splits = fused_splits(T, H, I);
        pl.ws_bytes = fused_ws_bytes(T, H, pl.splits);
        pl.sync_words = fused_sync_words(T, H, I);
    }
    return pl;
}

const char *layer_kernel_name(const LayerPlan &plan, uint32_t T, uint32_t H, uint32_t I, int wfmt)
{
    if (plan.gemv) return "gemv";
    if (gemv_covers(T, H, I, wfmt)) return "gemv_regs";
    return plan.small ? "small" : plan.token_major ? "token_major" : "weight_major";
}

int launch_layer(const LayerPlan &plan, FusedLaunch L, cudaStream_t st, const char **why)
{
    // decode-sized batches of 4-bit weights: weight-streaming GEMV kernels
    if (!L.gemm_only && plan.gemv) return gv::launch(L, st, why);
    if (!L.gemm_only && gemv_covers(L.T, L.H, L.I, L.wfmt)) return launch_gemv_layer(L, st, why);
    L.splits = plan.splits;
    if (plan.small) return sl::launch(L, st, why);
    return plan.token_major ? tok::launch(L, st, why) : launch_mlp_fused(L, st, why);
}

template <int W, int EG, bool F16, bool PAIR = false>
static int launch_ft(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    FusedParams p;
    memset(&p, 0, sizeof(p));
    p.T = L.T; p.H = L.H; p.I = L.I; p.splits = L.splits;
    p.NT = fused_nt(L.T);
    const uint32_t mt = (L.T + p.NT - 1) / p.NT;
    if (L.I % (L.splits * kFBK)) { *why = "intermediate not a multiple of splits x 128"; return 1; }
    if (L.gemm_only ? L.splits != 1 : L.splits != fused_splits(L.T, L.H, L.I)) {
        *why = "splits differ from fused_splits (counter layout)";
        return 1;
    }
    const uint64_t rawH = (uint64_t)L.H * wfmt_bits(W) / 8, rawI = (uint64_t)L.I * wfmt_bits(W) / 8;
    if ((!L.gemm_only && rawH < (uint64_t)kChunkRow) || rawI < (uint64_t)kChunkRow) {
        *why = "packed rows shorter than one chunk";
        return 1;
    }
    if (W == W_MXFP4 && ((!L.gemm_only && L.H % 512) || L.I % 512 || (L.splits > 1 && (L.I / L.splits) % 512))) {
        *why = "MXFP4 scale rows need hidden, intermediate and the K split to be multiples of 512";
        return 1;
    }
    if (PAIR && (L.gemm_only || p.NT != (uint32_t)kMaxNT || L.H % (2 * kWRows) || L.I % (2 * kGCh))) {
        *why = "CTA pairs need full 128-token tiles, hidden a multiple of 256 and intermediate of 128";
        return 1;
    }
    // pairs: tile counts are pair tiles (G 128 channels, D 256 outputs)
    p.n_gtiles = L.gemm_only ? 0 : (L.I / (PAIR ? 2 * kGCh : kGCh)) * mt;
    p.n_dtiles = (L.H / (PAIR ? 2 * kWRows : kWRows)) * L.splits * mt;
    p.g_per_slice = L.gemm_only ? 0 : L.I / L.splits / kGCh;
    if (L.splits > 1 && !L.ws) { *why = "workspace"; return 1; }
    // GEMM mode has no gate/up phase: its G maps are built over the down
    // operands only so that they are valid, and are never read
    const void *gx = L.gemm_only ? L.mid : L.x, *gg = L.gemm_only ? L.wd : L.wg, *gu = L.gemm_only ? L.wd : L.wu;
    const uint64_t grow = L.gemm_only ? rawI : rawH;
    const uint32_t gk = L.gemm_only ? L.I : L.H, gn = L.gemm_only ? L.H : L.I;
    const uint32_t nt_box = PAIR ? p.NT / 2 : p.NT;   // tokens each CTA loads per stage
    bool ok = make_map_kblocks(&p.tm_x, gx, gk, L.T, nt_box, 2) && make_map_kblocks(&p.tm_mid, L.mid, L.I, L.T, nt_box, 2) &&
              make_map(&p.tm_wg, gg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, grow, gn, kChunkRow, kGCh, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map(&p.tm_wu, gu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, grow, gn, kChunkRow, kGCh, CU_TENSOR_MAP_SWIZZLE_128B) &&
              make_map(&p.tm_wd, L.wd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rawI, L.H, kChunkRow, kWRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (ok && W == W_MXFP4)
        ok = make_map(&p.tm_sg, L.gemm_only ? L.sd : L.sg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gk / 32, gn, kScRow, kGCh,
                      CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_su, L.gemm_only ? L.sd : L.su, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gk / 32, gn, kScRow, kGCh,
                      CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map(&p.tm_sd, L.sd, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.I / 32, L.H, kScRow, kWRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) { *why = "tensor maps (16-byte aligned bases and row pitches needed)"; return 1; }
    p.mid = static_cast<__half *>(L.mid);
    p.out = L.out;
    p.ws = L.ws;
    p.sync = L.sync;
    p.err = L.err;
    p.trace = L.trace;

    auto kern = mlp_fused_kernel<W, EG, F16, PAIR>;
    const uint32_t smem = kFusedSmem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFThreads, smem);
    if (e != cudaSuccess || per_sm < 1) { cudaGetLastError(); *why = "occupancy"; return 2; }
    const uint32_t ntiles = p.n_gtiles + p.n_dtiles;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    uint32_t grid = (uint32_t)sms;   // one CTA per SM: each holds all 512 TMEM columns
    if (PAIR) {
        // every CTA must be resident (grid-wide waits): as many pairs as fit at once
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr + 1;
        cfg.numAttrs = 1;
        cfg.gridDim = dim3(2);
        // co-resident pairs of this kernel, per device (the query costs a driver call)
        static int cached[64] = {0};
        int clusters = dev < 64 ? cached[dev] : 0;
        if (clusters < 1) {
            e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
            if (e != cudaSuccess || clusters < 1) { cudaGetLastError(); *why = "cluster occupancy"; return 2; }
            if (dev < 64) cached[dev] = clusters;
        }
        grid = 2u * (uint32_t)clusters;
        if (grid > (uint32_t)sms) grid = (uint32_t)sms & ~1u;
        if (grid > 2 * ntiles) grid = 2 * ntiles;
    } else if (grid > ntiles) {
        grid = ntiles;
    }
    // tiles go to CTAs (pairs) round-robin, down tiles last: with no more down
    // tiles than CTAs (pairs) each holds at most one and it is its final tile
    p.d_spin = p.n_dtiles <= (PAIR ? grid / 2 : grid) ? 1u : 0u;
    cfg.gridDim = dim3(grid);
    // Programmatic stream serialization: this grid may launch while the previous
    // kernel on the stream finishes (it only prefetches and decodes weights until
    // griddepcontrol.wait). Every grid-wide wait of this kernel comes after that
    // wait, when the previous grid has exited and all of this grid's CTAs (at
    // most one per SM) can be resident.
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = PAIR ? 2 : 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) { cudaGetLastError(); *why = cudaGetErrorString(e); return 2; }
    return 0;
}

// CTA pairs for MXFP4 layers with full token tiles when MPP41_FUSED_PAIR=1 (opt-in:
// on B200 the pair form measured on par with the single-CTA form).
static bool want_pair(const FusedLaunch &L)
{
    const char *e = getenv("MPP41_FUSED_PAIR");
    if (!e || strcmp(e, "1") != 0) return false;
    return !L.gemm_only && L.T >= (uint32_t)kMaxNT && L.H % (2 * kWRows) == 0 && L.I % (2 * kGCh) == 0;
}

template <int W>
static int launch_fw(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if constexpr (W == W_MXFP4) {
        if (want_pair(L)) {
            switch (L.gate_epi * 2 + (L.out_f16 ? 1 : 0)) {
            case EPI_SWIGLU_HALF * 2 + 1: return launch_ft<W, EPI_SWIGLU_HALF, true, true>(L, st, why);
            case EPI_SWIGLU_HALF_H * 2 + 1: return launch_ft<W, EPI_SWIGLU_HALF_H, true, true>(L, st, why);
            case EPI_SWIGLU_PLAIN * 2 + 1: return launch_ft<W, EPI_SWIGLU_PLAIN, true, true>(L, st, why);
            case EPI_SWIGLU_HALF * 2: return launch_ft<W, EPI_SWIGLU_HALF, false, true>(L, st, why);
            case EPI_SWIGLU_HALF_H * 2: return launch_ft<W, EPI_SWIGLU_HALF_H, false, true>(L, st, why);
            case EPI_SWIGLU_PLAIN * 2: return launch_ft<W, EPI_SWIGLU_PLAIN, false, true>(L, st, why);
            }
        }
    }
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

int launch_mlp_fused(const FusedLaunch &L, cudaStream_t st, const char **why)
{
    if (L.H % kWRows || L.I % kFBK || !L.splits) { *why = "hidden and intermediate must be multiples of 128"; return 1; }
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

}  // namespace mpp41
