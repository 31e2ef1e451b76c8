// Internal launch interface shared by the .cu files of libmpp41.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "mpp41.h"

namespace mpp41 {

// Weight formats; values match enum mpp41_wfmt of include/mpp41.h.
enum WFmt : int {
    W_F16 = 0, W_I8 = 1, W_I4 = 2, W_I2 = 3, W_FP4 = 4, W_E4M3 = 5, W_E5M2 = 6, W_MXFP4 = 7,
    W_E4M3_MX = 8, W_E5M2_MX = 9    // FP8 with an E8M0 scale per 32 weights along K (MXFP8)
};

// Formats that carry an E8M0 scale per 32 weights ([rows][k/32]).
__host__ __device__ constexpr bool wfmt_mx(int w) { return w == W_MXFP4 || w == W_E4M3_MX || w == W_E5M2_MX; }

// Bits per packed weight.
__host__ __device__ constexpr int wfmt_bits(int w)
{
    return (w == W_F16) ? 16 : (w == W_I4 || w == W_FP4 || w == W_MXFP4) ? 4 : (w == W_I2) ? 2 : 8;
}

cudaError_t launch_pack(int fmt, const float *in, size_t n, uint8_t *out, cudaStream_t st);
cudaError_t launch_unpack(int fmt, const uint8_t *in, size_t n, float *out, cudaStream_t st);
// Exact operand widening (n elements, n % 8 == 0): kind 0 E2M1 -> fp16,
// 1 int8 -> fp16, 2 INT4 -> int8.
cudaError_t launch_widen(int kind, const void *in, size_t n, void *out, cudaStream_t st);
cudaError_t launch_roundtrip(int fmt, const float *in, uint8_t *packed, float *out, cudaStream_t st);
cudaError_t launch_dequant(int lut, const uint8_t *packed, const uint8_t *scales, void *out, uint32_t rows,
                           uint32_t depth, cudaStream_t st);
cudaError_t launch_swiglu(int kind, const void *gate, const void *up, void *mid, size_t n, cudaStream_t st);
cudaError_t launch_scalar_mlp(int wfmt, uint32_t T, uint32_t H, uint32_t I, const void *x, const void *wg,
                              const void *wu, void *mid, const void *wd, void *out, cudaStream_t st);
cudaError_t launch_scalar_matmul(int kind, uint32_t M, uint32_t N, uint32_t K, const void *a, const void *b, void *c,
                                 cudaStream_t st);

// Quantized-weight tensor-core GEMM (mpp41_wq_gemm.cuh). epi is an Epi
// value; b1/s1 are the up-projection operands of the SwiGLU pair epilogues.
struct WqLaunch {
    int wfmt;
    int epi;
    const void *a;          // fp16 [M][K]
    const void *b0;
    const void *b1;
    const uint8_t *s0;
    const uint8_t *s1;
    void *out;
    uint32_t M, N, K, ldc;
    uint32_t splits;        // split-K factor (EPI_ATOMIC_F32 only)
    uint32_t *err;
    void *zero;             // optional buffer to clear (16-byte aligned)
    size_t zero_bytes;      // multiple of 16
    float *ws;              // split-K fp16 output: fp32 workspace [M][ldc] (clear)
    uint32_t *tile_count;   // split-K fp16 output: per-tile arrival counters (clear)
};

// Integer tensor-core GEMM (mpp41_i8_gemm.cuh): A int8 [M][K] x B (INT8/INT4/
// INT2 [N][K]) -> int32 [M][ldc] (epi 0 store, 1 split-K atomic add into a
// cleared C), or epi 2: gate (b0) / up (b1) pair through mpp_mlp_swiglu_i8 to
// an int8 mid [M][ldc].
struct I8Launch {
    int wfmt, epi;   // epi: 0 int32, 1 int32 split-K add, 2 swiglu_i8 pair, 3 dequant + SwiGLU -> fp16 pair, 4 dequant -> fp16
    const void *a, *b0, *b1;
    void *out;
    const float *row_scale, *col_scale0, *col_scale1;   // epi 3 and 4
    uint32_t M, N, K, ldc, splits;
    uint32_t *err;
};
int launch_i8_gemm(const I8Launch &L, cudaStream_t st, const char **why);

// fp32-activation GEMM (mpp41_f32_gemm.cuh): A fp32 [M][K] x B (half or INT8
// [N][K]) -> fp32 [M][ldc]; splits > 1 adds into a cleared C.
struct F32Launch {
    int wfmt;
    const float *a;
    const void *b;
    float *out;
    uint32_t M, N, K, ldc, splits;
    uint32_t *err;
};
int launch_f32_gemm(const F32Launch &L, cudaStream_t st, const char **why);

// Block-scaled FP4 GEMM (W4A4, kind::mxf4): A [M][K/2] E2M1 + [M][K/32] E8M0
// against B [N][K/2]; with the SwiGLU epilogues b0 holds the gate rows and b1
// the up rows, otherwise b0 == b1. epi 0: fp32 C,
// 1: fp16 C, 2: silu(gate) * up re-quantized to MXFP4 (out = packed mid
// [M][ldc/2], out_scales = [M][ldc/32]), 3: silu(gate) * up as fp16 [M][ldc].
// nv: NVFP4 operands (scales [rows][K/16] UE4M3; C scaled by the tensor scales).
struct MxLaunch {
    const void *a, *sa;
    const void *b0, *sb0, *b1, *sb1;
    uint32_t b_rows;                        // rows of the B maps
    void *out;
    uint8_t *out_scales;
    uint32_t M, N, K, ldc;
    int epi;
    bool nv;                                // NVFP4 operands (UE4M3 per 16 + fp32 tensor scales)
    const float *ts_a, *ts_b0, *ts_b1;      // NVFP4 tensor scales (device)
    uint32_t *amax_out;                     // SWIGLU_F16: atomicMax of |mid| (float bits), or null
    const uint4 *tiles;                     // grouped: {expert, row0, row_end, 0} per row tile (device)
    const uint32_t *n_tiles;                // grouped: number of valid tiles (device)
    uint32_t max_tiles, b_expert_rows;      // grouped: grid bound; B rows per expert
    uint32_t *err;
};
int launch_mxf4_gemm(const MxLaunch &L, cudaStream_t st, const char **why);

// Mixture-of-experts pieces (mpp41_moe.cu).
cudaError_t launch_moe_route(const float *logits, uint32_t T, uint32_t E, uint32_t k, int32_t *ids, float *weights,
                             cudaStream_t st);
cudaError_t launch_moe_permute(const int32_t *ids, uint32_t n, uint32_t E, uint32_t bm, uint32_t *counts,
                               uint32_t *offsets, uint4 *tiles, uint32_t *n_tiles, uint32_t *perm_src, uint32_t *inv,
                               uint32_t *err, cudaStream_t st);
cudaError_t launch_moe_gather(const void *src, uint32_t row_bytes, const uint32_t *perm_src, uint32_t k,
                              const uint32_t *n_rows, uint32_t max_rows, void *dst, cudaStream_t st);
cudaError_t launch_moe_ep_plan(const uint32_t *allc, uint32_t P, uint32_t E, uint32_t rank, uint32_t bm, uint4 *segs,
                               uint4 *tiles, uint32_t *n_tiles, cudaStream_t st);
cudaError_t launch_moe_segments(const void *src, void *dst, uint32_t row_bytes, const uint4 *segs, uint32_t nsegs,
                                bool to_recv, cudaStream_t st);
cudaError_t launch_moe_combine(const float *y, const uint32_t *inv, const float *w, uint32_t T, uint32_t k, uint32_t H,
                               const float *shared_y, void *out, bool out_f16, cudaStream_t st);

bool make_map(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint32_t elem, uint64_t cols, uint64_t rows,
              uint32_t bc, uint32_t br, CUtensorMapSwizzle sw);
// fp16 [rows][cols] viewed as [cols/64][rows][64]: one copy of box {64, br, nblk}
// lands nblk consecutive 128-byte-swizzled K atoms of br rows each.
bool make_map_kblocks(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t br, uint32_t nblk);
// Packed byte rows [rows][row_bytes] viewed as [row_bytes/128][rows][128 B]: one
// copy of box {128, box_rows, box_chunks} lands box_chunks 128-byte-swizzled
// column chunks of box_rows rows each.
bool make_map_rows128(CUtensorMap *m, const void *base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows,
                      uint32_t box_chunks);

// OCP-MX quantization of fp32 [rows][depth] to E2M1 [rows][depth/2] + E8M0 [rows][depth/32].
cudaError_t launch_quantize_mxfp4(const float *w, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales,
                                  cudaStream_t st);
// Activation quantization (fp16 in): OCP-MX MXFP4, and per-token int8 absmax.
cudaError_t launch_quantize_mxfp4_f16(const void *x, uint32_t rows, uint32_t depth, uint8_t *packed, uint8_t *scales,
                                      cudaStream_t st);
// NVFP4 quantization (fp32 or fp16 in) with a computed tensor scale; amax_tmp
// is one device word of scratch (amax_ready: it already holds the tensor's
// absolute maximum as float bits, so the reduction pass is skipped).
cudaError_t launch_quantize_nvfp4(const void *x, bool f16_in, uint32_t rows, uint32_t depth, uint32_t *amax_tmp,
                                  uint8_t *packed, uint8_t *scales, float *tensor_scale, cudaStream_t st,
                                  bool amax_ready = false);
// Per-row symmetric INT8/INT4/INT2 weights with fp32 row scales.
cudaError_t launch_quantize_int_rows(const float *w, uint32_t rows, uint32_t depth, int bits, uint8_t *packed,
                                     float *scales, cudaStream_t st);
cudaError_t launch_quantize_act_s8(const void *x, uint32_t tokens, uint32_t hidden, int8_t *q, float *scale,
                                   cudaStream_t st);
// Returns 0 on success, 1 for an unsupported combination/shape, 2 for a CUDA error.
int launch_wq_gemm(const WqLaunch &L, cudaStream_t st, const char **why);

// One whole MLP layer as a single persistent cooperative kernel
// (mpp41_mlp_fused.cuh). gate_epi is an Epi SwiGLU value; out_f16 selects fp16
// output through `ws`. sync: device counters, zero on first use, left zero.
struct FusedLaunch {
    int wfmt, gate_epi;
    bool out_f16;
    const void *x, *wg, *wu, *wd;
    const uint8_t *sg, *su, *sd;
    void *mid, *out;
    float *ws;                   // fused_ws_bytes(T, H, splits): fp32 split partials
    uint32_t *sync;
    uint32_t *err;
    uint32_t T, H, I, splits;
    unsigned long long *trace;   // optional per-CTA phase/wait counters (profiling)
    // sg / su / sd are fp16 per-output-row scales (INT weights; small-layer kernel only)
    bool row_scales = false;
    // GEMM only: out[T][H] = mid[T][I] x wd[H][I]^T (down tiles, no split, no
    // gate/up phase); x / wg / wu / sg / su are not read
    bool gemm_only = false;
};
// Number of uint32 sync counters a launch needs.
size_t fused_sync_words(uint32_t T, uint32_t H, uint32_t I);
// Bytes of the fp32 workspace a launch needs (one T x H partial per K split;
// none without splits).
size_t fused_ws_bytes(uint32_t T, uint32_t H, uint32_t splits);
// K splits of the down projection the fused kernel uses for this shape.
uint32_t fused_splits(uint32_t T, uint32_t H, uint32_t I);

// Token-major variant of the fused layer kernel (mpp41_mlp_tok.cuh): same
// launch description, its own workspace layout ([splits][T][H] fp32) and
// counters.
namespace tok {
size_t sync_words(uint32_t T, uint32_t H, uint32_t splits);
size_t ws_bytes(uint32_t T, uint32_t H, uint32_t splits);
uint32_t splits(uint32_t T, uint32_t H, uint32_t I, bool out_f16);
int launch(const FusedLaunch &L, cudaStream_t st, const char **why);
}  // namespace tok

// Small-layer variant of the fused layer kernel (mpp41_mlp_small.cuh): T <= 128,
// H <= 1024, 4-bit weights; one G and one D tile per CTA, the down projection's
// 8 K splits reduced through a workspace of ws_bytes(T, H).
namespace sl {
bool covers(uint32_t T, uint32_t H, uint32_t I, int wfmt);
size_t sync_words(uint32_t T, uint32_t H);
size_t ws_bytes(uint32_t T, uint32_t H);
int launch(const FusedLaunch &L, cudaStream_t st, const char **why);
}  // namespace sl

// Which fused kernel runs a layer, with its K splits and the workspace and
// counter words it needs. Depends on the shape only.
struct LayerPlan {
    bool gemv;          // decode-sized weight-streaming kernel (mpp41_gemv.cuh)
    bool small;         // small-layer kernel (mpp41_mlp_small.cuh)
    bool token_major;
    uint32_t splits;
    size_t ws_bytes, sync_words;
};
LayerPlan plan_layer(uint32_t T, uint32_t H, uint32_t I, bool out_f16, int wfmt);
// Decode-sized layers, 4-bit weights (MXFP4 / FP4 / INT4). T <= 16 with H and
// I multiples of 256 and H * I >= 8M: one persistent weight-streaming kernel (mpp41_gemv.cuh)
// with gv::ws_bytes() of workspace and gv::sync_words(H, I) counters.
namespace gv {
bool covers(uint32_t T, uint32_t H, uint32_t I, int wfmt);
size_t ws_bytes();
size_t sync_words(uint32_t H, uint32_t I);
int launch(const FusedLaunch &L, cudaStream_t st, const char **why);
}  // namespace gv
// T <= 32 otherwise (H and I multiples of 128): two register-fed kernels
// (gate/up + SwiGLU, then down; mpp41_gemv.cu). The mid goes to L.mid; no workspace.
bool gemv_covers(uint32_t T, uint32_t H, uint32_t I, int wfmt);
int launch_gemv_layer(const FusedLaunch &L, cudaStream_t st, const char **why);
// Name of the kernel family launch_layer uses for this plan and shape.
const char *layer_kernel_name(const LayerPlan &plan, uint32_t T, uint32_t H, uint32_t I, int wfmt);
// 0 = launched, 1 = shape/format not covered, 2 = CUDA error.
int launch_layer(const LayerPlan &plan, FusedLaunch L, cudaStream_t st, const char **why);
// 0 = launched, 1 = this shape/format is not covered by the fused kernel, 2 = CUDA error.
int launch_mlp_fused(const FusedLaunch &L, cudaStream_t st, const char **why);

// Multi-GPU state of a context (mpp41_tp.cu); NULL until mpp41_comm_init.
struct CommState;
mpp41_status set_last_error(mpp41_status s, const char *msg);
// Weight format of a GEMM kernel name with fp16 activations, or -1.
int gemm_kernel_wfmt(const char *name);
// Weight handles (mpp41_weight.cu): the map cache of the handle, active on this
// host thread, that owns `base` (nullptr when none); lookups and inserts of
// encoded tensor maps keyed by every encoding argument.
struct WeightMapCache;
WeightMapCache *active_cache_for(const void *base);
bool cache_find(WeightMapCache *c, const uint64_t (&key)[8], CUtensorMap *m);
void cache_put(WeightMapCache *c, const uint64_t (&key)[8], const CUtensorMap &m);
cudaError_t launch_wait_probe(const uint32_t *flag, uint32_t target, uint64_t limit_ns, uint32_t *err,
                              cudaStream_t st);
cudaError_t launch_f32_to_f16(const float *in, size_t n, void *out, cudaStream_t st);

}  // namespace mpp41

// The context: device, stream, device error word, fused-kernel counters.
struct mpp41_ctx {
    int device;
    cudaStream_t own_stream;
    cudaStream_t stream;
    uint32_t *err;          // device error word
    uint32_t *amax;         // one word of scratch for tensor-maximum reductions
    uint32_t *sync;         // grid-wide counters of the fused layer kernel (kept zero between launches)
    size_t sync_words;
    unsigned long long *trace;
    cudaEvent_t ev0, ev1;
    mpp41::CommState *comm = nullptr;
    char last_mlp_kernel[192] = "";     // kernel family of the last enqueued mpp41_mlp layer (+ why a planned kernel declined)
};

namespace mpp41 {
// One-shot all-reduce over peer memory (mpp41_allreduce.cu): data[s] = rank
// s's fp32 partial for this call, flags[s] = rank s's flag slots (one per rank).
constexpr int kMaxPeers = 8;
struct ArPeers {
    const float *data[kMaxPeers];
    uint32_t *flags[kMaxPeers];
};
cudaError_t launch_oneshot_allreduce(const ArPeers &pe, int P, int rank, uint32_t epoch, size_t n, void *out,
                                     bool out_f16, uint32_t *err, cudaStream_t st);
void comm_release(mpp41_ctx *ctx);
int comm_size(const mpp41_ctx *ctx);
int comm_rank(const mpp41_ctx *ctx);
mpp41_status comm_allgather(mpp41_ctx *ctx, const void *send, void *recv, size_t bytes_per_rank);
mpp41_status comm_alltoallv(mpp41_ctx *ctx, const void *send, const size_t *send_bytes, const size_t *send_off,
                            void *recv, const size_t *recv_bytes, const size_t *recv_off);
}  // namespace mpp41
