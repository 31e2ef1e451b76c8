// mpp41_mlp_noalloc: one MLP layer that allocates no device memory.
//
// Who needs this: callers that may not call cudaMalloc at all -- for example
// code that runs inside a host framework owning every allocation through its
// own pool, or a plugin loaded into a process whose allocator is locked while
// it runs. mpp41_mlp needs a context (mpp41_create allocates its stream,
// error word and counters) and a caller-provided scratch buffer; this entry
// point needs neither. Its scratch (the fp16 mid activations, the fp32
// split-K workspace, the kernel's grid counters and error word) lives in
// file-scope __device__ arrays of fixed size that every GPU loading the
// library holds until the process exits.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/mpp41.h"
#include "mpp41_internal.h"
#include "mpp41_wq_gemm.cuh"

namespace mpp41 {
mpp41_status set_last_error(mpp41_status s, const char *msg);
}

namespace {

constexpr size_t kSyncWords = 4096;
static __device__ __align__(256) unsigned char g_noalloc_scratch[MPP41_NOALLOC_SCRATCH_BYTES];
static __device__ __align__(256) uint32_t g_noalloc_sync[kSyncWords];
static __device__ __align__(256) uint32_t g_noalloc_err[4];

// Device addresses of the arrays above, looked up once per device. In host
// code the array names are only host-side stand-ins; a kernel must be given
// the address cudaGetSymbolAddress returns for the current device.
struct DevPtrs {
    bool ready;
    unsigned char *scratch;
    uint32_t *sync;
    uint32_t *err;
};
constexpr int kMaxDevices = 64;
DevPtrs g_ptrs[kMaxDevices];
std::mutex g_mu;

mpp41_status err(mpp41_status s, const char *fmt, ...)
{
    char buf[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return mpp41::set_last_error(s, buf);
}

mpp41_status setup(int dev, DevPtrs *out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DevPtrs &p = g_ptrs[dev];
    if (!p.ready) {
        cudaDeviceProp prop;
        cudaError_t e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
        if (prop.major != 10 || prop.minor != 0)
            return err(MPP41_ERR_NO_DEVICE, "libmpp41 is built for sm_100a (B200); device is sm_%d%d", prop.major,
                       prop.minor);
        void *a = nullptr, *b = nullptr, *c = nullptr;
        e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&b, g_noalloc_sync);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&c, g_noalloc_err);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return err(MPP41_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        }
        p.scratch = static_cast<unsigned char *>(a);
        p.sync = static_cast<uint32_t *>(b);
        p.err = static_cast<uint32_t *>(c);
        p.ready = true;
    }
    *out = p;
    return MPP41_OK;
}

// Same split rule as mpp41_mlp, so both entry points compute the same layer.
mpp41::LayerPlan noalloc_plan(const mpp41_mlp_desc *d)
{
    return mpp41::plan_layer(d->tokens, d->hidden, d->intermediate, d->out_dtype == MPP41_F16, d->wfmt);
}

}  // namespace

extern "C" size_t mpp41_mlp_noalloc_scratch_bytes(const mpp41_mlp_desc *d)
{
    if (!d) return 0;
    const size_t mid = ((size_t)d->tokens * d->intermediate * 2 + 255) & ~size_t(255);
    return mid + noalloc_plan(d).ws_bytes;
}

extern "C" mpp41_status mpp41_mlp_noalloc(const mpp41_mlp_desc *d, const void *x, const void *wg, const void *wu,
                                          const void *wd, const uint8_t *sg, const uint8_t *su, const uint8_t *sd,
                                          void *out, void *cuda_stream)
{
    using namespace mpp41;
    if (!d) return err(MPP41_ERR_INVALID_ARGUMENT, "null descriptor");
    if (!x || !wg || !wu || !wd || !out) return err(MPP41_ERR_INVALID_ARGUMENT, "null buffer");
    if (!d->tokens || !d->hidden || !d->intermediate) return err(MPP41_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (d->afmt != MPP41_A_F16 || d->wfmt == MPP41_W_F16 || d->wfmt < 0 || d->wfmt > MPP41_W_E5M2_MX)
        return err(MPP41_ERR_MISSING_KERNEL, "mpp41_mlp_noalloc covers fp16 activations with packed weights only");
    if (d->epilogue != MPP41_SWIGLU_HALF && d->epilogue != MPP41_SWIGLU_HALF_FROM_HALF &&
        d->epilogue != MPP41_SWIGLU_FP32)
        return err(MPP41_ERR_MISSING_KERNEL, "mpp41_mlp_noalloc needs an fp16-mid SwiGLU variant");
    if (d->out_dtype != MPP41_F32 && d->out_dtype != MPP41_F16)
        return err(MPP41_ERR_INVALID_ARGUMENT, "output dtype must be F32 or F16");
    const bool scaled = d->wfmt == MPP41_W_E4M3_MX || d->wfmt == MPP41_W_E5M2_MX || (d->flags & MPP41_MLP_ROW_SCALES);
    if ((d->wfmt == MPP41_W_MXFP4 || scaled) && (!sg || !su || !sd))
        return err(MPP41_ERR_INVALID_ARGUMENT, "scaled weights need gate, up and down scales");
    const size_t need = mpp41_mlp_noalloc_scratch_bytes(d);
    if (need > MPP41_NOALLOC_SCRATCH_BYTES)
        return err(MPP41_ERR_UNSUPPORTED_SHAPE,
                   "layer needs %zu bytes of scratch (tokens x intermediate x 2 + splits x tokens x hidden x 4); "
                   "the static scratch of mpp41_mlp_noalloc holds %u bytes -- use mpp41_mlp with a "
                   "caller-allocated buffer",
                   need, (unsigned)MPP41_NOALLOC_SCRATCH_BYTES);
    const LayerPlan plan = noalloc_plan(d);
    if (scaled && !plan.small)
        return err(MPP41_ERR_UNSUPPORTED_SHAPE,
                   "MXFP8 weights and per-row scales run on the small-layer kernel (33..128 tokens, hidden <= 1024)");
    if (plan.sync_words > kSyncWords)
        return err(MPP41_ERR_UNSUPPORTED_SHAPE, "too many output tiles for the static counters");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return err(MPP41_ERR_NO_DEVICE, "no current CUDA device");
    DevPtrs P;
    mpp41_status s = setup(dev, &P);
    if (s) return s;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    // The counters must start at zero. The kernel leaves them zero, but a
    // launch that gave up may not have; clearing them is a memset, not an
    // allocation. The error word is NOT cleared here: it keeps the first
    // device-side error of any call until mpp41_mlp_noalloc_status reads it.
    e = cudaMemsetAsync(P.sync, 0, plan.sync_words * sizeof(uint32_t), st);
    if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "clear counters: %s", cudaGetErrorString(e));

    FusedLaunch L{};
    L.wfmt = d->wfmt;
    L.gate_epi = d->epilogue == MPP41_SWIGLU_HALF ? EPI_SWIGLU_HALF
                                                  : (d->epilogue == MPP41_SWIGLU_FP32 ? EPI_SWIGLU_PLAIN : EPI_SWIGLU_HALF_H);
    L.out_f16 = d->out_dtype == MPP41_F16;
    L.x = x; L.wg = wg; L.wu = wu; L.wd = wd; L.sg = sg; L.su = su; L.sd = sd;
    L.mid = P.scratch;
    L.out = out;
    L.ws = reinterpret_cast<float *>(P.scratch + (((size_t)d->tokens * d->intermediate * 2 + 255) & ~size_t(255)));
    L.sync = P.sync;
    L.err = P.err;
    L.T = d->tokens; L.H = d->hidden; L.I = d->intermediate;
    L.row_scales = (d->flags & MPP41_MLP_ROW_SCALES) != 0;
    const char *why = "";
    const int rc = launch_layer(plan, L, st, &why);
    if (rc == 1) return err(MPP41_ERR_UNSUPPORTED_SHAPE, "mpp41_mlp_noalloc: %s", why);
    if (rc == 2) return err(MPP41_ERR_CUDA, "mpp41_mlp_noalloc: %s", why);
    return MPP41_OK;
}

// Reads (and clears) the device error word the no-alloc kernels report into:
// a bounded wait that ran out or a bounds check that tripped in any call since
// the last read. Synchronizes `cuda_stream` first; the copies go through
// pageable host memory (no allocation).
extern "C" mpp41_status mpp41_mlp_noalloc_status(void *cuda_stream)
{
    using namespace mpp41;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return err(MPP41_ERR_NO_DEVICE, "no current CUDA device");
    DevPtrs P;
    mpp41_status s = setup(dev, &P);
    if (s) return s;
    e = cudaStreamSynchronize(static_cast<cudaStream_t>(cuda_stream));
    if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "stream synchronize: %s", cudaGetErrorString(e));
    uint32_t w = 0;
    e = cudaMemcpy(&w, P.err, sizeof(w), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "read device error word: %s", cudaGetErrorString(e));
    if (!w) return MPP41_OK;
    e = cudaMemset(P.err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "clear device error word: %s", cudaGetErrorString(e));
    const uint32_t code = w & 0xFFFFu, site = w >> 16;
    return err(code == 7 ? MPP41_ERR_TIMEOUT : code == 8 ? MPP41_ERR_BOUNDS : MPP41_ERR_CUDA,
               "mpp41_mlp_noalloc: device-side error code %u at site 0x%x", code, site);
}
