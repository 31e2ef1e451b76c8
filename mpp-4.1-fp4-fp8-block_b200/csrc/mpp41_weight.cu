// Weight handles: the counterpart of the reference's host-built multi-plane
// MTLTensor (main.swift:2172-2212 builds one tensor over the packed weights and
// their scale plane, 2254-2262 binds it; MXFP4Kernels.metal:180-226 reads
// through it). Here a handle names a weight's planes once -- packed values and
// scales, format, K x N -- and keeps the TMA descriptors the kernels encode for
// them: the first launch that uses a given box encodes it, every later launch
// through the handle reuses it. The planes stay owned by the caller.
//
// Mechanism: while a handle entry point runs, its handles are active on the
// calling host thread; make_map / make_map_rows128 (mpp41_wq_gemm.cu) consult
// the active handles and serve a plane's map from the owning handle's cache.
// No launcher changes its arguments, and calls without handles do one
// thread-local check.
#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "mpp41_internal.h"

namespace mpp41 {

struct WeightMapCache {
    std::mutex mu;
    std::vector<std::pair<std::array<uint64_t, 8>, CUtensorMap>> maps;
    uint64_t encoded = 0, reused = 0;
};

}  // namespace mpp41

struct mpp41_weight {
    int device;
    int32_t wfmt;
    uint32_t k, n;
    const void *data;
    const uint8_t *scales;
    mutable mpp41::WeightMapCache cache;
};

namespace mpp41 {

static thread_local const mpp41_weight *tls_active[3];
static thread_local int tls_n_active = 0;

// Handles active for the duration of one entry-point call on this thread.
struct ActiveHandles {
    ActiveHandles(const mpp41_weight *a, const mpp41_weight *b, const mpp41_weight *c)
    {
        tls_active[0] = a; tls_active[1] = b; tls_active[2] = c;
        tls_n_active = 3;
    }
    ~ActiveHandles() { tls_n_active = 0; }
};

WeightMapCache *active_cache_for(const void *base)
{
    for (int i = 0; i < tls_n_active; ++i) {
        const mpp41_weight *h = tls_active[i];
        if (h && (base == h->data || (h->scales && base == static_cast<const void *>(h->scales)))) return &h->cache;
    }
    return nullptr;
}

bool cache_find(WeightMapCache *c, const uint64_t (&key)[8], CUtensorMap *m)
{
    std::lock_guard<std::mutex> g(c->mu);
    for (auto &e : c->maps)
        if (std::memcmp(e.first.data(), key, sizeof(key)) == 0) {
            *m = e.second;
            ++c->reused;
            return true;
        }
    return false;
}

void cache_put(WeightMapCache *c, const uint64_t (&key)[8], const CUtensorMap &m)
{
    std::lock_guard<std::mutex> g(c->mu);
    std::array<uint64_t, 8> k;
    std::memcpy(k.data(), key, sizeof(key));
    c->maps.emplace_back(k, m);
    ++c->encoded;
}

static bool formats_match(int32_t a, int32_t b) { return a == b; }

static mpp41_status err(mpp41_status s, const char *fmt, ...)
{
    char msg[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    return set_last_error(s, msg);
}

}  // namespace mpp41

using namespace mpp41;

extern "C" mpp41_status mpp41_weight_create(mpp41_ctx *ctx, int32_t wfmt, const void *data, const uint8_t *scales,
                                            uint32_t k, uint32_t n, mpp41_weight **out)
{
    if (!out) return err(MPP41_ERR_INVALID_ARGUMENT, "null output pointer");
    *out = nullptr;
    if (!ctx) return err(MPP41_ERR_INVALID_ARGUMENT, "null context");
    if (!data || !k || !n) return err(MPP41_ERR_INVALID_ARGUMENT, "weight handle needs data, k and n");
    if (wfmt < MPP41_W_F16 || wfmt > MPP41_W_E5M2_MX)
        return err(MPP41_ERR_INVALID_ARGUMENT, "unknown weight format %d", (int)wfmt);
    if ((wfmt == MPP41_W_MXFP4 || wfmt_mx(wfmt)) && !scales)
        return err(MPP41_ERR_INVALID_ARGUMENT, "block-scaled weights need their scale plane");
    mpp41_weight *w = new (std::nothrow) mpp41_weight();
    if (!w) return err(MPP41_ERR_OUT_OF_MEMORY, "weight handle");
    w->device = ctx->device;
    w->wfmt = wfmt;
    w->k = k;
    w->n = n;
    w->data = data;
    w->scales = scales;
    *out = w;
    return MPP41_OK;
}

extern "C" void mpp41_weight_destroy(mpp41_weight *w) { delete w; }

extern "C" mpp41_status mpp41_weight_map_counts(const mpp41_weight *w, uint64_t *encoded, uint64_t *reused)
{
    if (!w) return err(MPP41_ERR_INVALID_ARGUMENT, "null handle");
    std::lock_guard<std::mutex> g(w->cache.mu);
    if (encoded) *encoded = w->cache.encoded;
    if (reused) *reused = w->cache.reused;
    return MPP41_OK;
}

static mpp41_status check_handle(const mpp41_ctx *ctx, const mpp41_weight *w, int32_t wfmt, uint32_t n, uint32_t k,
                                 const char *what)
{
    if (!w) return err(MPP41_ERR_INVALID_ARGUMENT, "%s: null handle", what);
    if (w->device != ctx->device)
        return err(MPP41_ERR_INVALID_ARGUMENT, "%s: handle made on device %d, context on %d", what,
                              w->device, ctx->device);
    if (!formats_match(w->wfmt, wfmt))
        return err(MPP41_ERR_INVALID_ARGUMENT, "%s: handle format %d, call wants %d", what, (int)w->wfmt,
                              (int)wfmt);
    if (w->n != n || w->k != k)
        return err(MPP41_ERR_INVALID_ARGUMENT, "%s: handle is %u x %u, call wants %u x %u", what, w->n,
                              w->k, n, k);
    return MPP41_OK;
}

extern "C" mpp41_status mpp41_gemm_weight(mpp41_ctx *ctx, const char *kernel_name, const void *a,
                                          const mpp41_weight *w, void *c, uint32_t m)
{
    if (!ctx) return err(MPP41_ERR_INVALID_ARGUMENT, "null context");
    if (!w) return err(MPP41_ERR_INVALID_ARGUMENT, "null handle");
    const int wfmt = gemm_kernel_wfmt(kernel_name);
    if (wfmt < 0) return err(MPP41_ERR_MISSING_KERNEL, "%s: not a GEMM kernel with fp16 activations", kernel_name ? kernel_name : "(null)");
    mpp41_status s = check_handle(ctx, w, wfmt, w->n, w->k, "gemm");
    if (s) return s;
    ActiveHandles active(w, nullptr, nullptr);
    return mpp41_gemm(ctx, kernel_name, a, w->data, c, m, w->n, w->k, w->scales);
}

extern "C" mpp41_status mpp41_mlp_weights(mpp41_ctx *ctx, const mpp41_mlp_desc *desc, const void *x,
                                          const mpp41_weight *wg, const mpp41_weight *wu, const mpp41_weight *wd,
                                          void *scratch, void *out)
{
    if (!ctx) return err(MPP41_ERR_INVALID_ARGUMENT, "null context");
    if (!desc) return err(MPP41_ERR_INVALID_ARGUMENT, "null descriptor");
    mpp41_status s = check_handle(ctx, wg, desc->wfmt, desc->intermediate, desc->hidden, "gate");
    if (!s) s = check_handle(ctx, wu, desc->wfmt, desc->intermediate, desc->hidden, "up");
    if (!s) s = check_handle(ctx, wd, desc->wfmt, desc->hidden, desc->intermediate, "down");
    if (s) return s;
    ActiveHandles active(wg, wu, wd);
    return mpp41_mlp(ctx, desc, x, wg->data, wu->data, wd->data, wg->scales, wu->scales, wd->scales, scratch, out);
}
