// Tensor-parallel MLP layer: local fused layer on this rank's slice of the
// intermediate dimension, fp32 partial output, NCCL all-reduce (sum) over the
// ranks. NCCL is resolved with dlopen so that the library loads (and its
// single-GPU entry points work) on hosts without it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "mpp41_internal.h"

namespace mpp41 {

namespace {

struct NcclApi {
    void *lib = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclReduceScatter) reduce_scatter = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

mpp41_status err(mpp41_status s, const char *fmt, const char *detail)
{
    char buf[384];
    snprintf(buf, sizeof(buf), fmt, detail ? detail : "");
    return set_last_error(s, buf);
}

const NcclApi *nccl()
{
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.lib) return &g_nccl;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return nullptr;
    NcclApi a;
    a.lib = h;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.reduce_scatter = reinterpret_cast<decltype(a.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    a.send = reinterpret_cast<decltype(a.send)>(dlsym(h, "ncclSend"));
    a.recv = reinterpret_cast<decltype(a.recv)>(dlsym(h, "ncclRecv"));
    a.group_start = reinterpret_cast<decltype(a.group_start)>(dlsym(h, "ncclGroupStart"));
    a.group_end = reinterpret_cast<decltype(a.group_end)>(dlsym(h, "ncclGroupEnd"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_reduce || !a.error_string ||
        !a.all_gather || !a.reduce_scatter || !a.send || !a.recv || !a.group_start || !a.group_end)
        return nullptr;
    g_nccl = a;
    return &g_nccl;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// The one-shot path, on request (MPP41_TP_ALLREDUCE=oneshot): fp32/fp16
// outputs up to 2 MiB of fp32 partial (T * H * 4; e.g. T <= 128 at H = 4096),
// at most kMaxPeers ranks. On 2 B200s it measured no faster than NCCL for the
// Llama-3-8B layer (89 vs 85 us per layer at T = 1, both dominated by the
// local layer), so NCCL stays the default. Allowed up to 256 MiB it also lost at
// large T (T = 4096: 1171 us against NCCL's 1115): the partial makes one more
// round trip through the shared buffer than NCCL's reduction.
constexpr size_t kOneShotMaxBytes = 2u << 20;

// The layer one rank computes: same shape with the intermediate slice, fp32
// (or int32) output so the partial sums add exactly before the final rounding.
// Intermediate slice [i0, i1) of rank r of P: 512-channel units dealt in order
// (the first I/512 mod P ranks take one more) when I is a multiple of 512 with
// at least P units -- every slice then keeps scale rows of a multiple of 16
// bytes (the fused kernels' TMA needs them; I = 14336 over 8 ranks is 4 x 2048 +
// 4 x 1536 rather than 8 x 1792); otherwise even slices of I/P.
void tp_slice(uint32_t I, int P, int r, uint32_t *i0, uint32_t *i1)
{
    const uint32_t u = I / 512;
    if (I % 512 == 0 && u >= (uint32_t)P) {
        const uint32_t base = u / (uint32_t)P, extra = u % (uint32_t)P;
        auto start = [&](uint32_t q) { return 512u * (q * base + (q < extra ? q : extra)); };
        *i0 = start((uint32_t)r);
        *i1 = start((uint32_t)r + 1);
    } else {
        *i0 = (uint32_t)r * I / (uint32_t)P;
        *i1 = (uint32_t)(r + 1) * I / (uint32_t)P;
    }
}

bool tp_even_slices(uint32_t I, int P) { return !(I % 512 == 0 && I / 512 >= (uint32_t)P); }

mpp41_mlp_desc local_desc(const mpp41_mlp_desc *d, int nranks, int rank)
{
    mpp41_mlp_desc l = *d;
    uint32_t i0, i1;
    tp_slice(d->intermediate, nranks, rank, &i0, &i1);
    l.intermediate = i1 - i0;
    if (l.out_dtype == MPP41_F16) l.out_dtype = MPP41_F32;
    return l;
}

}  // namespace

// Peer-mapped buffer of the one-shot all-reduce: every rank allocates
// [flags: kMaxPeers words, padded to 256 B][partial, parity 0][partial, parity 1]
// and maps the other ranks' allocations through CUDA IPC.
struct SymBuf {
    size_t cap = 0;                      // bytes of one partial
    uint8_t *base[kMaxPeers] = {};       // [rank]: own allocation or the mapped peer one
    uint32_t epoch = 0;
};

// Large-T pipelining: the layer runs in token chunks on the context's stream
// while each finished chunk's all-reduce runs on comm_stream.
constexpr int kMaxTpChunks = 8;

struct CommState {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0;
    SymBuf sym;
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t chunk_ev[kMaxTpChunks] = {};
    cudaEvent_t reduced_ev = nullptr;
};

namespace {
void sym_release(CommState *cs)
{
    for (int s = 0; s < cs->nranks && s < kMaxPeers; ++s) {
        if (!cs->sym.base[s]) continue;
        if (s == cs->rank) cudaFree(cs->sym.base[s]);
        else cudaIpcCloseMemHandle(cs->sym.base[s]);
        cs->sym.base[s] = nullptr;
    }
    cs->sym.cap = 0;
    cs->sym.epoch = 0;
}

// Collective: every rank calls it with the same size (the calls that use it
// are collective with the same layer shape).
mpp41_status sym_ensure(mpp41_ctx *ctx, size_t bytes)
{
    CommState *cs = ctx->comm;
    if (cs->sym.cap >= bytes) return MPP41_OK;
    const int P = cs->nranks;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t *dev = nullptr;
    if (cudaMalloc(&dev, hb * (size_t)(P + 1)) != cudaSuccess) return err(MPP41_ERR_OUT_OF_MEMORY, "handle exchange%s", nullptr);
    // barrier: once this all-gather completes every rank has finished its
    // previous calls, so no peer still reads the buffers about to be freed
    mpp41_status st = comm_allgather(ctx, dev + hb * (size_t)P, dev, hb);
    if (st == MPP41_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess) st = err(MPP41_ERR_CUDA, "barrier%s", nullptr);
    if (st != MPP41_OK) {
        cudaFree(dev);
        return st;
    }
    sym_release(cs);
    const size_t cap = (bytes + 255) & ~size_t(255);
    uint8_t *mine = nullptr;
    cudaIpcMemHandle_t h;
    if (cudaMalloc(&mine, 256 + 2 * cap) != cudaSuccess) {
        cudaFree(dev);
        return err(MPP41_ERR_OUT_OF_MEMORY, "peer buffer%s", nullptr);
    }
    // flags zero before any peer can map the buffer
    if (cudaMemset(mine, 0, 256) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
        cudaIpcGetMemHandle(&h, mine) != cudaSuccess ||
        cudaMemcpy(dev + hb * (size_t)P, &h, hb, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(mine);
        cudaFree(dev);
        return err(MPP41_ERR_CUDA, "peer buffer setup%s", nullptr);
    }
    st = comm_allgather(ctx, dev + hb * (size_t)P, dev, hb);
    std::vector<cudaIpcMemHandle_t> all((size_t)P);
    if (st == MPP41_OK && (cudaStreamSynchronize(ctx->stream) != cudaSuccess ||
                           cudaMemcpy(all.data(), dev, hb * (size_t)P, cudaMemcpyDeviceToHost) != cudaSuccess))
        st = err(MPP41_ERR_CUDA, "handle exchange%s", nullptr);
    cudaFree(dev);
    if (st != MPP41_OK) {
        cudaFree(mine);
        return st;
    }
    cs->sym.base[cs->rank] = mine;
    for (int s = 0; s < P; ++s) {
        if (s == cs->rank) continue;
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[s], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            sym_release(cs);
            return err(MPP41_ERR_COMM, "cudaIpcOpenMemHandle of a peer buffer%s", nullptr);
        }
        cs->sym.base[s] = static_cast<uint8_t *>(ptr);
    }
    cs->sym.cap = cap;
    return MPP41_OK;
}
}  // namespace

namespace {
bool use_oneshot(const CommState *cs, const mpp41_mlp_desc *d, size_t n)
{
    const char *env = getenv("MPP41_TP_ALLREDUCE");
    if (!env || strcmp(env, "oneshot") != 0) return false;
    return cs->nranks > 1 && cs->nranks <= kMaxPeers && d->out_dtype != MPP41_S32 && n % 4 == 0 &&
           n * 4 <= kOneShotMaxBytes;
}
}  // namespace

namespace {
// Token chunks of the NCCL path: one by default -- on 2 B200s the Llama-3-8B
// layer at T=4096 ran 1113 us in one chunk and 1145 us in 4 chunks whose
// all-reduces overlap the next chunk's layer (the smaller layers lose more than
// the overlap hides); MPP41_TP_CHUNKS=N (1..8, dividing T) asks for N chunks.
int tp_chunks(const mpp41_mlp_desc *d)
{
    int c = 1;
    if (const char *env = getenv("MPP41_TP_CHUNKS")) {
        const int v = atoi(env);
        if (v >= 1 && v <= kMaxTpChunks && d->tokens % (uint32_t)v == 0) c = v;
    }
    return c;
}

// fp16 output of at least 4 MB of fp32 partials goes through reduce-scatter +
// fp16 all-gather; MPP41_TP_REDUCE=allreduce asks for the fp32 all-reduce. On 2
// B200s, Llama-3-8B layer: T=4096 1084 us against 1101, T=256 134 against 140;
// below that the two collectives' latency loses (T=128: 100.5 us against 92.4,
// T=16: 50.7 against 42.0).
constexpr size_t kGatherMinElems = (size_t)1 << 20;

bool use_gather_f16(const CommState *cs, const mpp41_mlp_desc *d, size_t n)
{
    const char *env = getenv("MPP41_TP_REDUCE");
    if (env && strcmp(env, "allreduce") == 0) return false;
    return d->out_dtype == MPP41_F16 && n >= kGatherMinElems && n % (size_t)cs->nranks == 0 &&
           (n / cs->nranks) % 8 == 0;
}

mpp41_status comm_stream_ready(CommState *cs)
{
    if (cs->comm_stream) return MPP41_OK;
    if (cudaStreamCreateWithFlags(&cs->comm_stream, cudaStreamNonBlocking) != cudaSuccess)
        return err(MPP41_ERR_CUDA, "communication stream%s", nullptr);
    for (cudaEvent_t &e : cs->chunk_ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
            return err(MPP41_ERR_CUDA, "chunk events%s", nullptr);
    if (cudaEventCreateWithFlags(&cs->reduced_ev, cudaEventDisableTiming) != cudaSuccess)
        return err(MPP41_ERR_CUDA, "chunk events%s", nullptr);
    return MPP41_OK;
}
}  // namespace

int comm_size(const mpp41_ctx *ctx) { return ctx && ctx->comm ? ctx->comm->nranks : 0; }
int comm_rank(const mpp41_ctx *ctx) { return ctx && ctx->comm ? ctx->comm->rank : -1; }

mpp41_status comm_allgather(mpp41_ctx *ctx, const void *send, void *recv, size_t bytes_per_rank)
{
    const NcclApi *a = nccl();
    if (!a || !ctx->comm) return err(MPP41_ERR_COMM, "no communicator%s", nullptr);
    const ncclResult_t r = a->all_gather(send, recv, bytes_per_rank, ncclUint8, ctx->comm->comm, ctx->stream);
    if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclAllGather: %s", a->error_string(r));
    return MPP41_OK;
}

// Personalised all-to-all in one NCCL group: rank p gets send_bytes[p] bytes
// from send + send_off[p]; recv_bytes[s] bytes from rank s land at recv + recv_off[s].
mpp41_status comm_alltoallv(mpp41_ctx *ctx, const void *send, const size_t *send_bytes, const size_t *send_off,
                            void *recv, const size_t *recv_bytes, const size_t *recv_off)
{
    const NcclApi *a = nccl();
    if (!a || !ctx->comm) return err(MPP41_ERR_COMM, "no communicator%s", nullptr);
    const int P = ctx->comm->nranks;
    ncclResult_t r = a->group_start();
    for (int p = 0; p < P && r == ncclSuccess; ++p) {
        if (send_bytes[p])
            r = a->send(static_cast<const uint8_t *>(send) + send_off[p], send_bytes[p], ncclUint8, p, ctx->comm->comm,
                        ctx->stream);
        if (r == ncclSuccess && recv_bytes[p])
            r = a->recv(static_cast<uint8_t *>(recv) + recv_off[p], recv_bytes[p], ncclUint8, p, ctx->comm->comm,
                        ctx->stream);
    }
    const ncclResult_t r2 = a->group_end();
    if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclSend/ncclRecv: %s", a->error_string(r));
    if (r2 != ncclSuccess) return err(MPP41_ERR_COMM, "ncclGroupEnd: %s", a->error_string(r2));
    return MPP41_OK;
}

void comm_release(mpp41_ctx *ctx)
{
    if (!ctx || !ctx->comm) return;
    sym_release(ctx->comm);
    if (ctx->comm->comm_stream) {
        cudaStreamSynchronize(ctx->comm->comm_stream);
        cudaStreamDestroy(ctx->comm->comm_stream);
        for (cudaEvent_t &e : ctx->comm->chunk_ev)
            if (e) cudaEventDestroy(e);
        cudaEventDestroy(ctx->comm->reduced_ev);
    }
    const NcclApi *a = nccl();
    if (a && ctx->comm->comm) a->comm_destroy(ctx->comm->comm);
    delete ctx->comm;
    ctx->comm = nullptr;
}

}  // namespace mpp41

using namespace mpp41;

extern "C" {

mpp41_status mpp41_comm_unique_id(uint8_t id[MPP41_COMM_ID_BYTES])
{
    if (!id) return err(MPP41_ERR_INVALID_ARGUMENT, "null id%s", nullptr);
    const NcclApi *a = nccl();
    if (!a) return err(MPP41_ERR_COMM, "libnccl.so.2 could not be loaded%s", nullptr);
    ncclUniqueId uid;
    const ncclResult_t r = a->get_unique_id(&uid);
    if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclGetUniqueId: %s", a->error_string(r));
    static_assert(sizeof(uid.internal) == MPP41_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id, uid.internal, MPP41_COMM_ID_BYTES);
    return MPP41_OK;
}

mpp41_status mpp41_comm_init(mpp41_ctx *ctx, int nranks, int rank, const uint8_t id[MPP41_COMM_ID_BYTES])
{
    if (!ctx || !id) return err(MPP41_ERR_INVALID_ARGUMENT, "null context or id%s", nullptr);
    if (nranks < 1 || rank < 0 || rank >= nranks) return err(MPP41_ERR_INVALID_ARGUMENT, "bad rank / nranks%s", nullptr);
    const NcclApi *a = nccl();
    if (!a) return err(MPP41_ERR_COMM, "libnccl.so.2 could not be loaded%s", nullptr);
    comm_release(ctx);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return err(MPP41_ERR_CUDA, "cudaSetDevice%s", nullptr);
    ncclUniqueId uid;
    memcpy(uid.internal, id, MPP41_COMM_ID_BYTES);
    CommState *cs = new CommState();
    const ncclResult_t r = a->comm_init_rank(&cs->comm, nranks, uid, rank);
    if (r != ncclSuccess) {
        delete cs;
        return err(MPP41_ERR_COMM, "ncclCommInitRank: %s", a->error_string(r));
    }
    cs->nranks = nranks;
    cs->rank = rank;
    ctx->comm = cs;
    return MPP41_OK;
}

void mpp41_comm_destroy(mpp41_ctx *ctx) { comm_release(ctx); }

size_t mpp41_mlp_tp_scratch_bytes(const mpp41_mlp_desc *d, int nranks)
{
    if (!d || nranks < 1) return 0;
    if (tp_even_slices(d->intermediate, nranks) && d->intermediate % (uint32_t)nranks) return 0;
    const mpp41_mlp_desc l = local_desc(d, nranks, 0);   // rank 0 holds the largest slice
    size_t b = align256(mpp41_mlp_scratch_bytes(&l));
    if (d->out_dtype == MPP41_F16) b += (size_t)d->tokens * d->hidden * 4;   // fp32 partial
    return b;
}

mpp41_status mpp41_mlp_tp(mpp41_ctx *ctx, const mpp41_mlp_desc *d, const void *x, const void *wg,
                          const void *wu, const void *wd, const uint8_t *sg, const uint8_t *su,
                          const uint8_t *sd, void *scratch, void *out)
{
    if (!ctx || !d) return err(MPP41_ERR_INVALID_ARGUMENT, "null context or descriptor%s", nullptr);
    if (!ctx->comm) return err(MPP41_ERR_COMM, "mpp41_comm_init has not been called on this context%s", nullptr);
    const CommState *cs = ctx->comm;
    if (tp_even_slices(d->intermediate, cs->nranks) && d->intermediate % (uint32_t)(32 * cs->nranks))
        return err(MPP41_ERR_UNSUPPORTED_SHAPE, "intermediate must split into 32-aligned slices per rank%s", nullptr);
    if (d->out_dtype != MPP41_F32 && d->out_dtype != MPP41_F16 && d->out_dtype != MPP41_S32)
        return err(MPP41_ERR_INVALID_ARGUMENT, "tensor-parallel output must be F32, F16 or S32%s", nullptr);
    const mpp41_mlp_desc l = local_desc(d, cs->nranks, cs->rank);
    // the partial follows the largest slice's scratch, as mpp41_mlp_tp_scratch_bytes lays it out
    const mpp41_mlp_desc l0 = local_desc(d, cs->nranks, 0);
    const size_t local_scratch = align256(mpp41_mlp_scratch_bytes(&l0));
    const size_t n = (size_t)d->tokens * d->hidden;
    if (use_oneshot(cs, d, n)) {
        // partial straight into this rank's peer-mapped buffer, then the one-shot reduction
        mpp41_status s = sym_ensure(ctx, n * 4);
        if (s) return s;
        const uint32_t epoch = ++ctx->comm->sym.epoch;
        ArPeers pe{};
        for (int r = 0; r < cs->nranks; ++r) {
            pe.flags[r] = reinterpret_cast<uint32_t *>(cs->sym.base[r]);
            pe.data[r] = reinterpret_cast<const float *>(cs->sym.base[r] + 256 + (epoch & 1u) * cs->sym.cap);
        }
        s = mpp41_mlp(ctx, &l, x, wg, wu, wd, sg, su, sd, scratch, const_cast<float *>(pe.data[cs->rank]));
        if (s) return s;
        const cudaError_t e = launch_oneshot_allreduce(pe, cs->nranks, cs->rank, epoch, n, out,
                                                       d->out_dtype == MPP41_F16, ctx->err, ctx->stream);
        if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "one-shot all-reduce: %s", cudaGetErrorString(e));
        return MPP41_OK;
    }
    void *partial = d->out_dtype == MPP41_F16 ? static_cast<uint8_t *>(scratch) + local_scratch : out;
    const NcclApi *a = nccl();
    const ncclDataType_t dt = d->out_dtype == MPP41_S32 ? ncclInt32 : ncclFloat32;
    const int chunks = tp_chunks(d);
    if (chunks > 1) {
        // token chunks: chunk c's all-reduce (comm_stream) overlaps chunk c+1's layer (ctx stream)
        mpp41_status s = comm_stream_ready(ctx->comm);
        if (s) return s;
        const uint32_t Tc = d->tokens / (uint32_t)chunks;
        const size_t xb = d->afmt == MPP41_A_S8 ? 1 : 2;
        for (int c = 0; c < chunks; ++c) {
            mpp41_mlp_desc lc = l;
            lc.tokens = Tc;
            const size_t row0 = (size_t)c * Tc;
            s = mpp41_mlp(ctx, &lc, static_cast<const uint8_t *>(x) + row0 * d->hidden * xb, wg, wu, wd, sg, su, sd,
                          scratch, static_cast<uint8_t *>(partial) + row0 * d->hidden * 4);
            if (s) return s;
            if (cudaEventRecord(cs->chunk_ev[c], ctx->stream) != cudaSuccess ||
                cudaStreamWaitEvent(cs->comm_stream, cs->chunk_ev[c], 0) != cudaSuccess)
                return err(MPP41_ERR_CUDA, "chunk event%s", nullptr);
            void *pc = static_cast<uint8_t *>(partial) + row0 * d->hidden * 4;
            const ncclResult_t r = a->all_reduce(pc, pc, (size_t)Tc * d->hidden, dt, ncclSum, cs->comm, cs->comm_stream);
            if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclAllReduce: %s", a->error_string(r));
        }
        if (cudaEventRecord(cs->reduced_ev, cs->comm_stream) != cudaSuccess ||
            cudaStreamWaitEvent(ctx->stream, cs->reduced_ev, 0) != cudaSuccess)
            return err(MPP41_ERR_CUDA, "reduction event%s", nullptr);
    } else if (use_gather_f16(cs, d, n)) {
        // fp16 output: reduce-scatter the fp32 partials, round this rank's share to
        // fp16, all-gather the fp16 shares -- the values of an fp32 all-reduce
        // followed by the conversion, with a quarter fewer bytes on the links
        mpp41_status s = mpp41_mlp(ctx, &l, x, wg, wu, wd, sg, su, sd, scratch, partial);
        if (s) return s;
        const size_t share = n / (size_t)cs->nranks;
        float *mine = static_cast<float *>(partial) + (size_t)cs->rank * share;
        ncclResult_t r = a->reduce_scatter(partial, mine, share, ncclFloat32, ncclSum, cs->comm, ctx->stream);
        if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclReduceScatter: %s", a->error_string(r));
        __half *out_mine = static_cast<__half *>(out) + (size_t)cs->rank * share;
        const cudaError_t e = launch_f32_to_f16(mine, share, out_mine, ctx->stream);
        if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "fp16 conversion: %s", cudaGetErrorString(e));
        r = a->all_gather(out_mine, out, share, ncclFloat16, cs->comm, ctx->stream);
        if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclAllGather: %s", a->error_string(r));
        return MPP41_OK;
    } else {
        mpp41_status s = mpp41_mlp(ctx, &l, x, wg, wu, wd, sg, su, sd, scratch, partial);
        if (s) return s;
        const ncclResult_t r = a->all_reduce(partial, partial, n, dt, ncclSum, cs->comm, ctx->stream);
        if (r != ncclSuccess) return err(MPP41_ERR_COMM, "ncclAllReduce: %s", a->error_string(r));
    }
    if (d->out_dtype == MPP41_F16) {
        const cudaError_t e = launch_f32_to_f16(static_cast<const float *>(partial), n, out, ctx->stream);
        if (e != cudaSuccess) return err(MPP41_ERR_CUDA, "fp16 conversion: %s", cudaGetErrorString(e));
    }
    return MPP41_OK;
}

}  // extern "C"
