// One-shot all-reduce over NVLink peer memory for small tensor-parallel
// partials (no NCCL): every rank's fp32 partial sits in its own buffer that
// the other ranks have mapped (CUDA IPC). Each CTA publishes this call's epoch
// into every rank's flag slot for this rank (a system-scope release after the
// partial was written by the previous kernel on the stream), waits until all
// ranks have published the epoch into its own slots (acquire, bounded by
// kWaitLimitNs; on timeout it reports MPP41_ERR_TIMEOUT and returns), then
// sums the partials of ranks 0..P-1 in that order -- the same order on every
// rank, so all ranks hold identical results -- and writes fp32 or fp16.
// Buffers alternate by epoch parity: a rank rewrites a buffer only after every
// peer has published the following epoch, i.e. finished reading it.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mpp41_device.cuh"
#include "mpp41_internal.h"

namespace mpp41 {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void oneshot_kernel(ArPeers pe, int P, int rank, uint32_t epoch, size_t n, void *out, int out_f16,
                               uint32_t *err)
{
    __shared__ int failed;
    if (threadIdx.x == 0) {
        failed = 0;
        __threadfence_system();
        for (int s = 0; s < P; ++s) st_release_sys(pe.flags[s] + rank, epoch);
        const uint32_t *mine = pe.flags[rank];
        const uint64_t t0 = globaltimer_ns();
        for (int s = 0; s < P && !failed; ++s) {
            while ((int32_t)(ld_acquire_sys(mine + s) - epoch) < 0) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    report_error(err, kErrTimeout, 0xF01);
                    failed = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (failed) return;
    const size_t n4 = n / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 acc = __ldcg(reinterpret_cast<const float4 *>(pe.data[0]) + i);
        for (int s = 1; s < P; ++s) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(pe.data[s]) + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (out_f16) {
            __half2 *o = reinterpret_cast<__half2 *>(out) + 2 * i;
            o[0] = __floats2half2_rn(acc.x, acc.y);
            o[1] = __floats2half2_rn(acc.z, acc.w);
        } else {
            reinterpret_cast<float4 *>(out)[i] = acc;
        }
    }
}

}  // namespace

cudaError_t launch_oneshot_allreduce(const ArPeers &pe, int P, int rank, uint32_t epoch, size_t n, void *out,
                                     bool out_f16, uint32_t *err, cudaStream_t st)
{
    if (!n) return cudaSuccess;
    const size_t n4 = n / 4;
    size_t grid = (n4 + 255) / 256;
    if (grid > 148) grid = 148;   // every CTA resident: each one takes part in the handshake
    oneshot_kernel<<<(unsigned)grid, 256, 0, st>>>(pe, P, rank, epoch, n, out, out_f16 ? 1 : 0, err);
    return cudaGetLastError();
}

}  // namespace mpp41
