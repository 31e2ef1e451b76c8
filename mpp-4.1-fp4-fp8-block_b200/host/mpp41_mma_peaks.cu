// mpp41_mma_peaks: measured tcgen05.mma throughput per operand kind on this
// GPU (M=128, N=256, operands in shared memory, one CTA per SM, 2000 x 4
// back-to-back MMAs each). The roofline denominators for the fp16, int8,
// fp8 and fp4 rows: data values do not change the rate, so the operands are a
// constant fill and the block scales of kind::mxf4 are whatever tensor memory
// holds.
#include <cstdio>
#include <cuda_runtime.h>
#include "../csrc/mpp41_device.cuh"
using namespace mpp41;
template <int KIND>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t sfa, uint32_t sfb) {
    if (KIND == 0) asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d), "l"(a), "l"(b), "r"(id) : "memory");
    if (KIND == 1) asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\ttcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d), "l"(a), "l"(b), "r"(id) : "memory");
    if (KIND == 2) asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\ttcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d), "l"(a), "l"(b), "r"(id) : "memory");
    if (KIND == 3) asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\ttcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(sfa), "r"(sfb) : "memory");
}
template <int KIND>
__global__ void __launch_bounds__(128, 1) k(long long *out, int iters) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint8_t *s = (uint8_t *)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
    __shared__ uint32_t slot; __shared__ uint64_t bar;
    for (int i = threadIdx.x; i < (128 + 256) * 128 / 4; i += blockDim.x) ((uint32_t *)s)[i] = 0x22222222u;
    if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_mbar_init(); }
    if (threadIdx.x < 32) { tmem_alloc(&slot, 512); tmem_relinquish(); }
    fence_proxy_async_smem();
    tc_fence_before(); __syncthreads(); tc_fence_after();
    uint32_t tm = slot;
    if (threadIdx.x == 0) {
        const uint64_t ad = smem_desc_sw128(s), bd = smem_desc_sw128(s + 128 * 128);
        uint32_t id;
        if (KIND == 0) id = (1u << 4) | ((256u >> 3) << 17) | ((128u >> 4) << 24);                  // f16 x f16 -> f32
        if (KIND == 1) id = (2u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);   // s8 -> s32
        if (KIND == 2) id = (1u << 4) | (0u << 7) | (0u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);   // e4m3 x e4m3 -> f32
        if (KIND == 3) id = (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24);  // e2m1, UE8M0 scales
        long long c0 = clock64();
        for (int i = 0; i < iters; ++i)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma<KIND>(tm, ad + 2 * kk, bd + 2 * kk, id, tm + 256, tm + 384);
        mma_commit(&bar);
        mbar_wait(&bar, 0, nullptr, nullptr, 0);
        out[blockIdx.x] = clock64() - c0;
    }
    tc_fence_before(); __syncthreads();
    if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc(tm, 512); }
}
template <int KIND> void run(long long *d, const char *name, double macs_per_mma) {
    cudaFuncSetAttribute(k<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, 60000);
    int iters = 2000;
    k<KIND><<<148, 128, 60000>>>(d, iters);
    cudaError_t e = cudaDeviceSynchronize();
    long long h[148]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double c = (double)h[0] / (iters * 4);
    int clk = 0; cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, 0);
    printf("%-34s %.1f cycles/MMA, %6.0f MAC/clk/SM, %.2f PFLOP/s at %.0f MHz x 148 SMs (err %s)\n", name, c,
           macs_per_mma / c, 2.0 * macs_per_mma / c * 148 * clk * 1e3 / 1e15, clk / 1e3, cudaGetErrorString(e));
}
int main() {
    long long *d; cudaMalloc(&d, 148 * 8);
    run<0>(d, "kind::f16   128x256x16", 128.0 * 256 * 16);
    run<1>(d, "kind::i8    128x256x32", 128.0 * 256 * 32);
    run<2>(d, "kind::f8f6f4 e4m3 128x256x32", 128.0 * 256 * 32);
    run<3>(d, "kind::mxf4 block32 128x256x64", 128.0 * 256 * 64);
}
