// Device-side building blocks for the sm_100a kernels of libmpp41:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and the packed-format decoders shared by every kernel.
//
// Every spin-wait here is bounded (wall-clock limit read from %globaltimer).
// A wait that runs out records MPP41_ERR_TIMEOUT plus a site code in the
// context's device error word and returns false, so the kernel can wind
// down and the host reports the failure instead of the GPU hanging.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace mpp41 {

// Device error word layout: low 16 bits = status code, high 16 bits = site.
constexpr uint32_t kErrTimeout = 7;     // matches MPP41_ERR_TIMEOUT
constexpr uint32_t kErrBounds = 8;      // matches MPP41_ERR_BOUNDS
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void report_error(uint32_t *err, uint32_t code, uint32_t site)
{
    if (err) atomicCAS(err, 0u, (site << 16) | code);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe of a phase (acquire semantics when it reports complete).
// Issue it early and consume the result late: its latency then overlaps other work.
__device__ __forceinline__ uint32_t mbar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok;
}

// Bounded wait for the phase with the given parity to complete. Gives up
// after kWaitLimitNs, or early when another role of the CTA has set *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          uint32_t *err, uint32_t site)
{
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((it & 255u) == 0) {
            if (abort && *abort) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                report_error(err, kErrTimeout, site);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until *p >= target (a counter other CTAs bump; read with
// acquire semantics). Gives up after limit_ns, or early when another role of
// the CTA has set *abort; a wait that runs out records MPP41_ERR_TIMEOUT plus
// `site` in *err, sets *abort and returns false.
__device__ __forceinline__ bool wait_flag_ge(const uint32_t *p, uint32_t target, uint64_t limit_ns,
                                             volatile int *abort, uint32_t *err, uint32_t site)
{
    if (ld_acquire_gpu_u32(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        __nanosleep(32);
        if (ld_acquire_gpu_u32(p) >= target) return true;
        if (abort && *abort) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            report_error(err, kErrTimeout, site);
            if (abort) *abort = 1;
            return false;
        }
    }
}

// One lane of the (converged) warp: true in exactly one lane. Issuing
// tcgen05.mma / TMA from a converged warp with the work predicated on this is
// measurably faster than running the issue loop in one divergent lane while the
// other 31 wait elsewhere (43 vs ~70 cycles per M=128 N=64 MMA on B200 when the
// loop also waits on mbarriers).
__device__ __forceinline__ bool elect_one_sync()
{
    uint32_t p;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(p));
    return p != 0;
}

// mbar_wait made by all 32 lanes of a converged warp, with one outcome for
// the warp (a wait that gave up in any lane counts as given up in all), so
// the warp stays converged for the elect.sync that follows.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *err,
                                          uint32_t site)
{
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, err, site));
}

// Programmatic dependent launch: let the next kernel on the stream start its
// prologue now / wait until the previous kernel finished and its writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 2D tiled load, completion counted on an mbarrier (no multicast).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int32_t c0, int32_t c1, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int32_t c0, int32_t c1, int32_t c2,
                                            uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 B, 8-row groups 1024 B apart (SBO), tile
// base 1024-B aligned. Bits: [0,14) addr>>4, [16,30) LBO>>4, [32,46) SBO>>4,
// [46,48) version 1, [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *tile)
{
    const uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16 with fp16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N)
{
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor, kind::i8 with signed A/B, s32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N)
{
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread i gets lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ decoders
// E8M0 scale -> float, as_type<float>(bits << 23) (byte 0 -> +0, 255 -> +inf).
__device__ __forceinline__ float e8m0_to_float(uint32_t b) { return __uint_as_float(b << 23); }

// Two E2M1 nibbles (low nibble -> low half) of byte position j of w into
// an fp16x2 word. The 3 magnitude bits go to fp16 bits [9,12) and the sign
// to bit 15, which yields value * 2^-14 exactly (normal and subnormal
// codes alike); the caller multiplies by 2^14 (folded into the scale).
template <int j>
__device__ __forceinline__ uint32_t e2m1x2_bits(uint32_t lo_nibs, uint32_t hi_nibs)
{
    // lo_nibs = w & 0x0F0F0F0F (even elements), hi_nibs = (w >> 4) & 0x0F0F0F0F
    // byte0 = lo_j, byte2 = hi_j; bytes 1 and 3 are don't-care (masked below)
    const uint32_t h = __byte_perm(lo_nibs, hi_nibs, j | ((4 + j) << 8));
    return ((h & 0x00070007u) << 9) | ((h & 0x00080008u) << 12);
}

// 8 E2M1 values packed in w (element 2i in the low nibble of byte i) to
// 4 fp16x2 words holding value * 2^-14.
__device__ __forceinline__ void e2m1x8_to_half2_scaled14(uint32_t w, uint32_t (&o)[4])
{
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    o[0] = e2m1x2_bits<0>(lo, hi);
    o[1] = e2m1x2_bits<1>(lo, hi);
    o[2] = e2m1x2_bits<2>(lo, hi);
    o[3] = e2m1x2_bits<3>(lo, hi);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b)
{
    __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b)
{
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ uint32_t half2_bits(float lo, float hi)
{
    __half2 r = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&r);
}

}  // namespace mpp41
