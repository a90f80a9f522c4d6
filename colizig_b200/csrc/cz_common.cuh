// Device-side helpers shared by the colizig B200 kernels: E4M3 decode, the
// router's exp, and thin inline-PTX wrappers for mbarriers, bulk (TMA) copies
// and gpu-scope acquire/release.  sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#define CZ_DEV __device__ __forceinline__

// Result codes (reference convention colizig_cuda.cu:228-284, extended).
enum {
    CZ_OK = 0,
    CZ_EARGS = -1,
    CZ_EALLOC = -2,
    CZ_EH2D = -3,
    CZ_ELAUNCH = -4,
    CZ_ED2H = -5,
    CZ_ENOLAYER = -6,
    CZ_ETIMEOUT = -7,
    CZ_ESHAPE = -8,
    CZ_ENCCL = -9,
};

// Device error-word bits (OR-ed together by any CTA that gives up a wait).
enum : uint32_t {
    CZ_DERR_ROUTER_BARRIER = 1u << 0,
    CZ_DERR_FULL_WAIT = 1u << 1,
    CZ_DERR_EMPTY_WAIT = 1u << 2,
    CZ_DERR_READY_WAIT = 1u << 3,
    CZ_DERR_DRAIN_WAIT = 1u << 4,
    CZ_DERR_SHAPE = 1u << 5,
    CZ_DERR_SEQ_WAIT = 1u << 6,
    CZ_DERR_EP_WAIT = 1u << 7,  // a peer rank's partial sums never arrived
};

// Spin limits: every wait in these kernels is bounded.  With the nanosleep
// back-off below, CZ_SPIN_LIMIT iterations are roughly one to two seconds.
#define CZ_SPIN_LIMIT (1u << 21)

// ---- E4M3 -> f32 --------------------------------------------------------
// The hardware conversion cvt.rn.f16x2.e4m3x2 is exact (every E4M3 value,
// subnormals included, is a normal f16) and f16 -> f32 is exact, so this
// reproduces fp8.zig:40-51 decodeE4M3 bit for bit; 0x7F/0xFF give NaN.
CZ_DEV float2 e4m3x2_to_f32x2(uint16_t two) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(two));
    __half2 h = *reinterpret_cast<__half2*>(&h2);
    return __half22float2(h);
}

// 16 E4M3 bytes (one 16-byte chunk) -> 16 f32, in byte order.
CZ_DEV void decode16(const uint4 q, float* f) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 a = e4m3x2_to_f32x2((uint16_t)(w[k] & 0xffff));
        const float2 b = e4m3x2_to_f32x2((uint16_t)(w[k] >> 16));
        f[4 * k + 0] = a.x;
        f[4 * k + 1] = a.y;
        f[4 * k + 2] = b.x;
        f[4 * k + 3] = b.y;
    }
}

// ---- exp for the router ---------------------------------------------------
// The reference ranks experts on @exp(logit - max) (moe.zig:441-453), so the
// top-k pick depends on the exact f32 value of exp.  This is the reference's
// @exp(f32) restated as a fixed sequence of IEEE double operations: Cody-Waite
// reduction x = k*ln2 + r (LN2_HI has 42 fractional bits, so k*LN2_HI is
// exact), exp(r) by the degree-13 Taylor polynomial (coefficients 1/n!) in
// Horner form with fused multiply-adds, 2^k applied exactly, one final
// rounding to f32.  The result is the correctly rounded f32 exp except in
// vanishingly rare midpoint cases, and it is bit-identical to the CPU oracle,
// which evaluates the same operations.
__device__ __constant__ double cz_inv_fact[14] = {
    0x1.0000000000000p+0, 0x1.0000000000000p+0, 0x1.0000000000000p-1, 0x1.5555555555555p-3,
    0x1.5555555555555p-5, 0x1.1111111111111p-7, 0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
    0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26,
    0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};

__device__ __forceinline__ float cz_expf_inline(float x) {
    if (x != x) return x;
    if (x > 100.0f) return __int_as_float(0x7f800000);
    if (x < -110.0f) return 0.0f;
    const double xd = (double)x;
    // k = round-to-nearest-even(x * log2(e)): adding and removing 1.5*2^52 is an
    // exact RN-even rounding to an integer for |v| < 2^51.
    const double kd = __dadd_rn(__dadd_rn(__dmul_rn(xd, 0x1.71547652b82fep+0), 0x1.8p52), -0x1.8p52);
    double r = __fma_rn(-kd, 0x1.62e42fefa3800p-1, xd);
    r = __fma_rn(-kd, 0x1.ef35793c76730p-45, r);
    double p = cz_inv_fact[13];
#pragma unroll
    for (int n = 12; n >= 0; --n) p = __fma_rn(p, r, cz_inv_fact[n]);
    // * 2^k, exact (|k| < 160, the product stays a normal double)
    const long long k = (long long)kd;
    return __double2float_rn(__dmul_rn(p, __longlong_as_double((k + 1023) << 52)));
}

// Out-of-line copy for call sites where code size matters more than latency.
static __device__ __noinline__ float cz_expf(float x) { return cz_expf_inline(x); }

// activation.zig:8-20 (tolerance-checked path: CUDA's expf).
CZ_DEV float cz_sigmoid(float x) {
    if (x >= 0.0f) {
        const float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    const float z = expf(x);
    return z / (1.0f + z);
}

CZ_DEV float cz_silu(float x) { return x * cz_sigmoid(x); }

// ---- shared-memory addresses & mbarriers ----------------------------------
CZ_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

CZ_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

CZ_DEV void fence_mbarrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

CZ_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

CZ_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

CZ_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

CZ_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false if it gave up, either after
// CZ_SPIN_LIMIT polls or because *abort became non-zero.  The first poll is
// inline (the phase is often complete already); the loop is out of line.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    for (uint32_t it = 0; it < CZ_SPIN_LIMIT; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (it > 64) __nanosleep(it > 4096 ? 512 : 32);
    }
    return false;
}
CZ_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort);
}

// One bulk (TMA, non-tensor) global -> shared copy completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.  No multicast.
CZ_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- gpu-scope flags ---------------------------------------------------
CZ_DEV uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

CZ_DEV uint32_t ld_relaxed_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 8-byte exchange words: one single-copy-atomic access each.
CZ_DEV unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Two consecutive 8-byte words (16-byte aligned); each word is its own
// single-copy-atomic access.
CZ_DEV void ld_relaxed_u64x2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

CZ_DEV void st_relaxed_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

CZ_DEV void red_relaxed_add_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

CZ_DEV void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Exchange words between GPUs (a peer's memory mapped into this process): system
// scope, one single-copy-atomic 8-byte access each.
CZ_DEV void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

CZ_DEV unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Nanoseconds of the GPU's global timer (deadlines of waits on other GPUs).
CZ_DEV uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

CZ_DEV uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

CZ_DEV unsigned long long tag_word(uint32_t tag, float v) {
    return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}

// Prefetch of a tensor map (a __grid_constant__ kernel parameter) into the TMA
// unit's descriptor cache.
CZ_DEV void prefetch_tensormap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}


// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned global address.
CZ_DEV void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

CZ_DEV void red_release_add_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *p >= target (acquire).  Gives up after CZ_SPIN_LIMIT polls, or
// early when *err becomes non-zero (another CTA already gave up).
static __device__ __noinline__ bool wait_geq_bounded(const uint32_t* p, uint32_t target, const uint32_t* err) {
    for (uint32_t it = 0; it < CZ_SPIN_LIMIT; ++it) {
        if (ld_acquire_gpu(p) >= target) return true;
        if ((it & 63) == 63 && ld_relaxed_gpu(err) != 0) return false;
        if (it > 16) __nanosleep(it > 4096 ? 512 : 64);
    }
    return false;
}

// ---- warp reductions ------------------------------------------------------
CZ_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

CZ_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

CZ_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

CZ_DEV uint32_t redux_max_u32(uint32_t v) {
    uint32_t r;
    asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
    return r;
}

CZ_DEV uint32_t redux_min_u32(uint32_t v) {
    uint32_t r;
    asm volatile("redux.sync.min.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
    return r;
}

CZ_DEV float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
