// Device-side building blocks for the sm_100a kernels: mbarrier + bulk-async
// copy wrappers (hand-written PTX), bounded waits, warp reductions and the
// nibble/byte -> fp16 conversions used by the fused-dequant decode loop.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace lik {


constexpr unsigned kFull = 0xffffffffu;

// Bounded waits: a kernel never spins forever. After this many failed
// try_wait polls it records LIK device error 1 and bails out.
constexpr uint32_t kMaxPolls = 1u << 24;

// Device error word values (workspace offset 0). kDevBadBlock: a paged block
// table entry outside [0, num_blocks); the tile was masked, nothing read.
enum DeviceError : int { kDevOk = 0, kDevWaitTimeout = 1, kDevBadBlock = 2 };

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for phase `parity` of `bar` to complete, polling at most kMaxPolls
// times. Returns false on timeout (the caller records the error and leaves).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_polls = kMaxPolls) {
    // rolled: an unrolled poll loop costs kilobytes of code at every wait site
#pragma unroll 1
    for (uint32_t i = 0; i < max_polls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// 1-D bulk async copy global -> shared (no tensor map, no multicast),
// completion signalled on `bar` as transaction bytes. dst, src 16-byte
// aligned; bytes a multiple of 16. L2 policy: evict-first (the KV stream is
// read once per step).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// GPU-scope acquire-release fence (cumulative: covers the warp's writes
// ordered before it by __syncwarp).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// atom.add with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ unsigned atomic_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Programmatic dependent launch (sm_90+): wait until the grids this one
// depends on have completed and their memory is visible / allow the next
// grid on the stream to be scheduled.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 2^x with the hardware approximation (MUFU.EX2); ex2(-inf) = 0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ half2 as_h2(uint32_t u) {
    return *reinterpret_cast<half2*>(&u);
}
__device__ __forceinline__ uint32_t as_u32(half2 h) {
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---- code -> fp16 conversions (exact for the small integer ranges) -------
//
// fp16 with exponent field 0x19 (the bit pattern 0x6400) has unit spacing on
// [1024, 2048): OR-ing an 8-bit integer into its low mantissa bits gives
// 1024 + n exactly, and one packed subtract recovers n. A nibble placed in
// bits 4..7 gives 1024 + 16 n, recovered with a packed fma by 1/16.

// Four signed int8 codes (one 32-bit word) -> two half2: (b0, b1), (b2, b3).
__device__ __forceinline__ void i8x4_to_h2(uint32_t w, half2& lo, half2& hi) {
    const uint32_t x = w ^ 0x80808080u;  // two's complement -> offset binary (b + 128)
    const uint32_t a = __byte_perm(x, 0x64646464u, 0x4140);
    const uint32_t b = __byte_perm(x, 0x64646464u, 0x4342);
    const half2 bias = as_h2(0x64806480u);  // 1152 = 1024 + 128
    lo = __hsub2(as_h2(a), bias);
    hi = __hsub2(as_h2(b), bias);
}

// Four signed int8 codes -> two half2 holding 1152 + code (exact; the caller
// removes the offset): (b0, b1), (b2, b3).
__device__ __forceinline__ void i8x4_to_h2_offset(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t x = w ^ 0x80808080u;
    lo = __byte_perm(x, 0x64646464u, 0x4140);
    hi = __byte_perm(x, 0x64646464u, 0x4342);
}

// Eight packed nibbles (one word: byte i = channel 2i low nibble, 2i+1 high)
// -> four half2 holding channels (0,4), (1,5), (2,6), (3,7).
// SIGNED: two's complement nibbles in [-8, 7]; otherwise unsigned 0..15.
template <bool SIGNED>
__device__ __forceinline__ void i4x8_to_h2(uint32_t w, half2 (&o)[4]) {
    constexpr uint32_t LO_X = SIGNED ? 0x64086408u : 0x64006400u;
    constexpr uint32_t HI_X = SIGNED ? 0x64806480u : 0x64006400u;
    const half2 lo_bias = as_h2(SIGNED ? 0x64086408u : 0x64006400u);   // 1032 or 1024
    const half2 hi_mul = as_h2(0x2c002c00u);                          // 1/16
    const half2 hi_bias = as_h2(SIGNED ? 0xd480d480u : 0xd400d400u);  // -72 or -64
    const uint32_t w8 = w >> 8;
    uint32_t t0, t1, t2, t3;
    if (SIGNED) {
        t0 = (w & 0x000F000Fu) ^ LO_X;
        t1 = (w & 0x00F000F0u) ^ HI_X;
        t2 = (w8 & 0x000F000Fu) ^ LO_X;
        t3 = (w8 & 0x00F000F0u) ^ HI_X;
    } else {
        t0 = (w & 0x000F000Fu) | LO_X;
        t1 = (w & 0x00F000F0u) | HI_X;
        t2 = (w8 & 0x000F000Fu) | LO_X;
        t3 = (w8 & 0x00F000F0u) | HI_X;
    }
    o[0] = __hsub2(as_h2(t0), lo_bias);
    o[1] = __hfma2(as_h2(t1), hi_mul, hi_bias);
    o[2] = __hsub2(as_h2(t2), lo_bias);
    o[3] = __hfma2(as_h2(t3), hi_mul, hi_bias);
}

}  // namespace lik

namespace lik {

// ---- mixed-precision FMA (sm_100): d = a(f16) * b(f16) + c(f32) ----------
// The f16 x f16 product is exact in f32, so only the f32 accumulation rounds.

// acc += a.lo * b.lo + a.hi * b.hi   (a, b: packed half2)
__device__ __forceinline__ float fma_h2_dot(uint32_t a, uint32_t b, float acc) {
    asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
        : "+f"(acc)
        : "r"(a), "r"(b));
    return acc;
}

// (lo, hi) += s * (b.lo, b.hi)   (s: one f16 in the low half of a register)
__device__ __forceinline__ void fma_s_h2(uint16_t s, uint32_t b, float& lo, float& hi) {
    asm("{\n\t.reg .f16 bl, bh;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, %2, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, %2, bh, %1;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "h"(s), "r"(b));
}

}  // namespace lik

namespace lik {

// lo += a.lo * b.lo ; hi += a.hi * b.hi   (two independent accumulation chains)
__device__ __forceinline__ void fma_h2_2acc(uint32_t a, uint32_t b, float& lo, float& hi) {
    asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
        : "+f"(lo), "+f"(hi)
        : "r"(a), "r"(b));
}

}  // namespace lik

namespace lik {

// (lo, hi) += p * (v.lo, v.hi), p = half SEL (0: low, 1: high) of the packed
// register pp. The half is selected inside the asm, so no extraction op.
template <int SEL>
__device__ __forceinline__ void fma_p_h2(uint32_t pp, uint32_t v, float& lo, float& hi) {
    if (SEL == 0) {
        asm("{\n\t.reg .f16 p0, p1, vl, vh;\n\t"
            "mov.b32 {p0, p1}, %2;\n\t"
            "mov.b32 {vl, vh}, %3;\n\t"
            "fma.rn.f32.f16 %0, p0, vl, %0;\n\t"
            "fma.rn.f32.f16 %1, p0, vh, %1;\n\t}"
            : "+f"(lo), "+f"(hi)
            : "r"(pp), "r"(v));
    } else {
        asm("{\n\t.reg .f16 p0, p1, vl, vh;\n\t"
            "mov.b32 {p0, p1}, %2;\n\t"
            "mov.b32 {vl, vh}, %3;\n\t"
            "fma.rn.f32.f16 %0, p1, vl, %0;\n\t"
            "fma.rn.f32.f16 %1, p1, vh, %1;\n\t}"
            : "+f"(lo), "+f"(hi)
            : "r"(pp), "r"(v));
    }
}

}  // namespace lik
