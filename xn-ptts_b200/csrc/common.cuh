// Device helpers shared by the ptts_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace ptts {

// Spin limit of every mbarrier wait, in SM clock cycles (about two seconds at 1.9 GHz).
constexpr long long kWaitLimitCycles = 4000000000LL;

__device__ __forceinline__ void set_error(uint32_t* err, uint32_t bit) {
    if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier (shared::cta) -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Whether the phase of `parity` has completed (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `parity` to complete; false after kWaitLimitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
    return true;
}

// ---- 1-D bulk copy (TMA engine, no tensor map, no multicast) -----------------------------

// Global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned), completing
// `bytes` of transaction count on `bar`. L2 policy: evict first (K/V rows are read once).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Kernel timeline: slot s of `stamps` holds four u64 words, each the minimum over the CTAs that
// mark it: [0] global timer at entry, [1] after the wait on the predecessor, [2] and [3] the
// bitwise complements of the timer at the end and at entry (so the minimum is the last end and
// the last entry). The host fills the slots with all-ones before the step. An entry mark also
// records the last entry.
__device__ __forceinline__ void stamp_mark(unsigned long long* stamps, int slot, int field) {
    if (!stamps || slot < 0) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    atomicMin(stamps + 4 * slot + field, field == STAMP_END ? ~t : t);
    if (field == STAMP_ENTRY) atomicMin(stamps + 4 * slot + STAMP_LAST_ENTRY, ~t);
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- the split-KV partition (plan and decode kernels) --------------------------------------
// All attended keys of a decode batch lie end to end (prefix sums); `ctas_in_use` CTAs take
// equal ranges of them, at least kMinKeysPerCta keys each.
constexpr int kMinKeysPerCta = 32;
__device__ __forceinline__ int ctas_in_use(long long total, int grid) {
    const long long g = (total + kMinKeysPerCta - 1) / kMinKeysPerCta;
    return (int)(g < 1 ? 1 : (g > grid ? grid : g));
}
__device__ __forceinline__ long long cta_start(int c, long long total, int g) {
    return (long long)c * total / g;
}
// The CTA whose range holds key p: the largest c with cta_start(c) <= p.
__device__ __forceinline__ int cta_of(long long p, long long total, int g) {
    const long long c = ((p + 1) * g + total - 1) / total - 1;
    return (int)(c < g - 1 ? c : g - 1);
}

// ---- programmatic dependent launch ------------------------------------------------------
// A kernel launched with programmatic stream serialisation may start before its predecessor
// has finished. grid_dep_wait() returns once the predecessor grid has completed and its
// memory is visible (a no-op when the launch had no such attribute); everything read from
// the predecessor comes after it. grid_dep_launch() lets the successor start launching.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- bf16 / packing ----------------------------------------------------------------------

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// f16 pairs for the GEMM operands: values saturate at +-65504 instead of overflowing.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 v = __floats2half2_rn(fminf(fmaxf(lo, -65504.f), 65504.f), fminf(fmaxf(hi, -65504.f), 65504.f));
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float f16lo(uint32_t u) {
    return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu)));
}
__device__ __forceinline__ float f16hi(uint32_t u) {
    return __half2float(__ushort_as_half((unsigned short)(u >> 16)));
}
// Scalar form of split_f16x2: hi = f16(a) (saturated), lo = a - hi, both as floats.
__device__ __forceinline__ void split_f16(float a, float& hi, float& lo) {
    hi = __half2float(__float2half_rn(fminf(fmaxf(a, -65504.f), 65504.f)));
    lo = a - hi;
}

// hi = f16(a), lo = f16(a - hi) for two values: the split every GEMM input is stored in.
__device__ __forceinline__ void split_f16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = pack_f16x2(a, b);
    lo = pack_f16x2(a - f16lo(hi), b - f16hi(hi));
}

// Four int8 weights (one 32-bit word) -> two bf16x2 words, exactly, without int->float
// conversions: with the sign bit flipped, byte u = v + 128 placed under the f32 exponent of 2^23
// reads as 2^23 + u, and subtracting 2^23 + 128 leaves v.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& b01, uint32_t& b23) {
    const uint32_t u = w ^ 0x80808080u;
    const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
    const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
    const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
    const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
    b01 = pack_bf16x2(f0, f1);
    b23 = pack_bf16x2(f2, f3);
}

// Four int8 weights -> two f16x2 words, exactly: with the sign bit flipped, byte u = v + 128
// under the f16 exponent of 1024 reads as 1024 + u; one packed subtract of 1152 leaves v.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& h01, uint32_t& h23) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t p01 = __byte_perm(u, 0x64646464u, 0x5140);
    const uint32_t p23 = __byte_perm(u, 0x64646464u, 0x7362);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const __half2 r01 = __hsub2(*reinterpret_cast<const __half2*>(&p01), bias);
    const __half2 r23 = __hsub2(*reinterpret_cast<const __half2*>(&p23), bias);
    h01 = *reinterpret_cast<const uint32_t*>(&r01);
    h23 = *reinterpret_cast<const uint32_t*>(&r23);
}

template <bool F16>
__device__ __forceinline__ void i8x4_convert(uint32_t w, uint32_t& b01, uint32_t& b23) {
    if (F16) i8x4_to_f16x4(w, b01, b23);
    else i8x4_to_bf16x4(w, b01, b23);
}

// GELU, erf form (transformer.rs's gelu: 0.5 x (1 + erf(x / sqrt 2))), with erf from
// Abramowitz & Stegun, Handbook of Mathematical Functions (1964), formula 7.1.26: for z >= 0,
// erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z), with an
// absolute error of at most 1.5e-7. 1 + erf(z) is 2 - erfc(z) for z >= 0 and erfc(-z) for
// z < 0, so negative inputs lose no digits to cancellation. Branch-free: one reciprocal and one
// exp2 on the MUFU pipe (approximate forms, errors near 2^-22), the rest FMAs.
__device__ __forceinline__ float gelu_erf(float x) {
    const float z = fabsf(x) * 0.70710678118654752f;
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, z, 1.0f)));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * z * z));
    const float poly =
        fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
    const float c = t * poly * e;  // erfc(z)
    return 0.5f * x * (x >= 0.f ? 2.0f - c : c);
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace ptts
