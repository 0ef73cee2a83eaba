// Device-only helpers for the B200 MoE-FFN path (included by kernels.cu alone): half conversions, the
// format tables, inline-PTX wrappers for mbarrier / bulk copies / programmatic dependent launch,
// and the device error word that bounded waits report into.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ggml_tables.inc"
#include "params.h"

namespace moeb {

// ---------------------------------------------------------------- format tables (device copies)
// All device code of the library is one translation unit (kernels.cu includes the kernel
// headers), so these module-scope variables are defined here, once.
// IQ2_S codebook (1024 rows x 8 magnitudes), IQ4_NL levels, IQ2_XXS codebook (256 rows) and sign
// patterns: format constants of ggml's blocks.
__device__ uint64_t g_iq2s_grid[MOE_IQ2S_GRID_ROWS] = MOE_IQ2S_GRID_INIT;
__device__ int8_t g_iq4nl[16] = MOE_IQ4NL_VALUES_INIT;
__device__ uint64_t g_iq2xxs_grid[256] = MOE_IQ2XXS_GRID_INIT;
__device__ uint8_t g_iq2xxs_signs[128] = MOE_IQ2XXS_SIGNS_INIT;
// ggml-cpu's fp16 GELU table (gelu_tanh rounded to f16, indexed by the f16 bit pattern of the
// gate value); filled from the host once per device.
__device__ uint16_t g_gelu_f16[1 << 16];
// Error word: bounded waits that give up OR their code in here and return.
__device__ int32_t g_error;

// ERR_RANGE: a value outside the fp16 range of a tensor-core operand (prefill down input > 65504)
enum : int32_t { ERR_MBAR_TIMEOUT = 1, ERR_BAD_EXPERT = 2, ERR_CAPACITY = 4, ERR_RANGE = 16 };

// ---------------------------------------------------------------- small device helpers
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
// binary32 -> binary16, round to nearest even, in integer arithmetic (the bit pattern is used as a
// table index and as stored block bytes, so it is built explicitly rather than through a half type)
__device__ __forceinline__ uint16_t f2h_rn(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax == 0x7f800000u ? 0x7c00u : (0x7e00u | ((ax >> 13) & 0x1ffu))));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);       // rounds to >= 65520: infinity
    if (ax < 0x38800000u) {                                          // subnormal half (unit 2^-24) or zero
        const uint32_t e = ax >> 23;
        if (e < 102u) return (uint16_t)sign;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t sh = 126u - e;                                // 14..24
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax >> 13) & 0x3ffu);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;         // carries into the exponent as needed
    return (uint16_t)(sign | h);
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
    return (uint16_t)p[0] | ((uint16_t)p[1] << 8);
}
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t *p) {
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// 6-bit scale and min of sub-block j of a Q4_K super-block (get_scale_min_k4, ggml-quants.c:822)
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// byte-wise mask 0xff for each set bit of the low 4 bits of s
__device__ __forceinline__ uint32_t sign_bytes4(uint32_t s) {
    return ((s * 0x00204081u) & 0x01010101u) * 0xffu;
}

// ---------------------------------------------------------------- mbarrier + bulk copy (PTX)
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// one bulk copy global -> shared, completion signalled on `bar` (addresses and size 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records ERR_MBAR_TIMEOUT) if the phase
// did not complete within the iteration limit; each try_wait itself suspends for a
// hardware-chosen interval, so the limit bounds the wait to well under a second.
constexpr uint32_t kWaitLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(&g_error, ERR_MBAR_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------- programmatic dependent launch
// wait: block until the upstream grid has completed and its memory is visible.
// launch_dependents: allow the downstream grid to start its pre-wait prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- rms_norm (Gemma-4 block norms)
// ggml_rms_norm (ggml-cpu/ops.cpp:3813-3820): every square rounded to f32, the squares summed in
// double, mean = sum / n rounded to f32, scale = 1 / sqrt(mean + eps) with the correctly rounded f32
// square root and division. The double sum's order differs from the reference's sequential one;
// the f32 mean is the same unless the two sums straddle an f32 rounding boundary (their difference
// is a few units of 2^-53 relative).
__device__ __forceinline__ double sq_sum4(float4 v) {
    return ((double)__fmul_rn(v.x, v.x) + (double)__fmul_rn(v.y, v.y)) +
           ((double)__fmul_rn(v.z, v.z) + (double)__fmul_rn(v.w, v.w));
}
__device__ __forceinline__ float rms_row_scale(double sumsq, int n, float eps) {
    const float mean = (float)(sumsq / (double)n);
    return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
}
// 1 / sqrtf((float) n_embd) of the router input (gemma4.cpp:400)
__device__ __forceinline__ float router_input_scale(int d) { return __fdiv_rn(1.f, __fsqrt_rn((float)d)); }
// router input (x * s) * c * r and expert input (x * s) * w, each product rounded to f32 as the
// reference's separate rms_norm, scale and mul nodes round them (gemma4.cpp:394-402)
__device__ __forceinline__ float4 router_input4(float4 x, float s, float c, float4 r) {
    return make_float4(__fmul_rn(__fmul_rn(__fmul_rn(x.x, s), c), r.x), __fmul_rn(__fmul_rn(__fmul_rn(x.y, s), c), r.y),
                       __fmul_rn(__fmul_rn(__fmul_rn(x.z, s), c), r.z), __fmul_rn(__fmul_rn(__fmul_rn(x.w, s), c), r.w));
}
__device__ __forceinline__ float4 norm_weight4(float4 x, float s, float4 w) {
    return make_float4(__fmul_rn(__fmul_rn(x.x, s), w.x), __fmul_rn(__fmul_rn(x.y, s), w.y),
                       __fmul_rn(__fmul_rn(x.z, s), w.z), __fmul_rn(__fmul_rn(x.w, s), w.w));
}

}  // namespace moeb
