// activation.cuh -- tanh-GELU and SiLU on bf16 data, bit for bit as the reference computes
// them, for the activation kernels and the fused VAE channel norm + SiLU (sm_100a).
#pragma once

#include "common.cuh"

namespace anima {

// gelu.cu:22-31: tanh-GELU with the reference's constants and fma placement.
__device__ __forceinline__ float gelu_tanh_f(float v) {
    const float inner = 0.7978845608028654f * __fmaf_rn(0.044715f * (v * v), v, v);
    const float hv = 0.5f * v;
    return __fmaf_rn(hv, tanhf(inner), hv);
}

// silu.cu:20-21
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// ------------------------------------------- GELU / SiLU: fast path with exact fallback
//
// The reference formulas (tanhf, expf and an IEEE divide per element) cost ~25
// instructions per element, which makes them issue-bound on B200 rather than
// memory-bound. Here each element is first evaluated with hardware approximations
// (ex2.approx, rcp.approx) in a form without cancellation:
//   GELU: x/2 (1 + tanh u) = x * sigma(2u) = x / (1 + 2^(-2u log2 e)),
//   SiLU: x * sigma(x)     = x / (1 + 2^(-x log2 e)),
// and bracketed by an interval [a, b] that provably contains the reference's fp32 result.
// If a and b round to the same bf16 value, that value is the reference's bf16 output;
// otherwise (about 0.1% of N(0,1) inputs, mostly GELU at x < -2.5 where the reference's
// 1 + tanhf(u) cancels) the element takes the reference formula itself. The outputs are
// therefore the reference's bit for bit; the tests check all 65536 bf16 inputs.
//
// Bounds. x sigma_fast carries a relative error below 2^-21 + (1 - sigma) ln2 |dz|: ex2
// and rcp within 2 and 1 ulp (2^-22, 2^-23), three fp32 roundings, and the error dz of the
// exponent argument against the reference's own u or x, which moves 2^z by ln2 |dz|.
// GELU, z = -2u log2 e: z and the reference's u each carry up to four roundings, so
// ln2 |dz| <= |u| 2^-20. The reference's tanhf is within 2 ulp (<= 2^-23 absolute), so its
// fma(x/2, t, x/2) lies within |x| 2^-24 + |r| 2^-24 of x sigma(2u). The interval
// r (1 +- 2^-19) +- |x| 2^-23 holds it: for |u| <= 1.44 the fast error stays below
// 2^-19 - 2^-21 - 2^-24; beyond, sigma(2u) (|u| - 1.44) < 1/16 for u < 0, so the excess is
// covered by the spare |x| 2^-24 of the second term, and for u > 0 the damping does it
// ((1 - sigma(2u)) |u| <= 0.14).
// SiLU, z = -x log2 e: no cancellation; ln2 |dz| <= |x| 2^-23. The reference (expf within
// 2 ulp, the add and the IEEE divide each within half an ulp) stays within 1.5 * 2^-22 of
// x sigma(x) relative; the fast value (the argument's |x| 2^-23, ex2 2 ulp, the add, rcp 1 ulp,
// the product) within 2^-21 + |x| 2^-23. Their sum, 3.5 * 2^-22 + |x| 2^-23 (second-order
// terms ~2^-40), lies inside r +- |r| (2^-20 + |x| 2^-23), which therefore holds the
// reference's result. (An earlier build used 2^-19 for the first term: twice the undecided
// elements, each one a divergent walk of the reference formula.)

__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_fast(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

struct GeluF {
    __device__ static float f(float v) { return gelu_tanh_f(v); }
    // Two elements: both ends of the interval that holds each reference fp32 result.
    __device__ static void fast(float2 v, float2 &a, float2 &b) {
        // -2 log2(e) * u with u = sqrt(2/pi) (x + 0.044715 x^3), the polynomial as gelu.cu:27-28
        // z = x (K + K c x^2) with K = -2 log2(e) * 0.7978845608f and c = 0.044715f: three
        // roundings away from K times the reference's u, as the bound above assumes
        const float2 z = __fmul2_rn(v, __ffma2_rn(__fmul2_rn(v, v), f2(-0x1.26aec2p+1f * 0.044715f), f2(-0x1.26aec2p+1f)));
        const float2 d = __fadd2_rn(make_float2(ex2_fast(z.x), ex2_fast(z.y)), f2(1.0f));
        // x sigma(2u); adding +0 turns -0 into +0 as the reference's fma(-0, -0, -0) does
        const float2 r = __ffma2_rn(v, make_float2(rcp_fast(d.x), rcp_fast(d.y)), f2(0.0f));
        // r and x share a sign, so r c + x e and r c' - x e are the interval's two ends
        const float2 e = __fmul2_rn(v, f2(0x1p-23f));
        a = __ffma2_rn(r, f2(1.0f + 0x1p-19f), e);
        b = __ffma2_rn(r, f2(1.0f - 0x1p-19f), make_float2(-e.x, -e.y));
    }
};

struct SiluF {
    __device__ static float f(float v) { return silu_f(v); }
    __device__ static void fast(float2 v, float2 &a, float2 &b) {
        const float2 z = __fmul2_rn(v, f2(-1.4426950408889634f));  // -log2(e)
        const float2 d = __fadd2_rn(make_float2(ex2_fast(z.x), ex2_fast(z.y)), f2(1.0f));
        const float2 r = __fmul2_rn(v, make_float2(rcp_fast(d.x), rcp_fast(d.y)));
        // r +- r (2^-20 + |x| 2^-23): the rounding of the exponent argument grows with |x|.
        // A zero r (x < -87, where rcp.approx flushes a subnormal 1/d) gives the ends -0
        // and +0, which never pass as decided.
        const float2 ax = make_float2(fabsf(v.x), fabsf(v.y));
        const float2 dl = __fmul2_rn(r, __ffma2_rn(ax, f2(0x1p-23f), f2(0x1p-20f)));
        a = __fadd2_rn(r, dl);
        b = __fadd2_rn(r, make_float2(-dl.x, -dl.y));
    }
};

template <class F>
__device__ __forceinline__ uint32_t exact_bits(uint32_t b) {  // the reference formula on bf16 bits
    const __nv_bfloat16 r = __float2bfloat16_rn(F::f(__uint_as_float(b << 16)));
    return *reinterpret_cast<const uint16_t *>(&r);
}

// One 16-byte chunk: eight bf16 inputs -> eight bf16 outputs equal to bf16(F::f(x)).
template <class F>
__device__ __forceinline__ Vec8 fast_chunk(const Vec8 &v) {
    Vec8 o, alt;
    uint32_t diff = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 a, b;
        F::fast(make_float2(bf_lo(v.w[j]), bf_hi(v.w[j])), a, b);
        o.w[j] = pack_bf2(a.x, a.y);
        alt.w[j] = pack_bf2(b.x, b.y);
        diff |= o.w[j] ^ alt.w[j];
    }
    if (diff) {
        // Rare: elements whose interval holds a bf16 rounding boundary. Each lane walks only
        // its own (usually one), with one inlined copy of the reference formula; words are
        // picked by selects so that nothing is indexed at run time.
        uint32_t miss = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t d = o.w[j] ^ alt.w[j];
            miss |= (d & 0xffffu ? 1u : 0u) << (2 * j) | (d >> 16 ? 1u : 0u) << (2 * j + 1);
        }
        while (miss) {
            const int e = __ffs(miss) - 1;
            miss &= miss - 1;
            const int j = e >> 1;
            const uint32_t w = j == 0 ? v.w[0] : j == 1 ? v.w[1] : j == 2 ? v.w[2] : v.w[3];
            const uint32_t r = exact_bits<F>(e & 1 ? w >> 16 : w & 0xffffu);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (k == j) o.w[k] = e & 1 ? (o.w[k] & 0xffffu) | (r << 16) : (o.w[k] & 0xffff0000u) | r;
        }
    }
    return o;
}

}  // namespace anima
