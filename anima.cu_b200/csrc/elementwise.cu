// elementwise.cu -- GELU / SiLU / add / mul / broadcast modulate and gate kernels (sm_100a).
//
// One grid-stride kernel template covers them all: NS streamed bf16 inputs (1 or 2)
// read as 16-byte chunks with L1-bypassing loads, NB broadcast vectors (0..2) indexed by
// column (element % D, read through L1), and an Op that maps fp32 inputs to one fp32
// output. Each thread keeps U chunks per input in flight. The grid is sized to one
// resident wave (SMs x the CTAs that fit on one SM) and loops, so no CTA waits for a second wave.
// Elements past the last full chunk, and every element when a pointer is not 16-byte
// aligned, take a scalar path inside the same launch.
//
// The per-element arithmetic is the reference's own expression for each op (file:line
// at each Op), so results are bit-identical to the reference kernels.
#include "common.cuh"

#include <type_traits>

namespace anima {
namespace {

constexpr int kEwBlock = 256;

// gelu.cu:22-31: tanh-GELU with the reference's constants and fma placement.
__device__ __forceinline__ float gelu_tanh_f(float v) {
    const float inner = 0.7978845608028654f * __fmaf_rn(0.044715f * (v * v), v, v);
    const float hv = 0.5f * v;
    return __fmaf_rn(hv, tanhf(inner), hv);
}

// silu.cu:20-21
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

struct OpGelu {  // gelu.cu:12-34
    static constexpr int NS = 1, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return gelu_tanh_f(s[0]); }
};
struct OpGeluBias {  // gelu.cu:37-64
    static constexpr int NS = 1, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return gelu_tanh_f(s[0] + b[0]);
    }
};
struct OpSilu {  // silu.cu:7-24
    static constexpr int NS = 1, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return silu_f(s[0]); }
};
struct OpSiluBias {  // silu.cu:26-47
    static constexpr int NS = 1, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const { return silu_f(s[0] + b[0]); }
};
struct OpAdd {  // elementwise.cu:37-53
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return s[0] + s[1]; }
};
struct OpMul {  // elementwise.cu:125-141
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return s[0] * s[1]; }
};
struct OpSwiGLU {  // silu.cu:7-24 on gate, rounded to bf16, then elementwise.cu:125-141
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const {
        return bf16_round(silu_f(s[0])) * s[1];
    }
};
struct OpGatedGelu {  // gemma_ops.cu:5-22 (scalar formula; nvcc folds the cubic into an fma)
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const {
        const float g = s[0];
        const float inner = 0.7978845608f * __fmaf_rn(0.044715f * g * g, g, g);
        return (0.5f * g * (1.0f + tanhf(inner))) * s[1];
    }
};
struct OpScaleShift {  // elementwise.cu:216-236: fma(x, 1+scale[d], shift[d])
    static constexpr int NS = 1, NB = 2;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return __fmaf_rn(s[0], 1.0f + b[0], b[1]);
    }
};
struct OpResidualGate {  // elementwise.cu:249-269: fma(y, gate[d], x)
    static constexpr int NS = 2, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return __fmaf_rn(s[1], b[0], s[0]);
    }
};

struct EwArgs {
    const anima_bf16 *s0, *s1;  // streamed inputs
    const anima_bf16 *b0, *b1;  // broadcast vectors [D]
    anima_bf16 *out;
    int64_t n;       // elements to process
    int D;           // broadcast period (elements); 0 when NB == 0
    bool vec;        // 16-byte path usable
};

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}

template <class Op, int U>
__global__ void __launch_bounds__(kEwBlock) ew_kernel(EwArgs a, Op op) {
    pdl_wait();
    constexpr int NS = Op::NS, NB = Op::NB;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;  // elements covered by the vector loop
    if (a.vec) {
        const int64_t nch = a.n >> 3;
        done = nch << 3;
        const uint32_t dch = NB ? (uint32_t)(a.D >> 3) : 1u;
        for (int64_t base = tid; base < nch; base += stride * U) {
            Vec8 in[U][NS > 1 ? 2 : 1];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = base + u * stride;
                if (i < nch) {
                    in[u][0] = ld_stream(a.s0 + i * 8);
                    if constexpr (NS > 1) in[u][NS - 1] = ld_stream(a.s1 + i * 8);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = base + u * stride;
                if (i >= nch) break;
                float f0[8], f1[8], g0[8], g1[8];
                unpack8(in[u][0], f0);
                if constexpr (NS > 1) unpack8(in[u][NS - 1], f1);
                if constexpr (NB > 0) {
                    // column chunk of this chunk; chunk counts stay below 2^32 for any
                    // tensor that fits in memory at 8 elements per chunk x 2 bytes
                    const uint32_t c = (uint32_t)((uint64_t)i % dch);
                    unpack8(ld_cached(a.b0 + (int64_t)c * 8), g0);
                    if constexpr (NB > 1) unpack8(ld_cached(a.b1 + (int64_t)c * 8), g1);
                }
                float r[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float s[2] = {f0[e], NS > 1 ? f1[e] : 0.0f};
                    float b[2] = {NB > 0 ? g0[e] : 0.0f, NB > 1 ? g1[e] : 0.0f};
                    r[e] = op(s, b);
                }
                st_vec(a.out + i * 8, pack8(r));
            }
        }
    }
    pdl_launch();
    // Scalar path: the tail past the last full chunk, or everything when misaligned.
    for (int64_t e = done + tid; e < a.n; e += stride) {
        float s[2] = {ldb(a.s0 + e), NS > 1 ? ldb(a.s1 + e) : 0.0f};
        float b[2] = {0.0f, 0.0f};
        if constexpr (NB > 0) {
            const int64_t d = e % a.D;
            b[0] = ldb(a.b0 + d);
            if constexpr (NB > 1) b[1] = ldb(a.b1 + d);
        }
        *reinterpret_cast<__nv_bfloat16 *>(a.out + e) = __float2bfloat16_rn(op(s, b));
    }
}

template <class Op>
int launch_ew(const EwArgs &a, cudaStream_t stream) {
    if (a.n <= 0) return ANIMA_OK;
    constexpr int U = Op::NS > 1 ? 2 : 4;
    const int64_t work = a.vec ? ((a.n >> 3) + U - 1) / U : a.n;
    int err = ANIMA_OK;
    const unsigned blocks = wave_grid((const void *)ew_kernel<Op, U>, kEwBlock, 0, work, &err);
    if (err) return err;
    launch(ew_kernel<Op, U>, blocks, kEwBlock, 0, stream, a, Op{});
    return launch_status();
}

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
// Bounds. x sigma_fast carries a relative error below 2^-21 + (1 - sigma) |z| 2^-22.4:
// ex2 and rcp near 2^-22 each, three fp32 roundings, and the rounding of the exponent
// argument z (three roundings from the reference's u), which moves 2^z by |z| 2^-22.4
// relative and reaches sigma damped by 1 - sigma.
// GELU, z = -2u log2 e: the reference's tanhf is within 2 ulp (<= 2^-23 absolute), so its
// fma(x/2, t, x/2) lies within |x| 2^-24 + |r| 2^-24 of x sigma(2u). The interval
// r (1 +- 2^-19) +- |x| 2^-23 holds it: the argument term stays below 2^-20 up to |u| = 4,
// and beyond, sigma(2u) < 3e-4 makes it negligible against |x| 2^-24 (u < 0) or the
// damping does (u > 0).
// SiLU, z = -x log2 e: no cancellation; the reference (expf within 2 ulp, an IEEE divide)
// and the fast value each stay within 2^-21 + |x| 2^-24 of x sigma(x), so the interval
// r +- |r| (2^-19 + |x| 2^-23) holds the reference's result.

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
        // r +- r (2^-19 + |x| 2^-23): the rounding of the exponent argument grows with |x|.
        // A zero r (x < -87, where rcp.approx flushes a subnormal 1/d) gives the ends -0
        // and +0, which never pass as decided.
        const float2 ax = make_float2(fabsf(v.x), fabsf(v.y));
        const float2 dl = __fmul2_rn(r, __ffma2_rn(ax, f2(0x1p-23f), f2(0x1p-19f)));
        a = __fadd2_rn(r, dl);
        b = __fadd2_rn(r, make_float2(-dl.x, -dl.y));
    }
};

template <class F>
__device__ __forceinline__ uint32_t exact_bits(uint32_t b) {  // the reference formula on bf16 bits
    const __nv_bfloat16 r = __float2bfloat16_rn(F::f(__uint_as_float(b << 16)));
    return *reinterpret_cast<const uint16_t *>(&r);
}

template <class F>
__device__ __noinline__ uint32_t exact_bf16(uint32_t b) {  // out of line, for the ragged tail
    return exact_bits<F>(b);
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

// U chunks per thread and group, groups grid-strided; the next group's loads are issued
// before the current group is computed, so every thread keeps U 16-byte loads in flight.
template <int U, int NS>
__device__ __forceinline__ void load_group(Vec8 (&in)[U][NS], const EwArgs &a, int64_t base, int64_t stride,
                                           int64_t nch) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i < nch) {
            in[u][0] = ld_stream(a.s0 + i * 8);
            if constexpr (NS > 1) in[u][1] = ld_stream(a.s1 + i * 8);
        }
    }
}

template <class F, int U, int NS>
__device__ __forceinline__ void act_group(const Vec8 (&in)[U][NS], const EwArgs &a, int64_t base, int64_t stride,
                                          int64_t nch) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i >= nch) break;
        Vec8 o = fast_chunk<F>(in[u][0]);
        if constexpr (NS > 1) {  // elementwise.cu:138-140: product of the bf16 silu value and up
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t uw = in[u][1].w[j];
                const float2 p = __fmul2_rn(make_float2(bf_lo(o.w[j]), bf_hi(o.w[j])), make_float2(bf_lo(uw), bf_hi(uw)));
                o.w[j] = pack_bf2(p.x, p.y);
            }
        }
        st_vec(a.out + i * 8, o);
    }
}

// NS = 1: out = F(x). NS = 2 (SwiGLU): out = bf16(F(gate)) * up, as silu_bf16 then mul_bf16.
template <class F, int NS>
__global__ void __launch_bounds__(kEwBlock, NS == 1 ? 4 : 2) fast_act_kernel(EwArgs a) {
    pdl_wait();
    constexpr int U = 4;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nch = a.vec ? a.n >> 3 : 0;
    Vec8 x0[U][NS], x1[U][NS];
    const int64_t step = stride * U;
    load_group<U, NS>(x0, a, tid, stride, nch);
    for (int64_t base = tid; base < nch;) {  // unrolled by two so the buffers alternate without copies
        load_group<U, NS>(x1, a, base + step, stride, nch);
        act_group<F, U, NS>(x0, a, base, stride, nch);
        base += step;
        if (base >= nch) break;
        load_group<U, NS>(x0, a, base + step, stride, nch);
        act_group<F, U, NS>(x1, a, base, stride, nch);
        base += step;
    }
    pdl_launch();
    for (int64_t e = (nch << 3) + tid; e < a.n; e += stride) {
        const uint32_t r = exact_bf16<F>(*reinterpret_cast<const uint16_t *>(a.s0 + e));
        if constexpr (NS == 1) {
            a.out[e] = (anima_bf16)r;
        } else {
            const float up = __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(a.s1 + e));
            *reinterpret_cast<__nv_bfloat16 *>(a.out + e) = __float2bfloat16_rn(__uint_as_float(r << 16) * up);
        }
    }
}

template <class F, int NS>
int launch_fast_act(const EwArgs &a, cudaStream_t stream) {
    if (a.n <= 0) return ANIMA_OK;
    const int64_t work = a.vec ? ((a.n >> 3) + 3) / 4 : a.n;
    int err = ANIMA_OK;
    const unsigned blocks = wave_grid((const void *)fast_act_kernel<F, NS>, kEwBlock, 0, work, &err);
    if (err) return err;
    launch(fast_act_kernel<F, NS>, blocks, kEwBlock, 0, stream, a);
    return launch_status();
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

// Validates and launches a flat op over n elements (n = 2*floor(N/2), as the reference's
// pair loop covers).
template <class Op>
int flat_op(const anima_bf16 *s0, const anima_bf16 *s1, const anima_bf16 *bias, anima_bf16 *out,
            int64_t N, int D, cudaStream_t stream) {
    constexpr int NS = Op::NS, NB = Op::NB;
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (NB > 0 && (D <= 0 || (D & 1))) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = N / 2 * 2;
    if (n == 0) return ANIMA_OK;
    if (!s0 || !out || (NS > 1 && !s1) || (NB > 0 && !bias)) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(s0) || !bf16_ok(out) || (NS > 1 && !bf16_ok(s1)) || (NB > 0 && !bf16_ok(bias)))
        return ANIMA_ERR_MISALIGNED;
    if (n > INT64_MAX / 2) return ANIMA_ERR_TOO_LARGE;
    if (partial_overlap(s0, n * 2, out, n * 2) || (NS > 1 && partial_overlap(s1, n * 2, out, n * 2)))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{s0, NS > 1 ? s1 : nullptr, NB > 0 ? bias : nullptr, nullptr, out, n, NB > 0 ? D : 0, false};
    a.vec = aligned16(s0) && aligned16(out) && (NS < 2 || aligned16(s1)) &&
            (NB == 0 || (aligned16(bias) && D % 8 == 0));
    if constexpr (std::is_same<Op, OpGelu>::value) return launch_fast_act<GeluF, 1>(a, stream);
    if constexpr (std::is_same<Op, OpSilu>::value) return launch_fast_act<SiluF, 1>(a, stream);
    if constexpr (std::is_same<Op, OpSwiGLU>::value) return launch_fast_act<SiluF, 2>(a, stream);
    return launch_ew<Op>(a, stream);
}

// Validates and launches a row-broadcast op over [M, D].
template <class Op>
int bcast_op(const anima_bf16 *x, const anima_bf16 *y, const anima_bf16 *b0, const anima_bf16 *b1,
             anima_bf16 *out, int M, int D, cudaStream_t stream) {
    constexpr int NS = Op::NS, NB = Op::NB;
    if (M < 0 || D <= 0 || (D & 1)) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)M * D;
    if (n == 0) return ANIMA_OK;
    if (!x || !out || (NS > 1 && !y) || !b0 || (NB > 1 && !b1)) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out) || (NS > 1 && !bf16_ok(y)) || !bf16_ok(b0) ||
        (NB > 1 && !bf16_ok(b1)))
        return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(x, n * 2, out, n * 2) || (NS > 1 && partial_overlap(y, n * 2, out, n * 2)))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{x, NS > 1 ? y : nullptr, b0, NB > 1 ? b1 : nullptr, out, n, D, false};
    a.vec = D % 8 == 0 && aligned16(x) && aligned16(out) && (NS < 2 || aligned16(y)) &&
            aligned16(b0) && (NB < 2 || aligned16(b1));
    return launch_ew<Op>(a, stream);
}

}  // namespace
}  // namespace anima

using namespace anima;

// ================================================================ C ABI

extern "C" int anima_gelu_tanh_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N,
                                    anima_stream_t stream) {
    return flat_op<OpGelu>(x, nullptr, nullptr, out, N, 0, stream);
}

extern "C" int anima_gelu_tanh_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                         anima_bf16 *out, int64_t N, int D, anima_stream_t stream) {
    return flat_op<OpGeluBias>(x, nullptr, bias, out, N, D, stream);
}

extern "C" int anima_silu_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N,
                               anima_stream_t stream) {
    return flat_op<OpSilu>(x, nullptr, nullptr, out, N, 0, stream);
}

extern "C" int anima_silu_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out,
                                    int64_t N, int D, anima_stream_t stream) {
    return flat_op<OpSiluBias>(x, nullptr, bias, out, N, D, stream);
}

extern "C" int anima_add_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                              anima_stream_t stream) {
    return flat_op<OpAdd>(a, b, nullptr, out, N, 0, stream);
}

extern "C" int anima_mul_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                              anima_stream_t stream) {
    return flat_op<OpMul>(a, b, nullptr, out, N, 0, stream);
}

extern "C" int anima_swiglu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out,
                                 int64_t N, anima_stream_t stream) {
    return flat_op<OpSwiGLU>(gate, up, nullptr, out, N, 0, stream);
}

extern "C" int anima_gated_gelu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out,
                                     int64_t N, anima_stream_t stream) {
    // gemma_ops.cu:24-31 covers every element (no pair loop): process N, not 2*floor(N/2).
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!gate || !up || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(gate) || !bf16_ok(up) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(gate, N * 2, out, N * 2) || partial_overlap(up, N * 2, out, N * 2))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{gate, up, nullptr, nullptr, out, N, 0, false};
    a.vec = aligned16(gate) && aligned16(up) && aligned16(out);
    return launch_ew<OpGatedGelu>(a, stream);
}

extern "C" int anima_scale_shift_bcast_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                            const anima_bf16 *shift, anima_bf16 *out, int M, int D,
                                            anima_stream_t stream) {
    return bcast_op<OpScaleShift>(x, nullptr, scale, shift, out, M, D, stream);
}

extern "C" int anima_residual_gate_bcast_bf16(const anima_bf16 *x, const anima_bf16 *y,
                                              const anima_bf16 *gate, anima_bf16 *out, int M, int D,
                                              anima_stream_t stream) {
    return bcast_op<OpResidualGate>(x, y, gate, nullptr, out, M, D, stream);
}
