// rope.cu -- rotary embeddings (sm_100a): Cosmos 3-axis half-split RoPE on the strided
// [B*S, H*HD] layout, the standard half-split RoPE with fp32 tables, and the fused
// per-head QK RMSNorm + Cosmos RoPE.
//
// Work unit = one 8-element chunk of the first half of one head of one row, plus the
// matching chunk of the second half: two 16-byte streamed loads of x, 16-byte cached
// loads of the cos/sin table row (shared by every head of a token, so it is read from
// L1/L2, not HBM), two 16-byte stores. Two units per thread keep four streamed loads in
// flight. The reference instead runs one thread per element pair
// with scalar 2-byte accesses and 64-bit div/mod per thread (rope.cu:72-108).
#include "common.cuh"

namespace anima {
namespace {

constexpr int kRopeBlock = 256;
constexpr int kRopeU = 2;

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}
__device__ __forceinline__ void stb(anima_bf16 *p, float f) {
    *reinterpret_cast<__nv_bfloat16 *>(p) = __float2bfloat16_rn(f);
}

// rope.cu:101-107. Every operand is a bf16 value, so both products are exact in fp32 and
// the result has one rounding however the expression is contracted.
__device__ __forceinline__ void rot_bf16(float xr, float xi, float c, float s, float &o_r, float &o_i) {
    o_r = __fmaf_rn(xr, c, -(xi * s));
    o_i = __fmaf_rn(xi, c, xr * s);
}

// gemma_ops.cu:84-85 with fp32 tables: x1*c - x2*s and x2*c + x1*s. The reference build
// contracts each into one fma: the first folds x1*c, the second folds x1*s (pinned
// against the reference kernels' outputs on the GPU).
__device__ __forceinline__ void rot_f32(float x1, float x2, float c, float s, float &o1, float &o2) {
    o1 = __fmaf_rn(x1, c, -(x2 * s));
    o2 = __fmaf_rn(x1, s, x2 * c);
}

// rot_bf16 on packed bf16 words (two element pairs): every operand is a bf16 value, so
// sm_100's mixed-precision fma takes them unpacked-free. xi*s and xr*s are exact products
// (16 significant bits), formed as fma(a, b, -0.0), which returns the product with its own
// sign of zero; the outer fmas then round once each, as fmaf(xr, c, -(xi*s)) and
// fmaf(xi, c, xr*s) do. -(xi*s) is xi*(-s), with the sign flipped on the bf16 word.
__device__ __forceinline__ void rot_bf16_w(uint32_t xr, uint32_t xi, uint32_t c, uint32_t s, uint32_t &o_r,
                                           uint32_t &o_i) {
    const float2 nz = make_float2(-0.0f, -0.0f);
    const float2 r = bf2_fma(xr, c, bf2_fma(xi, s ^ 0x80008000u, nz));
    const float2 i = bf2_fma(xi, c, bf2_fma(xr, s, nz));
    o_r = pack_bf2(r.x, r.y);
    o_i = pack_bf2(i.x, i.y);
}

struct CosmosArgs {
    anima_bf16 *x;
    const anima_bf16 *cos_t, *sin_t;
    int S, H, HD;
    int64_t units;   // rows * H * (HD/16)
    uint32_t hc;     // chunks per half head = HD/16
    int hc_shift;    // log2(hc) when hc is a power of two, else -1
};

// One group of kRopeU units per thread (units blockIdx*256*U + u*256 + t: each warp-wide load
// covers consecutive chunks) and short-lived CTAs: measured faster than a resident wave of
// CTAs striding over the tensor (8192 rows: 11.6 against 12.4 us; 32768 rows: 40.6 against
// 44.8 us), since CTAs that retire early free their SM for the next ones instead of leaving a
// tail. kSmall: the unit index fits in 32 bits, so the (row, head, chunk) split uses 32-bit
// division.
template <bool kSmall>
__global__ void __launch_bounds__(kRopeBlock) rope_cosmos_vec(CosmosArgs a) {
    pdl_wait();
    const uint32_t per_row = (uint32_t)a.H * a.hc;
    const int half = a.HD / 2;
    const int64_t base = (int64_t)blockIdx.x * kRopeBlock * kRopeU + threadIdx.x;
    Vec8 xr[kRopeU], xi[kRopeU], cv[kRopeU], sv[kRopeU];
    anima_bf16 *p[kRopeU];
    bool ok[kRopeU];
#pragma unroll
    for (int u = 0; u < kRopeU; ++u) {
        const int64_t i = base + u * kRopeBlock;
        ok[u] = i < a.units;
        if (ok[u]) {
            int64_t row, pos;
            uint32_t rem;
            if constexpr (kSmall) {
                const uint32_t r32 = (uint32_t)i / per_row;
                rem = (uint32_t)i - r32 * per_row;
                row = r32;
                pos = r32 % (uint32_t)a.S;
            } else {
                row = i / per_row;
                rem = (uint32_t)(i - row * per_row);
                pos = row % a.S;
            }
            const uint32_t h = a.hc_shift >= 0 ? rem >> a.hc_shift : rem / a.hc;
            const uint32_t c = rem - h * a.hc;
            p[u] = a.x + row * (int64_t)a.H * a.HD + (int64_t)h * a.HD + c * 8;
            xr[u] = ld_stream(p[u]);
            xi[u] = ld_stream(p[u] + half);
            const int64_t t = pos * a.HD + c * 8;
            cv[u] = ld_cached(a.cos_t + t);
            sv[u] = ld_cached(a.sin_t + t);
        }
    }
#pragma unroll
    for (int u = 0; u < kRopeU; ++u) {
        if (!ok[u]) continue;
        Vec8 o_r, o_i;
#pragma unroll
        for (int j = 0; j < 4; ++j) rot_bf16_w(xr[u].w[j], xi[u].w[j], cv[u].w[j], sv[u].w[j], o_r.w[j], o_i.w[j]);
        st_vec(p[u], o_r);
        st_vec(p[u] + half, o_i);
    }
    pdl_launch();
}

// One thread per element pair, scalar accesses (any even HD, any 2-byte alignment).
__global__ void rope_cosmos_scalar(anima_bf16 *x, const anima_bf16 *cos_t, const anima_bf16 *sin_t,
                                   int S, int H, int HD, int64_t pairs) {
    pdl_wait();
    const int half = HD / 2;
    const int64_t per_row = (int64_t)H * half;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / per_row, rem = i % per_row;
        const int64_t h = rem / half, k = rem % half, s = row % S;
        anima_bf16 *b = x + row * H * HD + h * HD;
        float o_r, o_i;
        rot_bf16(ldb(b + k), ldb(b + k + half), ldb(cos_t + s * HD + k), ldb(sin_t + s * HD + k), o_r, o_i);
        stb(b + k, o_r);
        stb(b + k + half, o_i);
    }
}

struct StdArgs {
    anima_bf16 *x;
    const float *cos_t, *sin_t;
    int T, D;
    int64_t units;  // rows * (D/16)
    uint32_t hc;    // chunks per half row = D/16
};

__global__ void __launch_bounds__(kRopeBlock, 3) rope_standard_vec(StdArgs a) {
    pdl_wait();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int half = a.D / 2;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    UnitCursor cur(i, stride, a.hc, (uint32_t)a.T);
    while (i < a.units) {
        Vec8 x1[kRopeU], x2[kRopeU];
        float4 cv[kRopeU][2], sv[kRopeU][2];
        anima_bf16 *p[kRopeU];
        bool ok[kRopeU];
#pragma unroll
        for (int u = 0; u < kRopeU; ++u) {
            ok[u] = i < a.units;
            if (ok[u]) {
                const uint32_t c = cur.rem;
                p[u] = a.x + cur.row * a.D + c * 8;
                x1[u] = ld_stream(p[u]);
                x2[u] = ld_stream(p[u] + half);
                const int64_t t = (int64_t)cur.ph * half + c * 8;
                const float4 *cp = reinterpret_cast<const float4 *>(a.cos_t + t);
                const float4 *sp = reinterpret_cast<const float4 *>(a.sin_t + t);
                cv[u][0] = __ldg(cp);
                cv[u][1] = __ldg(cp + 1);
                sv[u][0] = __ldg(sp);
                sv[u][1] = __ldg(sp + 1);
            }
            i += stride;
            cur.advance(a.hc, (uint32_t)a.T);
        }
#pragma unroll
        for (int u = 0; u < kRopeU; ++u) {
            if (!ok[u]) break;
            float f1[8], f2[8], o1[8], o2[8];
            unpack8(x1[u], f1);
            unpack8(x2[u], f2);
            const float c[8] = {cv[u][0].x, cv[u][0].y, cv[u][0].z, cv[u][0].w,
                                cv[u][1].x, cv[u][1].y, cv[u][1].z, cv[u][1].w};
            const float s[8] = {sv[u][0].x, sv[u][0].y, sv[u][0].z, sv[u][0].w,
                                sv[u][1].x, sv[u][1].y, sv[u][1].z, sv[u][1].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) rot_f32(f1[e], f2[e], c[e], s[e], o1[e], o2[e]);
            st_vec(p[u], pack8(o1));
            st_vec(p[u] + half, pack8(o2));
        }
    }
    pdl_launch();
}

__global__ void rope_standard_scalar(anima_bf16 *x, const float *cos_t, const float *sin_t, int T,
                                     int D, int64_t pairs) {
    pdl_wait();
    const int half = D / 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / half, d = i % half, t = row % T;
        anima_bf16 *b = x + row * D;
        float o1, o2;
        rot_f32(ldb(b + d), ldb(b + half + d), cos_t[t * half + d], sin_t[t * half + d], o1, o2);
        stb(b + d, o1);
        stb(b + half + d, o2);
    }
}

// ----------------------------------------------- fused QK RMSNorm + Cosmos RoPE
// One 8-lane team per (token row, head) with HD = 128: lane l holds chunk l (elements
// 8l..8l+7 of the first half) and chunk l+8 (the second half), i.e. both members of its
// rotation pairs. The RMS statistics replay the reference's reduction tree for a
// 128-wide row (ref_pair_tree_sum<8,2>), the normalised values are rounded to bf16 as
// rms_norm_bf16 stores them, then rotated exactly as rope_cosmos_strided_bf16 does.
struct QkArgs {
    anima_bf16 *x;
    const anima_bf16 *w, *cos_t, *sin_t;
    int S, H;
    int64_t heads;  // B*S*H
    float eps;
};

// kNarrow (heads < 2^32): token and table row by 32-bit division. A compile-time choice: with
// a run-time flag the unused 64-bit path cost 0.7 us per launch at [8192 x 16, 128].
template <bool kNarrow>
__global__ void __launch_bounds__(kRopeBlock) qk_norm_rope_128(QkArgs a) {
    pdl_wait();
    constexpr int LPR = 8, K = 2, HD = 128;
    const int l = threadIdx.x & (LPR - 1);
    const int64_t hid = (int64_t)blockIdx.x * (blockDim.x / LPR) + threadIdx.x / LPR;
    const bool live = hid < a.heads;
    const int64_t token = kNarrow ? (int64_t)((uint32_t)hid / (uint32_t)a.H) : hid / a.H;
    anima_bf16 *p = a.x + hid * HD + l * 8;
    Vec8 v[K] = {Vec8{{0u, 0u, 0u, 0u}}, Vec8{{0u, 0u, 0u, 0u}}};
    Vec8 w[K], cv, sv;
    if (live) {
        v[0] = ld_stream(p);
        v[1] = ld_stream(p + 64);
    }
    w[0] = ld_cached(a.w + l * 8);
    w[1] = ld_cached(a.w + 64 + l * 8);
    const int64_t s = !live ? 0 : kNarrow ? (int64_t)((uint32_t)token % (uint32_t)a.S) : token % a.S;
    cv = ld_cached(a.cos_t + s * HD + l * 8);
    sv = ld_cached(a.sin_t + s * HD + l * 8);

    float q[K][4];
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float2 t = sq_pair2(v[k].w[j], v[k].w[j + 1]);
            q[k][j] = t.x;
            q[k][j + 1] = t.y;
        }
    const float sq = ref_pair_tree_sum<LPR, K>(q, l, 0xffffffffu);
    const float r = rsqrtf(div_pow2<HD>(sq) + a.eps);
    pdl_launch();
    if (!live) return;
    // rms_norm.cu:62-64 ((x*r)*w, stored as bf16) then rope.cu:101-107, on element pairs with
    // packed fp32x2 ops (each lane rounds as the scalar op does)
    Vec8 o0, o1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 rr = make_float2(r, r);
        const float2 n0 = __fmul2_rn(__fmul2_rn(make_float2(bf_lo(v[0].w[j]), bf_hi(v[0].w[j])), rr),
                                     make_float2(bf_lo(w[0].w[j]), bf_hi(w[0].w[j])));
        const float2 n1 = __fmul2_rn(__fmul2_rn(make_float2(bf_lo(v[1].w[j]), bf_hi(v[1].w[j])), rr),
                                     make_float2(bf_lo(w[1].w[j]), bf_hi(w[1].w[j])));
        const uint32_t p0 = pack_bf2(n0.x, n0.y), p1 = pack_bf2(n1.x, n1.y);
        rot_bf16_w(p0, p1, cv.w[j], sv.w[j], o0.w[j], o1.w[j]);
    }
    st_vec(p, o0);
    st_vec(p + 64, o1);
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

// -------------------------- fused head transpose + QK RMSNorm + standard RoPE (Qwen3)
// qwen3.cpp:164-178: head_transpose_bf16 ([T, H*HD] -> [H, T, HD]), rms_norm_bf16 on each
// head row (weight nullable), rope_standard_bf16 (fp32 tables [T, HD/2]). One 8-lane team per
// (token t, head h) with HD = 128, teams in source order (the heads of a token share their
// table row in L1): lane l holds elements 8l..8l+7 and 64+8l..64+8l+7, i.e. both members of
// its rotation pairs. The statistics replay the reference's tree (ref_pair_tree_sum<8,2>),
// the normalised values are rounded to bf16 as rms_norm_bf16 stores them, and the rotation
// is rope_standard_bf16's own contraction (rot_f32); no tables = no rotation.
struct HeadArgs {
    const anima_bf16 *src, *w;
    const float *cos_t, *sin_t;
    anima_bf16 *dst;
    int H, T;
    int64_t heads;  // T*H
    float eps;
};

__global__ void __launch_bounds__(kRopeBlock) head_norm_rope_128(HeadArgs a) {
    pdl_wait();
    constexpr int LPR = 8, K = 2, HD = 128;
    const int l = threadIdx.x & (LPR - 1);
    const int64_t hid = (int64_t)blockIdx.x * (blockDim.x / LPR) + threadIdx.x / LPR;  // t*H + h
    const bool live = hid < a.heads;
    const int64_t t = live ? hid / a.H : 0, h = hid - t * a.H;
    const anima_bf16 *p = a.src + hid * HD + l * 8;
    Vec8 v[K] = {Vec8{{0u, 0u, 0u, 0u}}, Vec8{{0u, 0u, 0u, 0u}}};
    if (live) {
        v[0] = ld_stream(p);
        v[1] = ld_stream(p + 64);
    }
    Vec8 w[K];
    if (a.w) {
        w[0] = ld_cached(a.w + l * 8);
        w[1] = ld_cached(a.w + 64 + l * 8);
    }
    float4 cv[2], sv[2];
    if (a.cos_t) {
        const float4 *cp = reinterpret_cast<const float4 *>(a.cos_t + t * 64 + l * 8);
        const float4 *sp = reinterpret_cast<const float4 *>(a.sin_t + t * 64 + l * 8);
        cv[0] = __ldg(cp);
        cv[1] = __ldg(cp + 1);
        sv[0] = __ldg(sp);
        sv[1] = __ldg(sp + 1);
    }
    float q[K][4];
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float2 t = sq_pair2(v[k].w[j], v[k].w[j + 1]);
            q[k][j] = t.x;
            q[k][j + 1] = t.y;
        }
    const float r = rsqrtf(div_pow2<HD>(ref_pair_tree_sum<LPR, K>(q, l, 0xffffffffu)) + a.eps);
    pdl_launch();
    if (!live) return;
    // rms_norm.cu:62-64: (x * r) * w, stored as bf16
    Vec8 n[K];
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 f = __fmul2_rn(make_float2(bf_lo(v[k].w[j]), bf_hi(v[k].w[j])), make_float2(r, r));
            if (a.w) f = __fmul2_rn(f, make_float2(bf_lo(w[k].w[j]), bf_hi(w[k].w[j])));
            n[k].w[j] = pack_bf2(f.x, f.y);
        }
    anima_bf16 *o = a.dst + (h * a.T + t) * HD + l * 8;
    if (a.cos_t) {  // gemma_ops.cu:80-86 on the bf16 values
        const float c[8] = {cv[0].x, cv[0].y, cv[0].z, cv[0].w, cv[1].x, cv[1].y, cv[1].z, cv[1].w};
        const float sn[8] = {sv[0].x, sv[0].y, sv[0].z, sv[0].w, sv[1].x, sv[1].y, sv[1].z, sv[1].w};
        float f1[8], f2[8], o1[8], o2[8];
        unpack8(n[0], f1);
        unpack8(n[1], f2);
#pragma unroll
        for (int e = 0; e < 8; ++e) rot_f32(f1[e], f2[e], c[e], sn[e], o1[e], o2[e]);
        n[0] = pack8(o1);
        n[1] = pack8(o2);
    }
    st_vec(o, n[0]);
    st_vec(o + 64, n[1]);
}

}  // namespace
}  // namespace anima

using namespace anima;

// ================================================================ C ABI

extern "C" int anima_rope_cosmos_strided_bf16(anima_bf16 *x, const anima_bf16 *cos_table,
                                              const anima_bf16 *sin_table, int B, int S, int H,
                                              int HD, anima_stream_t stream) {
    if (B < 0 || S < 0 || H < 0 || HD <= 0 || (HD & 1)) return ANIMA_ERR_BAD_SHAPE;
    const int64_t rows = (int64_t)B * S;
    if (rows == 0 || H == 0) return ANIMA_OK;
    if (!x || !cos_table || !sin_table) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(cos_table) || !bf16_ok(sin_table)) return ANIMA_ERR_MISALIGNED;
    const int64_t nx = rows * H * HD * 2, nt = (int64_t)S * HD * 2;
    if (partial_overlap(x, nx, cos_table, nt) || partial_overlap(x, nx, sin_table, nt) ||
        x == cos_table || x == sin_table)
        return ANIMA_ERR_OVERLAP;
    if (HD % 16 == 0 && aligned16(x) && aligned16(cos_table) && aligned16(sin_table)) {
        const int hc = HD / 16;
        CosmosArgs a{x, cos_table, sin_table, S, H, HD, rows * H * hc, (uint32_t)hc,
                     (hc & (hc - 1)) == 0 ? __builtin_ctz((unsigned)hc) : -1};
        const int64_t blocks = (a.units + kRopeBlock * kRopeU - 1) / (kRopeBlock * kRopeU);
        if (blocks > 2147483647) return ANIMA_ERR_TOO_LARGE;
        if (a.units <= 0xffffffffll) launch(rope_cosmos_vec<true>, (unsigned)blocks, kRopeBlock, 0, stream, a);
        else launch(rope_cosmos_vec<false>, (unsigned)blocks, kRopeBlock, 0, stream, a);
    } else {
        const int64_t pairs = rows * H * (HD / 2);
        int err = ANIMA_OK;
        const unsigned grid = wave_grid((const void *)rope_cosmos_scalar, kRopeBlock, 0, pairs, &err);
        if (err) return err;
        launch(rope_cosmos_scalar, grid, kRopeBlock, 0, stream, x, cos_table, sin_table, S, H, HD, pairs);
    }
    return launch_status();
}

extern "C" int anima_rope_standard_bf16(anima_bf16 *x, const float *cos_table, const float *sin_table,
                                        int total_rows, int T, int D, anima_stream_t stream) {
    if (total_rows < 0 || T <= 0 || D <= 0 || (D & 1)) return ANIMA_ERR_BAD_SHAPE;
    if (total_rows == 0) return ANIMA_OK;
    if (!x || !cos_table || !sin_table) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !aligned_to(cos_table, 4) || !aligned_to(sin_table, 4)) return ANIMA_ERR_MISALIGNED;
    if (D % 16 == 0 && aligned16(x) && aligned16(cos_table) && aligned16(sin_table)) {
        StdArgs a{x, cos_table, sin_table, T, D, (int64_t)total_rows * (D / 16), (uint32_t)(D / 16)};
        int err = ANIMA_OK;
        const unsigned grid = wave_grid((const void *)rope_standard_vec, kRopeBlock, 0, (a.units + kRopeU - 1) / kRopeU, &err);
        if (err) return err;
        launch(rope_standard_vec, grid, kRopeBlock, 0, stream, a);
    } else {
        const int64_t pairs = (int64_t)total_rows * (D / 2);
        int err = ANIMA_OK;
        const unsigned grid = wave_grid((const void *)rope_standard_scalar, kRopeBlock, 0, pairs, &err);
        if (err) return err;
        launch(rope_standard_scalar, grid, kRopeBlock, 0, stream, x, cos_table, sin_table, T, D, pairs);
    }
    return launch_status();
}

extern "C" int anima_qk_norm_rope_bf16(anima_bf16 *x, const anima_bf16 *weight,
                                       const anima_bf16 *cos_table, const anima_bf16 *sin_table,
                                       int B, int S, int H, int HD, float eps, anima_stream_t stream) {
    if (B < 0 || S < 0 || H < 0 || HD <= 0 || (HD & 1)) return ANIMA_ERR_BAD_SHAPE;
    const int64_t heads = (int64_t)B * S * H;
    if (heads == 0) return ANIMA_OK;
    if (!x || !weight || !cos_table || !sin_table) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(weight) || !bf16_ok(cos_table) || !bf16_ok(sin_table))
        return ANIMA_ERR_MISALIGNED;
    if (HD == 128 && aligned16(x) && aligned16(weight) && aligned16(cos_table) && aligned16(sin_table)) {
        const int64_t nx = heads * HD * 2, nt = (int64_t)S * HD * 2;
        if (partial_overlap(x, nx, cos_table, nt) || partial_overlap(x, nx, sin_table, nt) ||
            partial_overlap(x, nx, weight, HD * 2) || x == cos_table || x == sin_table || x == weight)
            return ANIMA_ERR_OVERLAP;
        QkArgs a{x, weight, cos_table, sin_table, S, H, heads, eps};
        const int64_t per_block = kRopeBlock / 8;
        const unsigned grid = (unsigned)((heads + per_block - 1) / per_block);
        if (heads < 4294967296LL) launch(qk_norm_rope_128<true>, grid, kRopeBlock, 0, stream, a);
        else launch(qk_norm_rope_128<false>, grid, kRopeBlock, 0, stream, a);
        return launch_status();
    }
    // Other head sizes: the same two steps as the reference, back to back.
    if (heads > 2147483647) return ANIMA_ERR_TOO_LARGE;
    if (int e = anima_rms_norm_bf16(x, weight, x, (int)heads, HD, eps, stream)) return e;
    return anima_rope_cosmos_strided_bf16(x, cos_table, sin_table, B, S, H, HD, stream);
}

extern "C" int anima_head_transpose_qk_norm_rope_bf16(const anima_bf16 *src, const anima_bf16 *weight,
                                                      const float *cos_table, const float *sin_table,
                                                      anima_bf16 *dst, int H, int T, int HD, float eps,
                                                      anima_stream_t stream) {
    if (H < 0 || T < 0 || HD <= 0 || (HD & 1)) return ANIMA_ERR_BAD_SHAPE;
    const int64_t heads = (int64_t)T * H, n = heads * HD;
    if (n == 0) return ANIMA_OK;
    if (!src || !dst || (!cos_table != !sin_table)) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(src) || !bf16_ok(dst) || (weight && !bf16_ok(weight)) ||
        (cos_table && (!aligned_to(cos_table, 4) || !aligned_to(sin_table, 4))))
        return ANIMA_ERR_MISALIGNED;
    if (overlaps(src, n * 2, dst, n * 2) || (weight && overlaps(weight, (int64_t)HD * 2, dst, n * 2)) ||
        (cos_table && (overlaps(cos_table, (int64_t)T * HD * 2, dst, n * 2) ||
                       overlaps(sin_table, (int64_t)T * HD * 2, dst, n * 2))))
        return ANIMA_ERR_OVERLAP;
    if (HD == 128 && aligned16(src) && aligned16(dst) && (!weight || aligned16(weight)) &&
        (!cos_table || (aligned16(cos_table) && aligned16(sin_table)))) {
        HeadArgs a{src, weight, cos_table, sin_table, dst, H, T, heads, eps};
        const int64_t per_block = kRopeBlock / 8;
        launch(head_norm_rope_128, (unsigned)((heads + per_block - 1) / per_block), kRopeBlock, 0, stream, a);
        return launch_status();
    }
    // Other head sizes: the reference's three steps, back to back.
    if (heads > 2147483647) return ANIMA_ERR_TOO_LARGE;
    if (int e = anima_head_transpose_bf16(src, dst, H, T, HD, stream)) return e;
    if (int e = anima_rms_norm_bf16(dst, weight, dst, (int)heads, HD, eps, stream)) return e;
    return cos_table ? anima_rope_standard_bf16(dst, cos_table, sin_table, (int)heads, T, HD, stream) : ANIMA_OK;
}
