// rownorm.cu -- LayerNorm / adaLN / residual-gate adaLN / RMSNorm row kernels (sm_100a).
//
// Fast path (D a multiple of 64, D <= 2048, 16-byte aligned rows): a row belongs to a
// team of LPR lanes, each lane streams K 16-byte chunks of it into registers with
// L1-bypassing vector loads, so the row crosses HBM exactly once (read once, written
// once), with no shared memory and no __syncthreads. The statistics go through
// ref_pair_tree_sum, which reproduces the reference CTA's addition order, and the
// per-element epilogue uses the reference's expressions, so outputs match the
// reference kernels bit for bit.
//
//   D      LPR  K  rows/warp       D      LPR  K  rows/warp
//   64      8   1      4           512     8   8      4
//   128     8   2      4           1024   16   8      2
//   256     8   4      4           2048   32   8      1
//
// Generic path (any even D, any 2-byte alignment): one CTA per row with the reference's
// own thread layout and scalar accesses. Same bits, reference-like speed.
#include "common.cuh"

namespace anima {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRowBlock = 256;

// var = sum_sq/D - mean*mean: nvcc contracts the reference's expression
// (layer_norm.cu:49,107,179) into one fma.
__device__ __forceinline__ float ln_var(float sq, float mean, int D) {
    return fmaf(-mean, mean, __fdiv_rn(sq, (float)D));
}

// sum_sq += h0*h0 + h1*h1 on unrounded fp32 h (layer_norm.cu:176): nvcc folds the first
// product into an fma with the second.
__device__ __forceinline__ float resid_sq_pair(float h0, float h1) { return fmaf(h0, h0, h1 * h1); }

// ---------------------------------------------------------------- row ops
// Each op loads its row chunks (first phase), produces per-pair sum / sum-of-squares
// values, and writes the outputs from the reduced statistics (second phase).

struct LayerNormOp {  // layer_norm.cu:26-59
    const anima_bf16 *x;
    anima_bf16 *out;
    int D;
    float eps;
};

struct AdaLNOp {  // layer_norm.cu:83-125
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    int D;
    float eps;
};

struct LnModulateOp {  // layer_norm.cu:26-59 then elementwise.cu:216-236
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    int D;
    float eps;
};

struct RmsOp {  // rms_norm.cu:9-67
    const anima_bf16 *x, *weight;  // weight nullable
    anima_bf16 *out;
    int D;
    float eps;
};

struct AdaRmsOp {  // adaln.cu:11-58 (per-row scale/shift)
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    int D;
    float eps;
};

// --------------------------------------------------- team (fast path) kernels

template <int LPR, int K>
struct TeamRow {
    int64_t row;
    int l;     // lane index inside the team
    bool live; // row < N; dead lanes still join every shuffle
    __device__ __forceinline__ int64_t chunk_off(int k) const {
        return (int64_t)(l + LPR * k) * 8;
    }
};

// Loads the K chunks of `base + row*D` (zeros for dead lanes).
template <int LPR, int K>
__device__ __forceinline__ void load_row(const TeamRow<LPR, K> &t, const anima_bf16 *base, int D,
                                         Vec8 (&v)[K]) {
    const anima_bf16 *r = base + t.row * (int64_t)D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        if (t.live) v[k] = ld_stream(r + t.chunk_off(k));
        else v[k] = Vec8{{0u, 0u, 0u, 0u}};
    }
}

// Per-pair statistics of plain bf16 data: s = v0 + v1, q = round(v0^2 + v1^2). The bf16
// squares are exact in fp32, so this is the same value whichever order the reference's
// kernels accumulate the pair in (layer_norm.cu:44-46, :103-104; rms_norm.cu:35-36).
template <int K>
__device__ __forceinline__ void pair_stats(const Vec8 (&v)[K], float (&s)[K][4], float (&q)[K][4]) {
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float a = bf_lo(v[k].w[j]), b = bf_hi(v[k].w[j]);
            s[k][j] = a + b;
            q[k][j] = fmaf(b, b, a * a);
        }
}

template <int LPR, int K>
__device__ __forceinline__ float row_mean_invstd(const TeamRow<LPR, K> &t, const Vec8 (&v)[K], int D,
                                                 float eps, float &mean) {
    float s[K][4], q[K][4];
    pair_stats<K>(v, s, q);
    const float sum = ref_pair_tree_sum<LPR, K>(s, t.l, kFull);
    const float sq = ref_pair_tree_sum<LPR, K>(q, t.l, kFull);
    mean = __fdiv_rn(sum, (float)D);
    return rsqrtf(ln_var(sq, mean, D) + eps);
}

template <int LPR, int K>
__device__ __forceinline__ float row_rms_inv(const TeamRow<LPR, K> &t, const Vec8 (&v)[K], int D,
                                             float eps) {
    float s[K][4], q[K][4];
    pair_stats<K>(v, s, q);
    const float sq = ref_pair_tree_sum<LPR, K>(q, t.l, kFull);
    return rsqrtf(__fdiv_rn(sq, (float)D) + eps);
}

template <int LPR, int K>
__device__ __forceinline__ TeamRow<LPR, K> team_row(int64_t N) {
    TeamRow<LPR, K> t;
    t.l = threadIdx.x & (LPR - 1);
    t.row = (int64_t)blockIdx.x * (blockDim.x / LPR) + threadIdx.x / LPR;
    t.live = t.row < N;
    return t;
}

template <int LPR, int K>
__global__ void __launch_bounds__(kRowBlock) layer_norm_team(LayerNormOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 v[K];
    load_row(t, op.x, op.D, v);
    float mean;
    const float inv = row_mean_invstd(t, v, op.D, op.eps, mean);
    if (!t.live) return;
    anima_bf16 *o = op.out + t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8];
        unpack8(v[k], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = (f[e] - mean) * inv;
        st_vec(o + t.chunk_off(k), pack8(f));
    }
}

template <int LPR, int K>
__global__ void __launch_bounds__(kRowBlock) adaln_team(AdaLNOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 v[K];
    load_row(t, op.x, op.D, v);
    float mean;
    const float inv = row_mean_invstd(t, v, op.D, op.eps, mean);
    if (!t.live) return;
    anima_bf16 *o = op.out + t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8], sc[8], sh[8];
        unpack8(v[k], f);
        unpack8(ld_cached(op.scale + t.chunk_off(k)), sc);
        unpack8(ld_cached(op.shift + t.chunk_off(k)), sh);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = fmaf((f[e] - mean) * inv, 1.0f + sc[e], sh[e]);
        st_vec(o + t.chunk_off(k), pack8(f));
    }
}

template <int LPR, int K>
__global__ void __launch_bounds__(kRowBlock) ln_modulate_team(LnModulateOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 v[K];
    load_row(t, op.x, op.D, v);
    float mean;
    const float inv = row_mean_invstd(t, v, op.D, op.eps, mean);
    if (!t.live) return;
    anima_bf16 *o = op.out + t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8], sc[8], sh[8];
        unpack8(v[k], f);
        unpack8(ld_cached(op.scale + t.chunk_off(k)), sc);
        unpack8(ld_cached(op.shift + t.chunk_off(k)), sh);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            f[e] = fmaf(bf16_round((f[e] - mean) * inv), 1.0f + sc[e], sh[e]);
        st_vec(o + t.chunk_off(k), pack8(f));
    }
}

struct ResGateAdaLNOp {  // layer_norm.cu:146-196
    anima_bf16 *hidden;
    const anima_bf16 *sub_out, *gate, *scale, *shift;
    anima_bf16 *normed;
    int D;
    float eps;
};

template <int LPR, int K>
__global__ void __launch_bounds__(kRowBlock) residual_gate_adaln_team(ResGateAdaLNOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 x[K], y[K];
    load_row(t, op.hidden, op.D, x);
    load_row(t, op.sub_out, op.D, y);
    float s[K][4], q[K][4];
    Vec8 hb[K];  // bf16(h), written back to hidden and re-read by the reference's pass 2
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const Vec8 g = ld_cached(op.gate + t.chunk_off(k));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // h = x + y*gate: the bf16 product is exact, so the reference's fma and
            // this one round identically.
            float h0 = fmaf(bf_lo(y[k].w[j]), bf_lo(g.w[j]), bf_lo(x[k].w[j]));
            float h1 = fmaf(bf_hi(y[k].w[j]), bf_hi(g.w[j]), bf_hi(x[k].w[j]));
            hb[k].w[j] = pack_bf2(h0, h1);
            s[k][j] = h0 + h1;
            q[k][j] = resid_sq_pair(h0, h1);
        }
    }
    const float sum = ref_pair_tree_sum<LPR, K>(s, t.l, kFull);
    const float sq = ref_pair_tree_sum<LPR, K>(q, t.l, kFull);
    const float mean = __fdiv_rn(sum, (float)op.D);
    const float inv = rsqrtf(ln_var(sq, mean, op.D) + op.eps);
    if (!t.live) return;
    anima_bf16 *hr = op.hidden + t.row * (int64_t)op.D;
    anima_bf16 *nr = op.normed + t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        st_vec(hr + t.chunk_off(k), hb[k]);
        float f[8], sc[8], sh[8];
        unpack8(hb[k], f);
        unpack8(ld_cached(op.scale + t.chunk_off(k)), sc);
        unpack8(ld_cached(op.shift + t.chunk_off(k)), sh);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = fmaf((f[e] - mean) * inv, 1.0f + sc[e], sh[e]);
        st_vec(nr + t.chunk_off(k), pack8(f));
    }
}

template <int LPR, int K, bool kWeight>
__global__ void __launch_bounds__(kRowBlock) rms_norm_team(RmsOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 v[K];
    load_row(t, op.x, op.D, v);
    Vec8 w[K];
    if constexpr (kWeight) {
#pragma unroll
        for (int k = 0; k < K; ++k) w[k] = ld_cached(op.weight + t.chunk_off(k));
    }
    const float r = row_rms_inv(t, v, op.D, op.eps);
    if (!t.live) return;
    anima_bf16 *o = op.out + t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8];
        unpack8(v[k], f);
        if constexpr (kWeight) {
            float g[8];
            unpack8(w[k], g);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * g[e];
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * r;
        }
        st_vec(o + t.chunk_off(k), pack8(f));
    }
}

template <int LPR, int K>
__global__ void __launch_bounds__(kRowBlock) adaln_rms_team(AdaRmsOp op, int64_t N) {
    auto t = team_row<LPR, K>(N);
    Vec8 v[K];
    load_row(t, op.x, op.D, v);
    const float r = row_rms_inv(t, v, op.D, op.eps);
    if (!t.live) return;
    const int64_t base = t.row * (int64_t)op.D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8], sc[8], sh[8];
        unpack8(v[k], f);
        unpack8(ld_stream(op.scale + base + t.chunk_off(k)), sc);
        unpack8(ld_stream(op.shift + base + t.chunk_off(k)), sh);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = fmaf(f[e] * r, 1.0f + sc[e], sh[e]);
        st_vec(op.out + base + t.chunk_off(k), pack8(f));
    }
}

// ------------------------------------------- generic (reference-structured) kernels
// One CTA of ref_row_threads(D) threads per row, thread t owning pairs t, t+T, ...,
// scalar bf16 accesses (valid for any 2-byte alignment), reference reduction tree.

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}
__device__ __forceinline__ void stb(anima_bf16 *p, float f) {
    *reinterpret_cast<__nv_bfloat16 *>(p) = __float2bfloat16_rn(f);
}

enum class GenKind { LayerNorm, AdaLN, LnModulate, Rms, AdaRms, ResGate };

struct GenArgs {
    const anima_bf16 *x;        // x, or hidden for ResGate
    anima_bf16 *hidden;         // ResGate only
    const anima_bf16 *y, *gate; // ResGate only
    const anima_bf16 *scale, *shift, *weight;
    anima_bf16 *out;
    int D;
    float eps;
};

template <GenKind KIND>
__global__ void row_generic(GenArgs a, int64_t N) {
    __shared__ float red[33];
    const int D2 = a.D / 2, T = blockDim.x;
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
        const int64_t base = row * (int64_t)a.D;
        float s = 0.0f, q = 0.0f;
        for (int i = threadIdx.x; i < D2; i += T) {
            const int64_t e = base + 2 * i;
            if constexpr (KIND == GenKind::ResGate) {
                float h0 = fmaf(ldb(a.y + e), ldb(a.gate + 2 * i), ldb(a.hidden + e));
                float h1 = fmaf(ldb(a.y + e + 1), ldb(a.gate + 2 * i + 1), ldb(a.hidden + e + 1));
                stb(a.hidden + e, h0);
                stb(a.hidden + e + 1, h1);
                s += h0 + h1;
                q += resid_sq_pair(h0, h1);
            } else if constexpr (KIND == GenKind::AdaLN) {
                float v0 = ldb(a.x + e), v1 = ldb(a.x + e + 1);
                s += v0 + v1;
                q += fmaf(v1, v1, v0 * v0);
            } else {  // layer_norm.cu:44-46 / rms_norm.cu:35-36: two chained fmas
                float v0 = ldb(a.x + e), v1 = ldb(a.x + e + 1);
                s += v0 + v1;
                q = fmaf(v0, v0, q);
                q = fmaf(v1, v1, q);
            }
        }
        constexpr bool kMean = KIND == GenKind::LayerNorm || KIND == GenKind::AdaLN ||
                               KIND == GenKind::LnModulate || KIND == GenKind::ResGate;
        float mean = 0.0f, inv;
        if constexpr (kMean) {
            mean = __fdiv_rn(ref_cta_sum(s, red), (float)a.D);
            inv = rsqrtf(ln_var(ref_cta_sum(q, red), mean, a.D) + a.eps);
        } else {
            inv = rsqrtf(__fdiv_rn(ref_cta_sum(q, red), (float)a.D) + a.eps);
        }
        // Pass 2 over the thread's own pairs, as in the reference (ResGate re-reads the
        // bf16 hidden it wrote in pass 1).
        for (int i = threadIdx.x; i < D2; i += T) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int d = 2 * i + h;
                const int64_t e = base + d;
                float o;
                if constexpr (KIND == GenKind::LayerNorm) {
                    o = (ldb(a.x + e) - mean) * inv;
                } else if constexpr (KIND == GenKind::AdaLN) {
                    o = fmaf((ldb(a.x + e) - mean) * inv, 1.0f + ldb(a.scale + d), ldb(a.shift + d));
                } else if constexpr (KIND == GenKind::LnModulate) {
                    o = fmaf(bf16_round((ldb(a.x + e) - mean) * inv), 1.0f + ldb(a.scale + d),
                             ldb(a.shift + d));
                } else if constexpr (KIND == GenKind::ResGate) {
                    o = fmaf((ldb(a.hidden + e) - mean) * inv, 1.0f + ldb(a.scale + d),
                             ldb(a.shift + d));
                } else if constexpr (KIND == GenKind::Rms) {
                    o = ldb(a.x + e) * inv;
                    if (a.weight) o = o * ldb(a.weight + d);
                } else {  // AdaRms
                    o = fmaf(ldb(a.x + e) * inv, 1.0f + ldb(a.scale + e), ldb(a.shift + e));
                }
                stb(a.out + e, o);
            }
        }
    }
}

// gemma_ops.cu:132-168: scalar loop over D with min(roundup32(D),1024) threads per row.
__global__ void gemma_rms_generic(const anima_bf16 *x, const anima_bf16 *w, anima_bf16 *out,
                                  int64_t N, int D, float eps) {
    __shared__ float red[33];
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
        const int64_t base = row * (int64_t)D;
        float q = 0.0f;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = ldb(x + base + i);
            q += v * v;
        }
        const float inv = rsqrtf(__fdiv_rn(ref_cta_sum(q, red), (float)D) + eps);
        for (int i = threadIdx.x; i < D; i += blockDim.x)
            stb(out + base + i, (ldb(x + base + i) * inv) * (1.0f + ldb(w + i)));
        __syncthreads();
    }
}

// ------------------------------------------------------------- dispatch

// Picks (LPR, K) for the fast path: K = 8 chunks per lane whenever the row is wide
// enough, so every lane has 128 bytes of loads in flight.
template <class Launch>
bool dispatch_team(int D, Launch &&launch) {
    switch (D) {
    case 64: launch.template go<8, 1>(); return true;
    case 128: launch.template go<8, 2>(); return true;
    case 256: launch.template go<8, 4>(); return true;
    case 512: launch.template go<8, 8>(); return true;
    case 1024: launch.template go<16, 8>(); return true;
    case 2048: launch.template go<32, 8>(); return true;
    default: return false;
    }
}

inline unsigned team_grid(int64_t N, int LPR) {
    const int64_t rows_per_block = kRowBlock / LPR;
    return (unsigned)((N + rows_per_block - 1) / rows_per_block);
}

inline unsigned generic_grid(int64_t N) { return (unsigned)(N < 2147483647 ? N : 2147483647); }

int check_row_args(int64_t N, int D) {
    if (N < 0 || D <= 0 || (D & 1)) return ANIMA_ERR_BAD_SHAPE;
    if (N > 0 && (int64_t)D > INT64_MAX / N) return ANIMA_ERR_TOO_LARGE;
    return ANIMA_OK;
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

// Launchers the C entry points hand to dispatch_team (one per row op).
struct LaunchLayerNormOp {
    LayerNormOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        layer_norm_team<LPR, K><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

struct LaunchAdaLNOp {
    AdaLNOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        adaln_team<LPR, K><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

struct LaunchLnModulateOp {
    LnModulateOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        ln_modulate_team<LPR, K><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

struct LaunchResGateAdaLNOp {
    ResGateAdaLNOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        residual_gate_adaln_team<LPR, K><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

struct LaunchRmsOp {
    RmsOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        if (op.weight) rms_norm_team<LPR, K, true><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
        else rms_norm_team<LPR, K, false><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

struct LaunchAdaRmsOp {
    AdaRmsOp op;
    int64_t N;
    cudaStream_t s;
    template <int LPR, int K> void go() {
        adaln_rms_team<LPR, K><<<team_grid(N, LPR), kRowBlock, 0, s>>>(op, N);
    }
};

}  // namespace
}  // namespace anima

using namespace anima;

// ================================================================ C ABI

extern "C" int anima_layer_norm_bf16(const anima_bf16 *x, anima_bf16 *out, int N, int D, float eps,
                                     anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    LayerNormOp op{x, out, D, eps};
    LaunchLayerNormOp l{op, N, stream};
    if (!(aligned16(x) && aligned16(out) && dispatch_team(D, l))) {
        GenArgs a{x, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, out, D, eps};
        row_generic<GenKind::LayerNorm><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_adaln_layernorm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                          const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                                          float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    AdaLNOp op{x, scale, shift, out, D, eps};
    LaunchAdaLNOp l{op, N, stream};
    if (!(aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) && dispatch_team(D, l))) {
        GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
        row_generic<GenKind::AdaLN><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_layer_norm_modulate_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                              const anima_bf16 *shift, anima_bf16 *out, int N,
                                              int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    LnModulateOp op{x, scale, shift, out, D, eps};
    LaunchLnModulateOp l{op, N, stream};
    if (!(aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) && dispatch_team(D, l))) {
        GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
        row_generic<GenKind::LnModulate><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_residual_gate_adaln_bf16(anima_bf16 *hidden, const anima_bf16 *sub_out,
                                              const anima_bf16 *gate, const anima_bf16 *scale,
                                              const anima_bf16 *shift, anima_bf16 *normed, int N,
                                              int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!hidden || !sub_out || !gate || !scale || !shift || !normed) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(hidden) || !bf16_ok(sub_out) || !bf16_ok(gate) || !bf16_ok(scale) ||
        !bf16_ok(shift) || !bf16_ok(normed))
        return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    // normed must be a separate buffer from hidden; sub_out may not overlap either output.
    if (partial_overlap(hidden, n, normed, n) || hidden == normed) return ANIMA_ERR_OVERLAP;
    if (partial_overlap(sub_out, n, hidden, n) || partial_overlap(sub_out, n, normed, n))
        return ANIMA_ERR_OVERLAP;
    ResGateAdaLNOp op{hidden, sub_out, gate, scale, shift, normed, D, eps};
    LaunchResGateAdaLNOp l{op, N, stream};
    if (!(aligned16(hidden) && aligned16(sub_out) && aligned16(gate) && aligned16(scale) &&
          aligned16(shift) && aligned16(normed) && dispatch_team(D, l))) {
        GenArgs a{hidden, hidden, sub_out, gate, scale, shift, nullptr, normed, D, eps};
        row_generic<GenKind::ResGate><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight, anima_bf16 *out,
                                   int N, int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out) || (weight && !bf16_ok(weight))) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    RmsOp op{x, weight, out, D, eps};
    LaunchRmsOp l{op, N, stream};
    if (!(aligned16(x) && aligned16(out) && (!weight || aligned16(weight)) && dispatch_team(D, l))) {
        GenArgs a{x, nullptr, nullptr, nullptr, nullptr, nullptr, weight, out, D, eps};
        row_generic<GenKind::Rms><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_adaln_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                         const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                                         float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n) || partial_overlap(scale, n, out, n) ||
        partial_overlap(shift, n, out, n))
        return ANIMA_ERR_OVERLAP;
    AdaRmsOp op{x, scale, shift, out, D, eps};
    LaunchAdaRmsOp l{op, N, stream};
    if (!(aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) && dispatch_team(D, l))) {
        GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
        row_generic<GenKind::AdaRms><<<generic_grid(N), ref_row_threads(D), 0, stream>>>(a, N);
    }
    return launch_status();
}

extern "C" int anima_gemma_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight,
                                         anima_bf16 *out, int N, int D, float eps,
                                         anima_stream_t stream) {
    if (N < 0 || D <= 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!x || !weight || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(weight) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int threads = (D <= 1024) ? ((D + 31) / 32 * 32) : 1024;
    gemma_rms_generic<<<generic_grid(N), threads, 0, stream>>>(x, weight, out, N, D, eps);
    return launch_status();
}
