// attention.cu -- the glue around the Qwen3 encoder's and the LLM adapter's cuBLAS attention,
// and the VAE attention's softmax (sm_100a):
//
//   head_transpose / head_untranspose [T, H*HD] <-> [H, T, HD]        transpose.cu:13-66
//   head_transpose_batched / _untranspose_batched [B*S, H*HD] <-> [B, H, S, HD]   :68-123
//   expand_kv   [B, KV_H, T, D] -> [B, Q_H, T, D], head q reads kv head q / (Q_H / KV_H)
//                                                                    gemma_ops.cu:99-127
//   causal_mask scores[h, i, j] = bf16(-1e9) for j > i               softmax.cu:62-80
//   softmax     row-wise, bf16 in and out, fp32 arithmetic           softmax.cu:8-60,115-122
//   softmax_f32_to_bf16  row-wise, fp32 in, bf16 out                 softmax.cu:153-252
//
// The permutations and the mask are exact by construction; they move 16-byte chunks when
// the head dimension allows (scalar otherwise), one chunk per thread over one resident wave,
// written in destination order so the stores coalesce. The mask writes only the masked part
// of each row, as the reference does, but one thread per 8 columns instead of a 1024-thread
// CTA per head walking T*T positions with integer division.
//
// softmax: the reference runs a CTA per row with t = min(1024, roundup32(D)) threads; thread
// t sums expf(x - max) over columns t, t + 1024, ... in that order, each warp reduces its 32
// partials with __shfl_down_sync offsets 16..1, and warp 0 reduces the warp sums the same way
// (zero-padded to 32 lanes). Here one warp -- or a team of RL lanes of one warp, when the
// row has at most RL reference warps -- owns a row: team lane w plays reference warp w,
// holding that warp's 32 columns of each 1024-column span in registers, so the warp-level
// tree is an in-register tree and the second level is a shuffle tree across the team. A
// team of RL lanes drops the tree levels whose partners are padding zeros (x + 0 == x), which
// leaves the sum's bits unchanged. The row maximum is order-free (fmaxf). Rows of at most
// 1024 columns are read once: the 32 exponentials stay in registers for the output.
//
// The opt-in causal form applies the mask inside the softmax: masked columns take the value
// the mask would have stored, and 16-byte chunks that are wholly masked are not read.
//
// softmax_f32_to_bf16 folds each element into a running (max, sum) pair per thread and
// merges pairs along the reference's tree; the merge is not associative, so this kernel keeps
// the reference's thread layout (one CTA per row) and its merge expressions, written the same
// way so that nvcc forms the same fused multiply-adds, with 8-byte output stores.
#include "common.cuh"

#include <math.h>

namespace anima {
namespace {

constexpr int kAttBlock = 256;
constexpr float kMaskValue = -1e9f;  // softmax.cu:72, stored as bf16

__device__ __forceinline__ float bf16_at(const anima_bf16 *p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

// ------------------------------------------------------------ head permutations
struct PermArgs {
    const anima_bf16 *src;
    anima_bf16 *dst;
    uint32_t H, S, U;  // heads, sequence length, units (16-byte chunks or elements) per head row
    uint64_t units;    // total units
    bool to_heads;     // [B, S, H, U] -> [B, H, S, U]; otherwise the inverse
};

template <bool kVec, typename Idx>
__global__ void __launch_bounds__(kAttBlock) head_permute_kernel(PermArgs a) {
    pdl_wait();
    const Idx stride = (Idx)gridDim.x * blockDim.x;
    for (Idx q = (Idx)blockIdx.x * blockDim.x + threadIdx.x; q < (Idx)a.units; q += stride) {
        const Idx u = q % a.U, r = q / a.U;  // destination row r, unit u
        Idx src_row;
        if (a.to_heads) {  // r = (b*H + h)*S + s  <-  (b*S + s)*H + h
            const Idx s = r % a.S, bh = r / a.S, h = bh % a.H, b = bh / a.H;
            src_row = (b * a.S + s) * a.H + h;
        } else {  // r = (b*S + s)*H + h  <-  (b*H + h)*S + s
            const Idx h = r % a.H, bs = r / a.H, s = bs % a.S, b = bs / a.S;
            src_row = (b * a.H + h) * a.S + s;
        }
        const Idx from = src_row * a.U + u;
        if constexpr (kVec) {
            st_vec(a.dst + (uint64_t)q * 8, ld_stream(a.src + (uint64_t)from * 8));
        } else {
            reinterpret_cast<uint16_t *>(a.dst)[q] = reinterpret_cast<const uint16_t *>(a.src)[from];
        }
    }
    pdl_launch();
}

int head_permute(const anima_bf16 *src, anima_bf16 *dst, int B, int H, int S, int HD, bool to_heads,
                 cudaStream_t stream) {
    if (B < 0 || H < 0 || S < 0 || HD < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)B * H * S * HD;
    if (n == 0) return ANIMA_OK;
    if (!src || !dst) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(src, 2) || !aligned_to(dst, 2)) return ANIMA_ERR_MISALIGNED;
    if (overlaps(src, n * 2, dst, n * 2)) return ANIMA_ERR_OVERLAP;  // a permutation cannot run in place
    const bool vec = HD % 8 == 0 && aligned16(src) && aligned16(dst);
    PermArgs a{src, dst, (uint32_t)H, (uint32_t)S, (uint32_t)(vec ? HD / 8 : HD), (uint64_t)(vec ? n / 8 : n),
               to_heads};
    const bool narrow = a.units < (1ull << 32);
    const void *k = vec ? (narrow ? (const void *)head_permute_kernel<true, uint32_t>
                                  : (const void *)head_permute_kernel<true, uint64_t>)
                        : (narrow ? (const void *)head_permute_kernel<false, uint32_t>
                                  : (const void *)head_permute_kernel<false, uint64_t>);
    int err = ANIMA_OK;
    const unsigned grid = wave_grid(k, kAttBlock, 0, (int64_t)a.units, &err);
    if (err) return err;
    if (vec && narrow) launch(head_permute_kernel<true, uint32_t>, grid, kAttBlock, 0, stream, a);
    else if (vec) launch(head_permute_kernel<true, uint64_t>, grid, kAttBlock, 0, stream, a);
    else if (narrow) launch(head_permute_kernel<false, uint32_t>, grid, kAttBlock, 0, stream, a);
    else launch(head_permute_kernel<false, uint64_t>, grid, kAttBlock, 0, stream, a);
    return launch_status();
}

// ------------------------------------------------------------------ expand_kv
struct ExpandArgs {
    const anima_bf16 *kv;
    anima_bf16 *out;
    uint64_t P;   // units per head plane (T*D, in chunks or elements)
    uint32_t QH, KVH, ratio;
    uint64_t units;
};

template <bool kVec>
__global__ void __launch_bounds__(kAttBlock) expand_kv_kernel(ExpandArgs a) {
    pdl_wait();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < a.units; q += stride) {
        const uint64_t plane = q / a.P, w = q - plane * a.P;
        const uint64_t b = plane / a.QH, qh = plane - b * a.QH;
        const uint64_t from = (b * a.KVH + qh / a.ratio) * a.P + w;  // gemma_ops.cu:112-115
        if constexpr (kVec) {
            st_vec(a.out + q * 8, ld_stream(a.kv + from * 8));
        } else {
            reinterpret_cast<uint16_t *>(a.out)[q] = reinterpret_cast<const uint16_t *>(a.kv)[from];
        }
    }
    pdl_launch();
}

// ---------------------------------------------------------------- causal mask
struct MaskArgs {
    anima_bf16 *scores;
    uint32_t T, cpr;  // row length, 16-byte chunks per row
    uint64_t chunks;
};

__global__ void __launch_bounds__(kAttBlock) causal_mask_kernel(MaskArgs a) {
    pdl_wait();
    const uint32_t mask2 = pack_bf2(kMaskValue, kMaskValue);
    const uint16_t mask1 = (uint16_t)mask2;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < a.chunks; q += stride) {
        const uint64_t row = q / a.cpr;
        const uint32_t c = (uint32_t)(q - row * a.cpr) * 8, i = (uint32_t)(row % a.T);
        anima_bf16 *p = a.scores + row * a.T + c;
        if (c > i) {  // the whole chunk lies above the diagonal
            st_vec(p, Vec8{{mask2, mask2, mask2, mask2}});
        } else if (c + 7 > i) {  // the diagonal crosses this chunk: columns i+1 .. c+7
            for (uint32_t j = i + 1; j < c + 8; ++j) reinterpret_cast<uint16_t *>(p)[j - c] = mask1;
        }
    }
    pdl_launch();
}

__global__ void __launch_bounds__(kAttBlock) causal_mask_scalar(anima_bf16 *scores, uint32_t T, uint64_t n) {
    pdl_wait();
    const uint16_t mask1 = (uint16_t)pack_bf2(kMaskValue, kMaskValue);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        const uint64_t row = e / T;
        const uint32_t j = (uint32_t)(e - row * T), i = (uint32_t)(row % T);
        if (j > i) reinterpret_cast<uint16_t *>(scores)[e] = mask1;
    }
    pdl_launch();
}

// ------------------------------------------------------------------- softmax
struct SoftmaxArgs {
    const anima_bf16 *x;
    anima_bf16 *out;
    int64_t rows;
    int D;
    int T;       // causal form: row r is query r % T of its head
    int rl_log;  // log2 of the lanes per row
    bool vec;    // 16-byte rows (D % 8 == 0, aligned pointers)
};

// Loads the 32 columns [c0, c0 + 32) of `row` into v (masked columns take the mask value;
// columns at or beyond D are marked absent in `present`, a bit per column).
// kFull: every team lane's 32 columns exist (D == 32 x lanes per row, 16-byte rows).
template <bool kCausal, bool kFull = false>
__device__ __forceinline__ uint32_t load_seg(const SoftmaxArgs &a, const anima_bf16 *xr, int c0, int qi,
                                             float (&v)[32]) {
    uint32_t present = 0;
    const float mv = bf16_round(kMaskValue);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int cc = c0 + 8 * g;
        if (kFull || (a.vec && cc + 8 <= a.D)) {
            if (kCausal && cc > qi) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[8 * g + e] = mv;
            } else {
                float f[8];
                unpack8(ld_cached(xr + cc), f);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[8 * g + e] = (kCausal && cc + e > qi) ? mv : f[e];
            }
            present |= 0xffu << (8 * g);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int c = cc + e;
                if (c < a.D) {
                    v[8 * g + e] = (kCausal && c > qi) ? mv : bf16_at(xr, c);
                    present |= 1u << (8 * g + e);
                } else {
                    v[8 * g + e] = 0.0f;
                }
            }
        }
    }
    return present;
}

// The reference warp's __shfl_down_sync tree over its 32 lanes, result at lane 0
// (cuda_utils.cuh:46-50), run over 32 values in registers.
__device__ __forceinline__ float warp_tree32(float (&t)[32]) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; ++i) t[i] = t[i] + t[i + o];
    return t[0];
}

// kFull (with kCache): rows of exactly 32 columns per team lane, so no lane has absent
// columns and the per-column presence tests drop out (measured 31 instructions per element
// with them at [16 x 512, 512]).
template <bool kCausal, bool kCache, bool kFull = false>
__global__ void __launch_bounds__(kAttBlock) softmax_rows_kernel(SoftmaxArgs a) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int RL = 1 << a.rl_log, w = lane & (RL - 1);  // team lane w plays reference warp w
    const int64_t rpw = 32 >> a.rl_log;                  // rows per warp
    const int64_t gwarp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int spans = kCache ? 1 : (a.D + 1023) / 1024;
    for (int64_t base = gwarp * rpw; base < a.rows; base += nwarp * rpw) {
        const int64_t row = base + (lane >> a.rl_log);
        const bool live = row < a.rows;
        const anima_bf16 *xr = a.x + (live ? row : 0) * (int64_t)a.D;
        const int qi = kCausal ? (int)(row % a.T) : 0;

        // softmax.cu:17-35: the row maximum, starting from -1e30.
        float v[32];
        uint32_t present = 0;
        float mx = -1e30f;
        for (int m = 0; m < spans; ++m) {
            if constexpr (kFull) {  // a row past the end reads row 0 and stores nothing
                load_seg<kCausal, true>(a, xr, 32 * w, qi, v);
#pragma unroll
                for (int k = 0; k < 32; ++k) mx = fmaxf(mx, v[k]);
            } else {
                present = live ? load_seg<kCausal>(a, xr, 1024 * m + 32 * w, qi, v) : 0u;
#pragma unroll
                for (int k = 0; k < 32; ++k)
                    if (present >> k & 1) mx = fmaxf(mx, v[k]);
            }
        }
        for (int o = RL >> 1; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o, RL));

        // softmax.cu:37-54: per reference thread, the sum of its columns' exponentials in
        // column order; then the warp tree in registers and the tree over warps across the team.
        float p[32];
        if constexpr (kFull) {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = expf(v[k] - mx);
                p[k] = v[k];  // 0.0f + e == e
            }
        } else if constexpr (kCache) {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = (present >> k & 1) ? expf(v[k] - mx) : 0.0f;
                p[k] = v[k];  // 0.0f + e == e
            }
        } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) p[k] = 0.0f;
            for (int m = 0; m < spans; ++m) {
                present = live ? load_seg<kCausal>(a, xr, 1024 * m + 32 * w, qi, v) : 0u;
#pragma unroll
                for (int k = 0; k < 32; ++k)
                    if (present >> k & 1) p[k] += expf(v[k] - mx);
            }
        }
        float s = warp_tree32(p);
        for (int o = RL >> 1; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o, RL);
        s = __shfl_sync(0xffffffffu, s, 0, RL);
        const float inv = 1.0f / s;  // softmax.cu:55

        // softmax.cu:57-59: out = bf16(expf(x - max) * inv).
        anima_bf16 *yr = a.out + (live ? row : 0) * (int64_t)a.D;
        for (int m = 0; m < spans && live; ++m) {
            const int c0 = 1024 * m + 32 * w;
            if constexpr (!kCache) {
                present = load_seg<kCausal>(a, xr, c0, qi, v);
#pragma unroll
                for (int k = 0; k < 32; ++k) v[k] = (present >> k & 1) ? expf(v[k] - mx) : 0.0f;
            }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int cc = c0 + 8 * g;
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[8 * g + e] * inv;
                if (kFull || (a.vec && cc + 8 <= a.D)) {
                    st_vec(yr + cc, pack8(f));
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (cc + e < a.D) reinterpret_cast<__nv_bfloat16 *>(yr)[cc + e] = __float2bfloat16_rn(f[e]);
                }
            }
        }
    }
    pdl_launch();
}

int softmax_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t rows, int D, int T, bool causal,
                 cudaStream_t stream) {
    if (rows == 0 || D == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(x, 2) || !aligned_to(out, 2)) return ANIMA_ERR_MISALIGNED;
    const int64_t nb = rows * D * 2;
    if (partial_overlap(x, nb, out, nb)) return ANIMA_ERR_OVERLAP;
    const int ref_warps = D >= 1024 ? 32 : (D + 31) / 32;
    int rl_log = 0;
    while ((1 << rl_log) < ref_warps) ++rl_log;
    SoftmaxArgs a{x, out, rows, D, T, rl_log, D % 8 == 0 && aligned16(x) && aligned16(out)};
    const int64_t warps = (rows + (32 >> rl_log) - 1) >> (5 - rl_log);
    const bool cache = D <= 1024;
    const bool full = cache && a.vec && D == (32 << rl_log);
    const void *k = causal ? (full ? (const void *)softmax_rows_kernel<true, true, true>
                                   : cache ? (const void *)softmax_rows_kernel<true, true>
                                           : (const void *)softmax_rows_kernel<true, false>)
                           : (full ? (const void *)softmax_rows_kernel<false, true, true>
                                   : cache ? (const void *)softmax_rows_kernel<false, true>
                                           : (const void *)softmax_rows_kernel<false, false>);
    int err = ANIMA_OK;
    const unsigned grid = wave_grid(k, kAttBlock, 0, warps * 32, &err);
    if (err) return err;
    if (causal && full) launch(softmax_rows_kernel<true, true, true>, grid, kAttBlock, 0, stream, a);
    else if (causal && cache) launch(softmax_rows_kernel<true, true>, grid, kAttBlock, 0, stream, a);
    else if (causal) launch(softmax_rows_kernel<true, false>, grid, kAttBlock, 0, stream, a);
    else if (full) launch(softmax_rows_kernel<false, true, true>, grid, kAttBlock, 0, stream, a);
    else if (cache) launch(softmax_rows_kernel<false, true>, grid, kAttBlock, 0, stream, a);
    else launch(softmax_rows_kernel<false, false>, grid, kAttBlock, 0, stream, a);
    return launch_status();
}

// ------------------------------------------------------- softmax fp32 -> bf16
// softmax.cu:160-166 and :185-193: one element into a running (max, sum) pair, and the
// merge of two pairs. The expressions are the reference's, in its order.
__device__ __forceinline__ void online_add(float xi, float &m, float &s) {
    if (xi > m) {
        s = s * expf(m - xi) + 1.0f;
        m = xi;
    } else {
        s += expf(xi - m);
    }
}
__device__ __forceinline__ void online_merge(float om, float os, float &m, float &s) {
    if (om > m) {
        s = s * expf(m - om) + os;
        m = om;
    } else {
        s = s + os * expf(om - m);
    }
}

__global__ void softmax_f32_bf16_kernel(const float *__restrict__ x, anima_bf16 *__restrict__ out, int D,
                                        bool vec) {
    pdl_wait();
    const int64_t row = blockIdx.x;
    const float *xr = x + row * D;
    __nv_bfloat16 *yr = reinterpret_cast<__nv_bfloat16 *>(out) + row * D;
    const int D4 = D / 4, t = threadIdx.x, nt = blockDim.x;
    float m = -1e30f, s = 0.0f;
    for (int i = t; i < D4; i += nt) {
        float4 v;
        if (vec) v = reinterpret_cast<const float4 *>(xr)[i];
        else v = make_float4(xr[4 * i], xr[4 * i + 1], xr[4 * i + 2], xr[4 * i + 3]);
        online_add(v.x, m, s);
        online_add(v.y, m, s);
        online_add(v.z, m, s);
        online_add(v.w, m, s);
    }
    for (int i = D4 * 4 + t; i < D; i += nt) online_add(xr[i], m, s);

    // softmax.cu:182-220: shfl_down merge inside each warp, then warp 0 over the warps.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_down_sync(0xffffffffu, m, o), os = __shfl_down_sync(0xffffffffu, s, o);
        online_merge(om, os, m, s);
    }
    __shared__ float s_m[32], s_s[32];
    const int lane = t & 31, warp = t >> 5, nw = (nt + 31) >> 5;
    if (lane == 0) {
        s_m[warp] = m;
        s_s[warp] = s;
    }
    __syncthreads();
    if (warp == 0) {
        m = lane < nw ? s_m[lane] : -1e30f;
        s = lane < nw ? s_s[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_down_sync(0xffffffffu, m, o), os = __shfl_down_sync(0xffffffffu, s, o);
            online_merge(om, os, m, s);
        }
    }
    __syncthreads();
    if (t == 0) {
        s_m[0] = m;
        s_s[0] = s;
    }
    __syncthreads();
    const float mx = s_m[0], inv = 1.0f / s_s[0];
    pdl_launch();

    // softmax.cu:230-244: out = bf16(expf(x - max) * inv), four columns per 8-byte store.
    for (int i = t; i < D4; i += nt) {
        float4 v;
        if (vec) v = reinterpret_cast<const float4 *>(xr)[i];
        else v = make_float4(xr[4 * i], xr[4 * i + 1], xr[4 * i + 2], xr[4 * i + 3]);
        const uint32_t lo = pack_bf2(expf(v.x - mx) * inv, expf(v.y - mx) * inv);
        const uint32_t hi = pack_bf2(expf(v.z - mx) * inv, expf(v.w - mx) * inv);
        if (vec) {
            *reinterpret_cast<uint2 *>(yr + 4 * i) = make_uint2(lo, hi);
        } else {
            yr[4 * i] = __ushort_as_bfloat16((unsigned short)lo);
            yr[4 * i + 1] = __ushort_as_bfloat16((unsigned short)(lo >> 16));
            yr[4 * i + 2] = __ushort_as_bfloat16((unsigned short)hi);
            yr[4 * i + 3] = __ushort_as_bfloat16((unsigned short)(hi >> 16));
        }
    }
    for (int i = D4 * 4 + t; i < D; i += nt) yr[i] = __float2bfloat16_rn(expf(xr[i] - mx) * inv);
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_head_transpose_bf16(const anima_bf16 *src, anima_bf16 *dst, int H, int T, int HD,
                                         anima_stream_t stream) {
    return head_permute(src, dst, 1, H, T, HD, true, stream);
}

extern "C" int anima_head_untranspose_bf16(const anima_bf16 *src, anima_bf16 *dst, int H, int T, int HD,
                                           anima_stream_t stream) {
    return head_permute(src, dst, 1, H, T, HD, false, stream);
}

extern "C" int anima_head_transpose_batched_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int H, int S,
                                                 int HD, anima_stream_t stream) {
    return head_permute(src, dst, B, H, S, HD, true, stream);
}

extern "C" int anima_head_untranspose_batched_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int H, int S,
                                                   int HD, anima_stream_t stream) {
    return head_permute(src, dst, B, H, S, HD, false, stream);
}

extern "C" int anima_expand_kv_bf16(const anima_bf16 *kv, anima_bf16 *out, int B, int KV_H, int Q_H, int T, int D,
                                    anima_stream_t stream) {
    if (B < 0 || KV_H < 0 || Q_H < 0 || T < 0 || D < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)B * Q_H * T * D;
    if (n == 0) return ANIMA_OK;
    if (KV_H == 0 || Q_H % KV_H != 0) return ANIMA_ERR_BAD_SHAPE;  // each q head maps to one kv head
    if (!kv || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(kv, 2) || !aligned_to(out, 2)) return ANIMA_ERR_MISALIGNED;
    if (overlaps(kv, (int64_t)B * KV_H * T * D * 2, out, n * 2)) return ANIMA_ERR_OVERLAP;
    const int64_t plane = (int64_t)T * D;
    const bool vec = plane % 8 == 0 && aligned16(kv) && aligned16(out);
    ExpandArgs a{kv, out, (uint64_t)(vec ? plane / 8 : plane), (uint32_t)Q_H, (uint32_t)KV_H,
                 (uint32_t)(Q_H / KV_H), (uint64_t)(vec ? n / 8 : n)};
    int err = ANIMA_OK;
    const void *k = vec ? (const void *)expand_kv_kernel<true> : (const void *)expand_kv_kernel<false>;
    const unsigned grid = wave_grid(k, kAttBlock, 0, (int64_t)a.units, &err);
    if (err) return err;
    if (vec) launch(expand_kv_kernel<true>, grid, kAttBlock, 0, stream, a);
    else launch(expand_kv_kernel<false>, grid, kAttBlock, 0, stream, a);
    return launch_status();
}

extern "C" int anima_causal_mask_bf16(anima_bf16 *scores, int num_heads, int T, anima_stream_t stream) {
    if (num_heads < 0 || T < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)num_heads * T * T;
    if (n == 0) return ANIMA_OK;
    if (!scores) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(scores, 2)) return ANIMA_ERR_MISALIGNED;
    int err = ANIMA_OK;
    if (T % 8 == 0 && aligned16(scores)) {
        MaskArgs a{scores, (uint32_t)T, (uint32_t)(T / 8), (uint64_t)(n / 8)};
        const unsigned grid = wave_grid((const void *)causal_mask_kernel, kAttBlock, 0, n / 8, &err);
        if (err) return err;
        launch(causal_mask_kernel, grid, kAttBlock, 0, stream, a);
    } else {
        const unsigned grid = wave_grid((const void *)causal_mask_scalar, kAttBlock, 0, n, &err);
        if (err) return err;
        launch(causal_mask_scalar, grid, kAttBlock, 0, stream, scores, (uint32_t)T, (uint64_t)n);
    }
    return launch_status();
}

extern "C" int anima_softmax_bf16(const anima_bf16 *x, anima_bf16 *out, int N, int D, anima_stream_t stream) {
    if (N < 0 || D < 0) return ANIMA_ERR_BAD_SHAPE;
    return softmax_bf16(x, out, N, D, 1, false, stream);
}

extern "C" int anima_causal_softmax_bf16(const anima_bf16 *scores, anima_bf16 *out, int num_heads, int T,
                                         anima_stream_t stream) {
    if (num_heads < 0 || T < 0) return ANIMA_ERR_BAD_SHAPE;
    return softmax_bf16(scores, out, (int64_t)num_heads * T, T, T, true, stream);
}

extern "C" int anima_softmax_f32_to_bf16(const float *x, anima_bf16 *out, int N, int D, anima_stream_t stream) {
    if (N < 0 || D < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0 || D == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(x, 4) || !aligned_to(out, 2)) return ANIMA_ERR_MISALIGNED;
    if (overlaps(x, (int64_t)N * D * 4, out, (int64_t)N * D * 2)) return ANIMA_ERR_OVERLAP;
    if (N > 2147483647) return ANIMA_ERR_TOO_LARGE;
    // The reference launches min(roundup32(D), 1024) threads per row (softmax.cu:248-249), so
    // for D <= 4096 thread t holds float4 t and nothing else, and the threads past D/4 -- whole
    // warps of them, 12 of 16 at D = 512 -- carry the empty pair (-1e30, 0), which every merge
    // passes through unchanged: merging it into (m, s) leaves (m, s), and merging (m, s) into
    // it yields (m, s). Launching only the warps that hold columns therefore gives the same
    // bits (warp 0's padding supplies the same empty pairs for the missing warps) with a
    // quarter of the threads and no idle warps at D = 512.
    const int ref_threads = D <= 1024 ? (D + 31) / 32 * 32 : 1024;
    const int used = (D / 4 + 31) / 32 * 32;
    const int threads = D <= 4096 ? (used < 32 ? 32 : used) : ref_threads;
    const bool vec = D % 4 == 0 && aligned16(x) && aligned_to(out, 8);
    launch(softmax_f32_bf16_kernel, (unsigned)N, threads, 0, stream, x, out, D, vec);
    return launch_status();
}
