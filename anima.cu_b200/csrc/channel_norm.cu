// channel_norm.cu -- VAE channel RMSNorm (+ optional fused SiLU) on NCHW bf16 (sm_100a).
//
// out[b,c,s] = x[b,c,s] * rsqrt(mean_c x[b,:,s]^2 + eps) * gamma[c]      (vae_kernels.cu:60-81)
// and its ungated sibling, the pixel norm (kPixel):
// out[b,c,s] = x[b,c,s] * (1 / sqrt(mean_c x[b,:,s]^2 + eps))              (vae_kernels.cu:15-52)
//
// The reduction runs over channels, which sit `spatial` elements apart. The reference
// gives each pixel a thread that walks the channels with 2-byte strided loads, twice
// (once for the sum, once for the output), launched once per batch item.
//
// Here one CTA owns a tile of P consecutive pixels x all C channels of one image (P = 64 for
// C <= 256, 32 for C = 512, 16 beyond, so that a tile stays <= 64 KB; the CTA has P*C/64
// threads, clamped to 64..256, i.e. eight 16-byte chunks of the tile per thread). The tile is
// staged into shared memory with 16-byte cp.async copies (each channel contributes one
// contiguous 2P-byte segment). Then P/2 lanes walk the channels, two adjacent pixels per lane
// with one 32-bit shared load and one packed fp32x2 fma per channel, in channel order -- the
// reference's own summation order per pixel, so statistics and outputs match it bit for bit.
// Finally every thread scales its eight chunks out of shared memory (its pixels' rms held in
// registers, gamma staged in shared memory as fp32) with 16-byte stores, the fused SiLU
// through the decided fast path of activation.cuh. x crosses HBM once and out once. Measured
// against the previous layout (64 threads walking one pixel each with 2-byte loads, 256
// threads per CTA at every C): the norm alone 85.9 against 93.5 us at [128, 1024^2] (0.96 of
// the measured peak), fused with SiLU 124 against 141 us.
//
// When the tiles are few, channel_norm_cluster (below) spreads each over a cluster of CTAs.
// Where it measured faster (the fused SiLU at C <= 512, the norm alone at C = 512),
// channel_norm_tma stages the tile with TMA bulk tensor loads, one per 64 channels on its own
// mbarrier, so the chain starts while the rest of the tile is still arriving.
//
// The conv-bias form (kBias) first adds the convolution's bias[c] to the staged tile in place,
// rounded to bf16 as the reference's bias launch stores it (causal_conv3d.cu:187-195); the
// bias is loaded into shared memory while the tile's copies are in flight.
//
// Tensors whose rows are not 16-byte aligned (spatial % 8 != 0) or whose tile would not
// fit in shared memory use the generic kernel: one thread per pixel, the reference's
// arithmetic, one launch for all batch items.
#include "common.cuh"
#include "activation.cuh"
#include "tma.cuh"

#include <cooperative_groups.h>

namespace anima {
namespace {

constexpr int kCnPix = 64;                  // pixels per tile of the cluster kernel
constexpr int kCnBlock = 256;               // threads per CTA of the cluster kernel (and the tile kernel's maximum)
constexpr int kCnMaxSmem = 200 * 1024;      // tile bytes we allow per CTA

// Tile width of the tile kernel for C channels, 16..64 pixels, and its CTA size (64, 128 or
// 256 threads), from a sweep at the VAE decoder's shapes. With the SiLU epilogue: tiles of
// <= 32 KB and about eight 16-byte chunks per thread (the epilogue wants many tiles in
// flight); the norm alone: tiles of <= 64 KB and about four chunks per thread.
inline int cn_tile_pix(int C, bool silu) {
    return silu ? (C <= 256 ? 64 : C <= 512 ? 32 : 16) : (C <= 512 ? 64 : C <= 1024 ? 32 : 16);
}
inline int cn_tile_threads(int C, int P, bool silu) {
    const int64_t t = (int64_t)P * C / (silu ? 64 : 32);
    return t <= 64 ? 64 : t <= 128 ? 128 : 256;
}

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// causal_conv3d.cu:193 on a staged 16-byte chunk in shared memory: x + bias[c], rounded to
// bf16 as the reference's bias launch stores it. The reference adds in fp32 and rounds to
// bf16; for two bf16 operands that is the exact sum rounded once (when their exponents are at
// most 16 apart the fp32 sum is exact, and otherwise the smaller addend lies far below half a
// bf16 ulp of the larger, which both roundings then return), so a packed bf16 add gives the
// same bits in a quarter of the instructions.
__device__ __forceinline__ uint32_t bias_pair(const anima_bf16 *p) {
    const uint32_t h = *reinterpret_cast<const unsigned short *>(p);
    return h | (h << 16);
}
__device__ __forceinline__ void add_bias8(anima_bf16 *chunk, uint32_t b2) {
    Vec8 &v = *reinterpret_cast<Vec8 *>(chunk);
#pragma unroll
    for (int j = 0; j < 4; ++j) asm("add.rn.bf16x2 %0, %0, %1;" : "+r"(v.w[j]) : "r"(b2));
}

// vae_kernels.cu:71, q += x*x for the two pixels of a packed bf16 pair: sm_100's mixed-precision
// fma takes the bf16 halves as multiplicands and the fp32 sum as addend and rounds once, which
// is fmaf(float(x), float(x), q) exactly (the conversion is exact), in two instructions where
// unpacking and a packed fp32x2 fma take three -- this serial chain is the kernels' critical
// path.
__device__ __forceinline__ float sq_acc_bf16(unsigned short x, float q) {
    float r;
    asm("{\n .reg .b16 t;\n mov.b16 t, %1;\n fma.rn.f32.bf16 %0, t, t, %2;\n}\n" : "=f"(r) : "h"(x), "f"(q));
    return r;
}
__device__ __forceinline__ void sq_acc_bf16x2(uint32_t w, float2 &q) {
    asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n fma.rn.f32.bf16 %0, l, l, %0;\n fma.rn.f32.bf16 %1, h, h, %1;\n}\n"
        : "+f"(q.x), "+f"(q.y)
        : "r"(w));
}

struct CnArgs {
    const anima_bf16 *x, *gamma;
    anima_bf16 *out;
    const anima_bf16 *bias;  // the convolution's bias[C], added first (kBias kernels only)
    int C, spatial;
    float eps;
    int tiles_per_image;
};

// The per-pixel scale from the sum of squares q: rsqrtf for the channel norm
// (vae_kernels.cu:74); 1.0f / sqrtf(...) in IEEE arithmetic for the pixel norm
// (vae_kernels.cu:30-31).
template <bool kPixel>
__device__ __forceinline__ float norm_scale(float q, int C, float eps) {
    const float m = __fdiv_rn(q, (float)C) + eps;
    return kPixel ? __fdiv_rn(1.0f, __fsqrt_rn(m)) : rsqrtf(m);
}

// vae_kernels.cu:75-80 on one staged 16-byte chunk (8 pixels of one channel): (x * rms) * gamma,
// rounded to bf16.
__device__ __forceinline__ Vec8 norm_chunk(const anima_bf16 *chunk, const float *rms_s, int v, float gm) {
    const Vec8 xv = *reinterpret_cast<const Vec8 *>(chunk);
    const float4 r0 = reinterpret_cast<const float4 *>(rms_s)[2 * v];
    const float4 r1 = reinterpret_cast<const float4 *>(rms_s)[2 * v + 1];
    const float r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    Vec8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 t = __fmul2_rn(make_float2(bf_lo(xv.w[j]), bf_hi(xv.w[j])), make_float2(r[2 * j], r[2 * j + 1]));
        const float2 u = __fmul2_rn(t, make_float2(gm, gm));
        o.w[j] = pack_bf2(u.x, u.y);
    }
    return o;
}

// The tile kernel (see the header): P pixels x C channels per CTA, T threads (a compile-time
// constant, so that the epilogue's channel loop has a fixed stride: measured faster than the
// same kernel with the CTA size read at run time).
// Shared memory: gamma as fp32 [C], the per-pixel rms [P], then the tile [C][P] (+ the
// conv-bias pairs [C] for kBias).
template <int P, int T, bool kSilu, bool kBias, bool kPixel>
__global__ void __launch_bounds__(T) channel_norm_tile(CnArgs a) {
    pdl_wait();
    constexpr int kVecs = P / 8;  // 16-byte chunks per channel row of the tile
    extern __shared__ __align__(16) unsigned char cn_smem[];
    float *gam = reinterpret_cast<float *>(cn_smem);            // [C]
    float *rms_s = gam + ((a.C + 3) & ~3);                      // [P]
    anima_bf16 *tile = reinterpret_cast<anima_bf16 *>(rms_s + P);  // [C][P]
    constexpr int nthr = T;
    const int b = blockIdx.x / a.tiles_per_image;
    const int s_tile = (blockIdx.x - b * a.tiles_per_image) * P;
    const int live_vecs = min(P, a.spatial - s_tile) / 8;  // spatial % 8 == 0
    const int64_t img = (int64_t)b * a.C * a.spatial;
    const int nchunks = a.C * kVecs;

    // Stage: chunk q = (channel q / kVecs, pixel vector q % kVecs) lands at tile + 8q.
    const anima_bf16 *src = a.x + img + s_tile;
    for (int q = threadIdx.x; q < nchunks; q += nthr) {
        const int c = q / kVecs, v = q % kVecs;
        if (v < live_vecs) cp_async16(tile + q * 8, src + (int64_t)c * a.spatial + v * 8);
    }
    uint32_t *bias_s = reinterpret_cast<uint32_t *>(tile + a.C * P);  // [C] (b, b) pairs (kBias)
    if constexpr (kBias) {  // loads in flight with the tile's copies
        for (int c = threadIdx.x; c < a.C; c += nthr) bias_s[c] = bias_pair(a.bias + c);
    }
    if constexpr (!kPixel) {
        for (int c = threadIdx.x; c < a.C; c += nthr) gam[c] = ldb(a.gamma + c);
    }
    cp_async_wait_all();
    __syncthreads();
    if constexpr (kBias) {
        for (int q = threadIdx.x; q < nchunks; q += nthr) {
            const int c = q / kVecs, v = q % kVecs;
            if (v < live_vecs) add_bias8(tile + q * 8, bias_s[c]);
        }
        __syncthreads();
    }

    // vae_kernels.cu:68-74: each pixel's sum of squares over the channels in order; lane t
    // walks pixels 2t and 2t+1 with one packed fma per channel (each lane of FFMA2 rounds like
    // the scalar fma), the next 8 channels' loads issued before the current 8 fmas.
    if (threadIdx.x < P / 2) {
        const uint32_t *col = reinterpret_cast<const uint32_t *>(tile) + threadIdx.x;
        float2 q2 = make_float2(0.0f, 0.0f);
        const int full = a.C & ~7;
        uint32_t cur[8];
        if (full > 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = col[j * (P / 2)];
        }
        for (int c = 0; c < full; c += 8) {
            uint32_t nxt[8];
            const bool more = c + 8 < full;
            if (more) {
#pragma unroll
                for (int j = 0; j < 8; ++j) nxt[j] = col[(c + 8 + j) * (P / 2)];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) sq_acc_bf16x2(cur[j], q2);
            if (more) {
#pragma unroll
                for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
            }
        }
        for (int c = full; c < a.C; ++c) {
            sq_acc_bf16x2(col[c * (P / 2)], q2);
        }
        // pixels beyond the tile's live width hold no data: their values are never used
        reinterpret_cast<float2 *>(rms_s)[threadIdx.x] =
            make_float2(norm_scale<kPixel>(q2.x, a.C, a.eps), norm_scale<kPixel>(q2.y, a.C, a.eps));
    }
    __syncthreads();
    pdl_launch();

    // vae_kernels.cu:75-80: out = (x * rms) * gamma[c], from shared memory; SiLU (silu.cu)
    // of the stored bf16 value when fused. Thread t owns pixel vector v = t % kVecs of
    // channels t / kVecs, t / kVecs + nthr / kVecs, ...
    const int v = threadIdx.x % kVecs;
    if (v >= live_vecs) return;
    float r[8];
    {
        const float4 r0 = reinterpret_cast<const float4 *>(rms_s)[2 * v];
        const float4 r1 = reinterpret_cast<const float4 *>(rms_s)[2 * v + 1];
        r[0] = r0.x; r[1] = r0.y; r[2] = r0.z; r[3] = r0.w;
        r[4] = r1.x; r[5] = r1.y; r[6] = r1.z; r[7] = r1.w;
    }
    anima_bf16 *dst = a.out + img + s_tile + v * 8;
    for (int c = threadIdx.x / kVecs; c < a.C; c += nthr / kVecs) {
        const Vec8 xv = *reinterpret_cast<const Vec8 *>(tile + c * P + v * 8);
        // the pixel norm has no gamma: a factor of exactly 1 leaves x * rms as it is
        const float gm = kPixel ? 1.0f : gam[c];
        Vec8 o;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t2 = __fmul2_rn(make_float2(bf_lo(xv.w[j]), bf_hi(xv.w[j])), make_float2(r[2 * j], r[2 * j + 1]));
            const float2 u = __fmul2_rn(t2, make_float2(gm, gm));
            o.w[j] = pack_bf2(u.x, u.y);
        }
        if constexpr (kSilu) o = fast_chunk<SiluF>(o);
        st_vec(dst + (int64_t)c * a.spatial, o);
    }
}

// The TMA tile kernel's shapes (pixels per tile, threads, channels per load group), chosen by
// kernel experiments at the VAE decoder's shapes against the cp.async tile kernel: with the
// SiLU epilogue it won at C = 128, 256 and 512 (105.3 against 110.6 us at [128, 1024^2],
// 60.6 against 64.9 at [256, 512^2], 43.1 against 47.9 at [512, 256^2]); the norm alone only
// at C = 512 (32.0 against 33.6 us at [512, 256^2]), elsewhere it tied. P = 0: not used.
struct CnTmaShape {
    int P, T, CG, id;
};
inline CnTmaShape cn_tma_shape(int C, bool silu, bool few_tiles) {
    if (silu) {
        if (C <= 128) return {64, 128, 64, 0};
        if (C <= 256) return {64, 256, 64, 1};
        if (C <= 512) return {32, 256, 64, 2};
        return {0, 0, 64, 0};
    }
    // at most ~2 tiles per SM: 512 threads per tile (10.5 against 12.2 us at [512, 128^2])
    if (C > 256 && C <= 512) return few_tiles ? CnTmaShape{64, 512, 64, 3} : CnTmaShape{64, 256, 64, 1};
    return {0, 0, 64, 0};
}

// Waits of the TMA tile kernel that ran out (never expected; read by anima_wait_timeouts).
__device__ unsigned int g_cn_wait_timeouts;

// The tile kernel with the tile staged by the TMA unit: one 3-D bulk tensor load per group of
// CG channels ([CG][P] boxes of the [B][C][spatial] tensor, this GPU's memory, no multicast),
// each completing on its own mbarrier. The P/2 chain lanes start on the first group as soon as
// it lands and wait for each next group only when they reach it, so the serial per-pixel chain
// runs while the rest of the tile is still arriving, and no thread spends issue slots on
// per-chunk copy addresses. Same chain order, epilogue and rounding as channel_norm_tile.
// Shared memory: the tile [C][P] at a 1024-byte boundary, gamma fp32 [C], rms [P], barriers.
template <int P, int T, bool kSilu, bool kBias, bool kPixel, int CG>
__global__ void __launch_bounds__(T) channel_norm_tma(const __grid_constant__ CUtensorMap xmap, CnArgs a) {
    constexpr int kVecs = P / 8;
    extern __shared__ unsigned char cn_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(cn_raw) + 1023) & ~uintptr_t(1023));
    anima_bf16 *tile = reinterpret_cast<anima_bf16 *>(base);                   // [C][P]
    float *gam = reinterpret_cast<float *>(base + (size_t)a.C * P * 2);        // [C]
    float *rms_s = gam + ((a.C + 3) & ~3);                                      // [P]
    uint64_t *bars = reinterpret_cast<uint64_t *>(rms_s + P);                  // [C / CG]
    const int groups = a.C / CG;
    uint32_t *bias_s = reinterpret_cast<uint32_t *>(bars + groups);            // [C] (b, b) pairs (kBias)
    const int b = blockIdx.x / a.tiles_per_image;
    const int s_tile = (blockIdx.x - b * a.tiles_per_image) * P;
    const int live_vecs = min(P, a.spatial - s_tile) / 8;  // spatial % 8 == 0
    const int64_t img = (int64_t)b * a.C * a.spatial;
    if (threadIdx.x == 0) {
        for (int g = 0; g < groups; ++g) mbar_init(&bars[g], 1);
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();
    if (threadIdx.x == 0) {
        for (int g = 0; g < groups; ++g) {
            mbar_arrive_expect_tx(&bars[g], (uint32_t)(CG * P * 2));  // out-of-range pixels arrive as zeros
            tma_load_3d(tile + (size_t)g * CG * P, &xmap, s_tile, g * CG, b, &bars[g]);
        }
    }
    if constexpr (!kPixel) {
        for (int c = threadIdx.x; c < a.C; c += T) gam[c] = ldb(a.gamma + c);
    }
    if constexpr (kBias) {
        // the conv bias is added to each value where it is read (the chain, the epilogue), with
        // the in-place pass's rounding (add_bias8), so no pass over the whole tile precedes the
        // chain and the chain can still start on the first group
        for (int c = threadIdx.x; c < a.C; c += T) bias_s[c] = bias_pair(a.bias + c);
        __syncthreads();
    }
    bool ok = true;
    // vae_kernels.cu:68-74 as in channel_norm_tile: lane t walks pixels 2t, 2t+1 over the channels
    // in order, one packed fma per channel, the next 8 channels' loads ahead within a group.
    if (threadIdx.x < P / 2) {
        const uint32_t *col = reinterpret_cast<const uint32_t *>(tile) + threadIdx.x;
        float2 q2 = make_float2(0.0f, 0.0f);
        for (int g = 0; g < groups; ++g) {
            ok = mbar_wait(&bars[g], 0) && ok;
            const int c0 = g * CG, c1 = c0 + CG;
            uint32_t cur[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = col[(c0 + j) * (P / 2)];
            for (int c = c0; c < c1; c += 8) {
                uint32_t nxt[8];
                const bool more = c + 8 < c1;
                if (more) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) nxt[j] = col[(c + 8 + j) * (P / 2)];
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t w = cur[j];
                    if constexpr (kBias) asm("add.rn.bf16x2 %0, %0, %1;" : "+r"(w) : "r"(bias_s[c + j]));
                    sq_acc_bf16x2(w, q2);
                }
                if (more) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
                }
            }
        }
        reinterpret_cast<float2 *>(rms_s)[threadIdx.x] =
            make_float2(norm_scale<kPixel>(q2.x, a.C, a.eps), norm_scale<kPixel>(q2.y, a.C, a.eps));
    }
    __syncthreads();
    // every thread observes the completed groups before reading the tile (completed phases
    // return at once)
    for (int g = 0; g < groups; ++g) ok = mbar_wait(&bars[g], 0) && ok;
    if (!ok) atomicAdd(&g_cn_wait_timeouts, 1u);
    pdl_launch();
    if (!ok) return;

    const int v = threadIdx.x % kVecs;
    if (v >= live_vecs) return;
    float r[8];
    {
        const float4 r0 = reinterpret_cast<const float4 *>(rms_s)[2 * v];
        const float4 r1 = reinterpret_cast<const float4 *>(rms_s)[2 * v + 1];
        r[0] = r0.x; r[1] = r0.y; r[2] = r0.z; r[3] = r0.w;
        r[4] = r1.x; r[5] = r1.y; r[6] = r1.z; r[7] = r1.w;
    }
    anima_bf16 *dst = a.out + img + s_tile + v * 8;
    for (int c = threadIdx.x / kVecs; c < a.C; c += T / kVecs) {
        Vec8 xv = *reinterpret_cast<const Vec8 *>(tile + c * P + v * 8);
        if constexpr (kBias) {
            const uint32_t b2 = bias_s[c];
#pragma unroll
            for (int j = 0; j < 4; ++j) asm("add.rn.bf16x2 %0, %0, %1;" : "+r"(xv.w[j]) : "r"(b2));
        }
        const float gm = kPixel ? 1.0f : gam[c];
        Vec8 o;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t2 = __fmul2_rn(make_float2(bf_lo(xv.w[j]), bf_hi(xv.w[j])), make_float2(r[2 * j], r[2 * j + 1]));
            const float2 u = __fmul2_rn(t2, make_float2(gm, gm));
            o.w[j] = pack_bf2(u.x, u.y);
        }
        if constexpr (kSilu) o = fast_chunk<SiluF>(o);
        st_vec(dst + (int64_t)c * a.spatial, o);
    }
}

// Cluster variant: a 64-pixel tile is spread over a cluster of kCnCluster CTAs, CTA r staging
// channels [r*Cq, (r+1)*Cq) (Cq = ceil(C / kCnCluster)) into its own shared memory, so loading
// and the epilogue run on kCnCluster times more threads -- what the small VAE shapes (few tiles
// per SM) lack. The per-pixel sum stays one serial chain in the reference's channel order: CTA
// 0 sums its slice, hands the 64 partial sums to CTA 1 through distributed shared memory, CTA 1
// continues over its slice, and so on; the last CTA forms the rms and writes it into every
// CTA. Every read of x is local. One cluster barrier per hand-off, reached by every thread of
// every CTA; the last also keeps each CTA's shared memory alive until all writes into it are
// done.
constexpr int kCnCluster = 4;

template <bool kSilu, bool kBias, bool kPixel>
__global__ void __launch_bounds__(kCnBlock) channel_norm_cluster(CnArgs a, int Cq) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    pdl_wait();
    constexpr int kVecs = kCnPix / 8;
    extern __shared__ __align__(16) anima_bf16 tile[];  // [Cq][kCnPix]: this CTA's channel slice
    __shared__ __align__(16) float rms_s[kCnPix];
    const unsigned rank = cluster.block_rank();
    const int64_t t = blockIdx.x / kCnCluster;  // tile index
    const int b = (int)(t / a.tiles_per_image);
    const int s_tile = (int)(t - (int64_t)b * a.tiles_per_image) * kCnPix;
    const int live_vecs = min(kCnPix, a.spatial - s_tile) / 8;
    const int64_t img = (int64_t)b * a.C * a.spatial;
    const int c0 = (int)rank * Cq, c1 = min(a.C, c0 + Cq);
    const int nchunks = max(0, c1 - c0) * kVecs;

    for (int q = threadIdx.x; q < nchunks; q += kCnBlock) {
        const int c = q / kVecs, v = q % kVecs;
        if (v < live_vecs)
            cp_async16(tile + c * kCnPix + v * 8, a.x + img + (int64_t)(c0 + c) * a.spatial + s_tile + v * 8);
    }
    uint32_t *bias_s = reinterpret_cast<uint32_t *>(tile + Cq * kCnPix);  // [Cq] (b, b) pairs (kBias)
    if constexpr (kBias) {
        for (int c = threadIdx.x; c < c1 - c0; c += kCnBlock) bias_s[c] = bias_pair(a.bias + c0 + c);
    }
    cp_async_wait_all();
    __syncthreads();
    if constexpr (kBias) {
        for (int q = threadIdx.x; q < nchunks; q += kCnBlock) {
            const int c = q / kVecs, v = q % kVecs;
            if (v < live_vecs) add_bias8(tile + c * kCnPix + v * 8, bias_s[c]);
        }
        __syncthreads();
    }

    __shared__ float part_s[kCnPix];  // the chain's partial sums, handed over by CTA rank - 1
    for (int r = 0; r < kCnCluster; ++r) {  // slices in channel order
        if (rank == (unsigned)r && threadIdx.x < kCnPix) {
            const int p = threadIdx.x;
            float q = r == 0 ? 0.0f : part_s[p];
            if (p < live_vecs * 8) {
                const unsigned short *col = reinterpret_cast<const unsigned short *>(tile) + p;
                const int n = c1 - c0, full = n & ~7;
                for (int c = 0; c < full; c += 8) {
                    unsigned short f[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) f[j] = col[(c + j) * kCnPix];
#pragma unroll
                    for (int j = 0; j < 8; ++j) q = sq_acc_bf16(f[j], q);
                }
                for (int c = full; c < n; ++c) q = sq_acc_bf16(col[c * kCnPix], q);
            }
            if (r + 1 < kCnCluster) {
                cluster.map_shared_rank(part_s, r + 1)[p] = q;
            } else {
                const float rv = norm_scale<kPixel>(q, a.C, a.eps);
                for (int k = 0; k < kCnCluster; ++k) cluster.map_shared_rank(rms_s, k)[p] = rv;
            }
        }
        cluster.sync();
    }
    pdl_launch();

    for (int q = threadIdx.x; q < nchunks; q += kCnBlock) {
        const int c = q / kVecs, v = q % kVecs;
        if (v >= live_vecs) continue;
        const Vec8 xv = *reinterpret_cast<const Vec8 *>(tile + c * kCnPix + v * 8);
        const float4 r0 = reinterpret_cast<const float4 *>(rms_s)[2 * v];
        const float4 r1 = reinterpret_cast<const float4 *>(rms_s)[2 * v + 1];
        const float r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        const float gm = kPixel ? 1.0f : ldb(a.gamma + c0 + c);
        Vec8 o;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t2 = __fmul2_rn(make_float2(bf_lo(xv.w[j]), bf_hi(xv.w[j])), make_float2(r[2 * j], r[2 * j + 1]));
            const float2 u = __fmul2_rn(t2, make_float2(gm, gm));
            o.w[j] = pack_bf2(u.x, u.y);
        }
        if constexpr (kSilu) o = fast_chunk<SiluF>(o);
        st_vec(a.out + img + (int64_t)(c0 + c) * a.spatial + s_tile + v * 8, o);
    }
}

// Reference-order kernel for any shape: one thread per (image, pixel).
template <bool kSilu, bool kBias, bool kPixel>
__global__ void channel_norm_serial(CnArgs a, int64_t pixels) {
    pdl_wait();
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pixels;
         p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = p / a.spatial, s = p % a.spatial;
        const anima_bf16 *xb = a.x + b * a.C * (int64_t)a.spatial;
        anima_bf16 *ob = a.out + b * a.C * (int64_t)a.spatial;
        const auto xin = [&](int c) {
            const float f = ldb(xb + (int64_t)c * a.spatial + s);
            return kBias ? bf16_round(f + ldb(a.bias + c)) : f;
        };
        float q = 0.0f;
        for (int c = 0; c < a.C; ++c) {
            const float f = xin(c);
            q = __fmaf_rn(f, f, q);
        }
        const float r = norm_scale<kPixel>(q, a.C, a.eps);
        for (int c = 0; c < a.C; ++c) {
            const int64_t i = (int64_t)c * a.spatial + s;
            float o = kPixel ? xin(c) * r : (xin(c) * r) * ldb(a.gamma + c);
            if constexpr (kSilu) o = silu_f(bf16_round(o));
            *reinterpret_cast<__nv_bfloat16 *>(ob + i) = __float2bfloat16_rn(o);
        }
    }
}

template <bool kSilu, bool kBias = false, bool kPixel = false>
int channel_norm(const anima_bf16 *x, const anima_bf16 *gamma, anima_bf16 *out, int B, int C,
                 int spatial, float eps, cudaStream_t stream, const anima_bf16 *bias = nullptr) {
    if (B < 0 || C <= 0 || spatial < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)B * C * spatial;
    if (n == 0) return ANIMA_OK;
    if (!x || (!kPixel && !gamma) || !out || (kBias && !bias)) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(x, 2) || (!kPixel && !aligned_to(gamma, 2)) || !aligned_to(out, 2) ||
        (kBias && !aligned_to(bias, 2)))
        return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(x, n * 2, out, n * 2) || (!kPixel && partial_overlap(gamma, (int64_t)C * 2, out, n * 2)) ||
        (kBias && overlaps(bias, (int64_t)C * 2, out, n * 2)))
        return ANIMA_ERR_OVERLAP;
    const int P = cn_tile_pix(C, kSilu);
    CnArgs a{x, gamma, out, bias, C, spatial, eps, (spatial + P - 1) / P};
    const int64_t tiles = (int64_t)B * a.tiles_per_image;
    // tile kernel shared bytes: gamma (fp32) + rms + tile rows (+ bias pairs)
    const int64_t smem = (int64_t)((C + 3) & ~3) * 4 + (int64_t)P * 4 + (int64_t)C * (P * 2 + (kBias ? 4 : 0));
    const int64_t per_ch = kCnPix * 2 + (kBias ? 4 : 0);  // cluster kernel: shared bytes per channel
    const int Cq = (C + kCnCluster - 1) / kCnCluster;
    const int64_t cl_tiles = (int64_t)B * ((spatial + kCnPix - 1) / kCnPix);
    int err = ANIMA_OK;
    // Few tiles (at most two per SM): the fused SiLU forms spread each over a cluster (their
    // epilogue needs the threads). Many tiles keep every SM busy already, and the cluster's
    // hand-offs would then only serialise each tile (measured); the norm alone runs the tile
    // kernel at every size (13.0 against 14.7 us on the cluster at [512, 128^2]).
    const bool cluster = kSilu && spatial % 8 == 0 && aligned16(x) && aligned16(out) && C >= 64 &&
                         (int64_t)Cq * per_ch <= kCnMaxSmem && cl_tiles <= 2 * (int64_t)sm_count();
    // The TMA tile kernel where it measured faster than the cp.async one (see cn_tma_shape).
    const bool few_tiles = cl_tiles <= 2 * (int64_t)sm_count();
    // Few tiles, large tensor, C in (256, 512]: the fused SiLU forms run the TMA norm (512
    // threads per tile) and then the SiLU table kernel in place, 14 us against 17 us for the
    // one-launch cluster kernel at [512, 128^2]: with 1.7 tiles per SM the fused epilogue's
    // decided-path SiLU runs on too few warps, the table kernel on every SM. Same bits.
    if (kSilu && !kPixel && cluster && C > 256 && C <= 512 && C % 64 == 0 && n >= (int64_t)1 << 22) {
        if (int e = channel_norm<false, kBias, kPixel>(x, gamma, out, B, C, spatial, eps, stream, bias)) return e;
        return anima_silu_bf16(out, out, n, stream);
    }
    const CnTmaShape tshape = cn_tma_shape(C, kSilu, few_tiles);
    if (!cluster && tshape.P > 0 && spatial % 8 == 0 && aligned16(x) && aligned16(out) &&
        C % tshape.CG == 0 && (int64_t)B * ((spatial + tshape.P - 1) / tshape.P) < 2147483647) {
        CUtensorMap xmap;
        if (encode_bf16_map_3d(&xmap, x, (uint64_t)spatial, (uint64_t)C, (uint64_t)B, (uint64_t)spatial * 2,
                               (uint64_t)C * spatial * 2, (uint32_t)tshape.P, (uint32_t)tshape.CG)) {
            a.tiles_per_image = (spatial + tshape.P - 1) / tshape.P;
            const int64_t tsmem = 1024 + (int64_t)C * tshape.P * 2 + (int64_t)((C + 3) & ~3) * 4 + tshape.P * 4 +
                                  (int64_t)(C / tshape.CG) * 8 + (kBias ? (int64_t)C * 4 : 0);
            if (tsmem <= kCnMaxSmem + 4096) {
                const unsigned grid = (unsigned)((int64_t)B * a.tiles_per_image);
                const int form = kPixel ? 3 : kBias ? 2 : kSilu ? 1 : 0;
                const int slot = 44 + 4 * tshape.id + form;
#define ANIMA_CN_TMA(Pv, Tv, CGv)                                                                          \
    {                                                                                                      \
        auto kern = channel_norm_tma<Pv, Tv, kSilu, kBias, kPixel, CGv>;                                   \
        if (int e = allow_dynamic_smem((const void *)kern, kCnMaxSmem + 4096, slot)) return e;            \
        launch(kern, grid, Tv, (size_t)tsmem, stream, xmap, a);                                            \
    }
                if (tshape.id == 0) ANIMA_CN_TMA(64, 128, 64)
                else if (tshape.id == 1) ANIMA_CN_TMA(64, 256, 64)
                else if (tshape.id == 2) ANIMA_CN_TMA(32, 256, 64)
                else ANIMA_CN_TMA(64, 512, 64)
#undef ANIMA_CN_TMA
                return launch_status();
            }
        }
        a.tiles_per_image = (spatial + P - 1) / P;
    }
    if (cluster) {
        a.tiles_per_image = (spatial + kCnPix - 1) / kCnPix;
        auto kern = channel_norm_cluster<kSilu, kBias, kPixel>;
        if (int e = allow_dynamic_smem((const void *)kern, kCnMaxSmem, kPixel ? 13 : kBias ? 7 : kSilu ? 5 : 4)) return e;
        launch_cluster(kern, kCnCluster, (unsigned)(cl_tiles * kCnCluster), kCnBlock, (size_t)(Cq * per_ch), stream,
                       a, Cq);
    } else if (spatial % 8 == 0 && aligned16(x) && aligned16(out) && smem <= kCnMaxSmem && tiles < 2147483647) {
        const int nthr = cn_tile_threads(C, P, kSilu);
        // one shared-memory slot per kernel instance: 16 + 4 * (P, T) shape + form
        const int form = kPixel ? 3 : kBias ? 2 : kSilu ? 1 : 0;
        const int shape = P == 64 ? (nthr == 64 ? 0 : nthr == 128 ? 1 : 2) : P == 32 ? (nthr == 256 ? 3 : 5) : 4;
        const int slot = 16 + 4 * shape + form;
#define ANIMA_CN_TILE(Pv, Tv)                                                                              \
    {                                                                                                      \
        auto kern = channel_norm_tile<Pv, Tv, kSilu, kBias, kPixel>;                                       \
        if (int e = allow_dynamic_smem((const void *)kern, kCnMaxSmem, slot)) return e;                    \
        launch(kern, (unsigned)tiles, Tv, (size_t)smem, stream, a);                                        \
    }
        if (P == 64 && nthr == 64) ANIMA_CN_TILE(64, 64)
        else if (P == 64 && nthr == 128) ANIMA_CN_TILE(64, 128)
        else if (P == 64) ANIMA_CN_TILE(64, 256)
        else if (P == 32 && nthr == 256) ANIMA_CN_TILE(32, 256)
        else if (P == 32) ANIMA_CN_TILE(32, 128)
        else ANIMA_CN_TILE(16, 256)
#undef ANIMA_CN_TILE
    } else {
        const int64_t pixels = (int64_t)B * spatial;
        const unsigned blocks = wave_grid((const void *)channel_norm_serial<kSilu, kBias, kPixel>, 256, 0, pixels, &err);
        if (err) return err;
        launch(channel_norm_serial<kSilu, kBias, kPixel>, blocks, 256, 0, stream, a, pixels);
    }
    return launch_status();
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_rms_norm_channel_bf16(const anima_bf16 *x, const anima_bf16 *gamma,
                                           anima_bf16 *out, int B, int C, int spatial, float eps,
                                           anima_stream_t stream) {
    return channel_norm<false>(x, gamma, out, B, C, spatial, eps, stream);
}

extern "C" int anima_rms_norm_channel_silu_bf16(const anima_bf16 *x, const anima_bf16 *gamma,
                                                anima_bf16 *out, int B, int C, int spatial,
                                                float eps, anima_stream_t stream) {
    return channel_norm<true>(x, gamma, out, B, C, spatial, eps, stream);
}

extern "C" int anima_conv_bias_rms_norm_channel_silu_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                                          const anima_bf16 *gamma, anima_bf16 *out, int B, int C,
                                                          int spatial, float eps, anima_stream_t stream) {
    return channel_norm<true, true>(x, gamma, out, B, C, spatial, eps, stream, bias);
}

extern "C" int anima_pixel_norm_bf16(const anima_bf16 *x, anima_bf16 *out, int B, int C, int spatial, float eps,
                                     anima_stream_t stream) {
    return channel_norm<false, false, true>(x, nullptr, out, B, C, spatial, eps, stream);
}

extern "C" int anima_wait_timeouts(unsigned int *count, int reset) {
    if (!count) return ANIMA_ERR_NULL_POINTER;
    unsigned int cn = 0, ew = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&cn, g_cn_wait_timeouts, sizeof(unsigned int));
    if (e == cudaSuccess && reset) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_cn_wait_timeouts, &zero, sizeof(unsigned int));
    }
    if (e != cudaSuccess) return (int)e;
    if (int st = ew_wait_timeouts(&ew, reset)) return st;
    *count = cn + ew;
    return ANIMA_OK;
}
