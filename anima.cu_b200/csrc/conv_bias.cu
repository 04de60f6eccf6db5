// conv_bias.cu -- the VAE convolution's per-channel bias add on NCHW bf16, alone or fused
// with the residual add that follows a residual block's second convolution (sm_100a).
//
//   out[b,c,s] = x[b,c,s] + bias[c]                          causal_conv3d.cu:187-195, launched
//                                                            after every biased conv (:247-254,
//                                                            :293-299), in place there
//   out[b,c,s] = (x[b,c,s] + bias[c]) + residual[b,c,s]      the same followed by add_bf16
//                                                            (elementwise.cu:37-53), as
//                                                            vae.cpp:190-194 and :277-280 chain them
//
// Each sum is taken in fp32 and rounded to bf16 (RNE), the intermediate too, as the
// reference's two launches store it, so the outputs are the reference's bit for bit.
//
// The reference gives each element a thread with 2-byte accesses and a 64-bit division for
// the channel. Here each thread moves 8 elements as 16-byte chunks (when spatial % 8 == 0 and
// the tensors are 16-byte aligned), two chunks in flight, over one resident wave; the channel
// of each chunk comes from a division-free cursor advanced by the grid stride. The residual
// form reads x and residual once and writes out once: 6 bytes per element where the
// reference's pair moves 10.
#include "common.cuh"

namespace anima {
namespace {

constexpr int kCbBlock = 256;
constexpr int kCbU = 2;  // chunks in flight per thread

struct CbArgs {
    const anima_bf16 *x, *bias, *res;
    anima_bf16 *out;
    int C;
    int64_t spatial, n;
    bool vec;
};

__device__ __forceinline__ float ldf(const anima_bf16 *p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

template <bool kRes>
__device__ __forceinline__ float cb_elem(float x, float b, float r) {
    const float h = x + b;  // causal_conv3d.cu:193
    if constexpr (kRes) return bf16_round(h) + r;  // elementwise.cu:48-49
    return h;
}

template <bool kRes>
__global__ void __launch_bounds__(kCbBlock) conv_bias_kernel(CbArgs a) {
    pdl_wait();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (a.vec) {
        const int64_t nch = a.n >> 3;
        const uint32_t cpc = (uint32_t)(a.spatial >> 3);  // chunks per channel plane
        UnitCursor cur(q, stride, cpc, (uint32_t)a.C);
        while (q < nch) {
            Vec8 xv[kCbU], rv[kCbU];
            float bv[kCbU];
            int64_t at[kCbU];
#pragma unroll
            for (int u = 0; u < kCbU; ++u) {
                at[u] = q < nch ? q : -1;
                if (at[u] >= 0) {
                    xv[u] = ld_stream(a.x + q * 8);
                    if constexpr (kRes) rv[u] = ld_stream(a.res + q * 8);
                    bv[u] = ldf(a.bias, cur.ph);
                }
                q += stride;
                cur.advance(cpc, (uint32_t)a.C);
            }
#pragma unroll
            for (int u = 0; u < kCbU; ++u) {
                if (at[u] < 0) continue;
                float f[8], r[8] = {};
                unpack8(xv[u], f);
                if constexpr (kRes) unpack8(rv[u], r);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = cb_elem<kRes>(f[e], bv[u], r[e]);
                st_vec(a.out + at[u] * 8, pack8(f));
            }
        }
    } else {
        for (; q < a.n; q += stride) {
            const int c = (int)((q / a.spatial) % a.C);
            const float h = cb_elem<kRes>(ldf(a.x, q), ldf(a.bias, c), kRes ? ldf(a.res, q) : 0.0f);
            reinterpret_cast<__nv_bfloat16 *>(a.out)[q] = __float2bfloat16_rn(h);
        }
    }
    pdl_launch();
}

template <bool kRes>
int conv_bias(const anima_bf16 *x, const anima_bf16 *bias, const anima_bf16 *res, anima_bf16 *out, int B, int C,
              int spatial, cudaStream_t stream) {
    if (B < 0 || C <= 0 || spatial < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)B * C * spatial;
    if (n == 0) return ANIMA_OK;
    if (!x || !bias || !out || (kRes && !res)) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(x, 2) || !aligned_to(bias, 2) || !aligned_to(out, 2) || (kRes && !aligned_to(res, 2)))
        return ANIMA_ERR_MISALIGNED;
    const int64_t nb = n * 2;
    if (partial_overlap(out, nb, x, nb) || overlaps(out, nb, bias, (int64_t)C * 2) ||
        (kRes && partial_overlap(out, nb, res, nb)))
        return ANIMA_ERR_OVERLAP;
    const bool vec = spatial % 8 == 0 && aligned16(x) && aligned16(out) && (!kRes || aligned16(res));
    CbArgs a{x, bias, res, out, C, spatial, n, vec};
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)conv_bias_kernel<kRes>, kCbBlock, 0, vec ? n / 8 : n, &err);
    if (err) return err;
    launch(conv_bias_kernel<kRes>, grid, kCbBlock, 0, stream, a);
    return launch_status();
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_conv_bias_add_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out, int B, int C,
                                        int spatial, anima_stream_t stream) {
    return conv_bias<false>(x, bias, nullptr, out, B, C, spatial, stream);
}

extern "C" int anima_conv_bias_residual_add_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                                 const anima_bf16 *residual, anima_bf16 *out, int B, int C,
                                                 int spatial, anima_stream_t stream) {
    return conv_bias<true>(x, bias, residual, out, B, C, spatial, stream);
}
