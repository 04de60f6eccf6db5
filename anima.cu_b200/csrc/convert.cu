// convert.cu -- dtype conversions, scaling by a scalar and the VAE's nearest 2x upsample (sm_100a):
//
//   f32_to_bf16   out = bf16(x) (RNE) over floor(N/2) pairs     elementwise.cu:311-331
//   bf16_to_f32   out = float(x) over floor(N/2) pairs           elementwise.cu:333-352
//   scale_bf16    out = bf16(x * s) over floor(N/2) pairs        elementwise.cu:97-122
//   nearest_upsample_2x_bf16  [B, C, H, W] -> [B, C, 2H, 2W]     vae_kernels.cu:98-133
//
// The conversions and the upsample are exact by construction; the scaling is one fp32 multiply
// and a rounding, as the reference's. The pair loops leave an odd last element untouched, as
// the reference's do. Each thread moves 8 elements per step with 16-byte
// accesses on the bf16 side (and 2 x 16 bytes on the fp32 side) when the pointers allow,
// over one resident wave; the upsample writes each output row's 16-byte chunks from 8-byte
// loads of the input row, one launch for all batch items (the reference launches per item).
#include "common.cuh"

namespace anima {
namespace {

constexpr int kCvBlock = 256;

// ------------------------------------------------------------------ conversions
template <bool kToBf16>
__global__ void __launch_bounds__(kCvBlock) convert_kernel(const void *src, void *dst, int64_t n, bool vec) {
    pdl_wait();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        for (; i < n / 8; i += stride) {
            if constexpr (kToBf16) {
                const float4 *s = reinterpret_cast<const float4 *>(src) + 2 * i;
                const float4 a = s[0], b = s[1];
                st_vec(static_cast<anima_bf16 *>(dst) + 8 * i,
                       Vec8{{pack_bf2(a.x, a.y), pack_bf2(a.z, a.w), pack_bf2(b.x, b.y), pack_bf2(b.z, b.w)}});
            } else {
                const Vec8 v = ld_stream(static_cast<const anima_bf16 *>(src) + 8 * i);
                float4 *d = reinterpret_cast<float4 *>(dst) + 2 * i;
                d[0] = make_float4(bf_lo(v.w[0]), bf_hi(v.w[0]), bf_lo(v.w[1]), bf_hi(v.w[1]));
                d[1] = make_float4(bf_lo(v.w[2]), bf_hi(v.w[2]), bf_lo(v.w[3]), bf_hi(v.w[3]));
            }
        }
        i = n / 8 * 8 + ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);  // the tail, element by element
    }
    for (; i < n; i += stride) {
        if constexpr (kToBf16)
            reinterpret_cast<__nv_bfloat16 *>(dst)[i] = __float2bfloat16_rn(static_cast<const float *>(src)[i]);
        else
            static_cast<float *>(dst)[i] = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(src)[i]);
    }
    pdl_launch();
}

template <bool kToBf16>
int convert(const void *src, void *dst, int64_t N, cudaStream_t stream) {
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = N / 2 * 2;  // the reference converts floor(N/2) pairs
    if (n == 0) return ANIMA_OK;
    if (!src || !dst) return ANIMA_ERR_NULL_POINTER;
    const unsigned sa = kToBf16 ? 4 : 2, da = kToBf16 ? 2 : 4;
    if (!aligned_to(src, sa) || !aligned_to(dst, da)) return ANIMA_ERR_MISALIGNED;
    if (overlaps(src, n * sa, dst, n * da)) return ANIMA_ERR_OVERLAP;
    const bool vec = aligned16(src) && aligned16(dst);
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)convert_kernel<kToBf16>, kCvBlock, 0, vec ? n / 8 + 1 : n, &err);
    if (err) return err;
    launch(convert_kernel<kToBf16>, grid, kCvBlock, 0, stream, src, dst, n, vec);
    return launch_status();
}

// ------------------------------------------------------------------ scale
__global__ void __launch_bounds__(kCvBlock) scale_kernel(const anima_bf16 *x, anima_bf16 *out, float s, int64_t n,
                                                        bool vec) {
    pdl_wait();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        for (; i < n / 8; i += stride) {
            float f[8];
            unpack8(ld_stream(x + 8 * i), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * s;  // elementwise.cu:109-110
            st_vec(out + 8 * i, pack8(f));
        }
        i = n / 8 * 8 + ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
    }
    for (; i < n; i += stride)
        reinterpret_cast<__nv_bfloat16 *>(out)[i] =
            __float2bfloat16_rn(__bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(x)[i]) * s);
    pdl_launch();
}

// ------------------------------------------------------------- nearest upsample
struct UpArgs {
    const anima_bf16 *in;
    anima_bf16 *out;
    int64_t rows;  // B*C*2H output rows
    int H, W;      // input height and width
    bool vec;      // 16-byte output chunks: W % 4 == 0 and aligned pointers
};

__global__ void __launch_bounds__(kCvBlock) upsample_kernel(UpArgs a) {
    pdl_wait();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int W2 = 2 * a.W;
    if (a.vec) {
        const int cpr = W2 / 8;  // 16-byte chunks per output row
        const int64_t units = a.rows * cpr;
        for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < units; q += stride) {
            const int64_t r = q / cpr;
            const int k = (int)(q - r * cpr);
            const int64_t plane = r / (2 * a.H);  // b*C + c
            const int h2 = (int)(r - plane * 2 * a.H);
            // vae_kernels.cu:109-116: out[c, h2, w2] = in[c, h2/2, w2/2]; 8 outputs from 4 inputs
            const uint2 v = *reinterpret_cast<const uint2 *>(a.in + (plane * a.H + h2 / 2) * a.W + 4 * k);
            const uint32_t e0 = v.x & 0xffffu, e1 = v.x >> 16, e2 = v.y & 0xffffu, e3 = v.y >> 16;
            st_vec(a.out + r * W2 + 8 * k, Vec8{{e0 | e0 << 16, e1 | e1 << 16, e2 | e2 << 16, e3 | e3 << 16}});
        }
    } else {
        const int64_t total = a.rows * W2;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int64_t r = i / W2;
            const int w2 = (int)(i - r * W2);
            const int64_t plane = r / (2 * a.H);
            const int h2 = (int)(r - plane * 2 * a.H);
            reinterpret_cast<uint16_t *>(a.out)[i] =
                reinterpret_cast<const uint16_t *>(a.in)[(plane * a.H + h2 / 2) * a.W + w2 / 2];
        }
    }
    pdl_launch();
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_f32_to_bf16(const float *x, anima_bf16 *out, int64_t N, anima_stream_t stream) {
    return convert<true>(x, out, N, stream);
}

extern "C" int anima_bf16_to_f32(const anima_bf16 *x, float *out, int64_t N, anima_stream_t stream) {
    return convert<false>(x, out, N, stream);
}

extern "C" int anima_scale_bf16(const anima_bf16 *x, anima_bf16 *out, float scale, int64_t N,
                                anima_stream_t stream) {
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = N / 2 * 2;
    if (n == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(x, 2) || !aligned_to(out, 2)) return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(x, n * 2, out, n * 2)) return ANIMA_ERR_OVERLAP;
    const bool vec = aligned16(x) && aligned16(out);
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)scale_kernel, kCvBlock, 0, vec ? n / 8 + 1 : n, &err);
    if (err) return err;
    launch(scale_kernel, grid, kCvBlock, 0, stream, x, out, scale, n, vec);
    return launch_status();
}

extern "C" int anima_nearest_upsample_2x_bf16(const anima_bf16 *in, anima_bf16 *out, int B, int C, int H, int W,
                                              anima_stream_t stream) {
    if (B < 0 || C < 0 || H < 0 || W < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n_in = (int64_t)B * C * H * W, n_out = 4 * n_in;
    if (n_in == 0) return ANIMA_OK;
    if (!in || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(in, 2) || !aligned_to(out, 2)) return ANIMA_ERR_MISALIGNED;
    if (overlaps(in, n_in * 2, out, n_out * 2)) return ANIMA_ERR_OVERLAP;
    if (W > 1073741823) return ANIMA_ERR_TOO_LARGE;
    UpArgs a{in, out, (int64_t)B * C * 2 * H, H, W, W % 4 == 0 && aligned16(out) && aligned_to(in, 8)};
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)upsample_kernel, kCvBlock, 0, a.vec ? n_out / 8 : n_out, &err);
    if (err) return err;
    launch(upsample_kernel, grid, kCvBlock, 0, stream, a);
    return launch_status();
}
