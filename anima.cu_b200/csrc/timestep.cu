// timestep.cu -- sinusoidal timestep embedding on the GPU (sm_100a).
//
// The reference builds the flip_sin_to_cos sinusoid of one timestep on the host, rounds it
// to bf16, uploads it with a synchronous copy, then runs rms_norm_bf16 on that single row
// (transformer.cpp:182-200). This kernel does all of it in one launch with no host work
// and no copy: one CTA computes the row, stores it, and RMS-normalises it with the
// reference block's own thread layout and reduction tree (rms_norm.cu:9-67).
//
// The host loop computes freq_i = expf(-ln(1e4)*i/half) and cosf/sinf(t*freq_i) with
// glibc's fp32 functions. Here the fp32 argument is formed with the host's exact operation
// sequence (multiply, then divide, each rounded), and exp, cos and sin are evaluated in
// double and rounded once to fp32: the correctly rounded fp32 value. glibc's fp32 functions
// are not correctly rounded everywhere (about 1% of the cos/sin values of dims 256-4096 sit
// one fp32 ulp away from the correctly rounded value), so the bf16 sinusoid, and the
// normalised row after it, can differ from the reference's by one bf16 ulp in rare
// elements: within the 1-ulp tolerance, but not bit-exact. Callers that need the
// reference's exact bits keep the host loop.
#include "common.cuh"

#include <math.h>

namespace anima {
namespace {

struct TsArgs {
    float t;
    float neg_ln1e4;  // -logf(10000.0f), computed on the host exactly as the reference does
    const anima_bf16 *w;  // nullable
    anima_bf16 *sinusoid, *normed;  // normed nullable
    int dim;
    float eps;
};

__global__ void timestep_embedding(TsArgs a) {
    pdl_wait();
    extern __shared__ __align__(16) __nv_bfloat16 row[];  // [dim]
    __shared__ float red[33];
    const int half = a.dim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float arg = __fdiv_rn(__fmul_rn(a.neg_ln1e4, (float)i), (float)half);
        const float freq = (float)exp((double)arg);
        const float angle = __fmul_rn(a.t, freq);
        double s, c;
        sincos((double)angle, &s, &c);
        const __nv_bfloat16 cb = __float2bfloat16_rn((float)c), sb = __float2bfloat16_rn((float)s);
        row[i] = cb;
        row[half + i] = sb;
        reinterpret_cast<__nv_bfloat16 *>(a.sinusoid)[i] = cb;
        reinterpret_cast<__nv_bfloat16 *>(a.sinusoid)[half + i] = sb;
    }
    if (!a.normed) return;  // uniform across the block
    __syncthreads();
    // rms_norm.cu:31-37 over the bf16 row, pairs t, t+T, ... per thread
    float q = 0.0f;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
        const float v0 = __bfloat162float(row[2 * p]), v1 = __bfloat162float(row[2 * p + 1]);
        q = __fmaf_rn(v0, v0, q);
        q = __fmaf_rn(v1, v1, q);
    }
    const float r = rsqrtf(__fdiv_rn(ref_cta_sum(q, red), (float)a.dim) + a.eps);
    for (int e = threadIdx.x; e < a.dim; e += blockDim.x) {
        float o = __bfloat162float(row[e]) * r;
        if (a.w) o = o * __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.w)[e]);
        reinterpret_cast<__nv_bfloat16 *>(a.normed)[e] = __float2bfloat16_rn(o);
    }
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_timestep_embedding_bf16(float timestep, const anima_bf16 *norm_weight,
                                             anima_bf16 *sinusoid_out, anima_bf16 *normed_out, int dim,
                                             float eps, anima_stream_t stream) {
    if (dim <= 0 || (dim & 1) || dim > 32768) return ANIMA_ERR_BAD_SHAPE;
    if (!sinusoid_out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(sinusoid_out, 2) || (normed_out && !aligned_to(normed_out, 2)) ||
        (norm_weight && !aligned_to(norm_weight, 2)))
        return ANIMA_ERR_MISALIGNED;
    if (normed_out && (partial_overlap(sinusoid_out, dim * 2, normed_out, dim * 2) ||
                       sinusoid_out == normed_out))
        return ANIMA_ERR_OVERLAP;
    TsArgs a{timestep, -logf(10000.0f), norm_weight, sinusoid_out, normed_out, dim, eps};
    const size_t smem = (size_t)dim * 2;
    if (smem > 48 * 1024) {
        if (int e = allow_dynamic_smem((const void *)timestep_embedding, 64 * 1024, 2)) return e;
    }
    launch(timestep_embedding, 1, ref_row_threads(dim), smem, stream, a);
    return launch_status();
}
