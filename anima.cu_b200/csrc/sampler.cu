// sampler.cu -- the denoising loop's per-step kernels and the DiT's latent I/O (sm_100a):
// fused CFG + Euler, Euler-ancestral (rectified flow) and ER-SDE steps (transpose.cu:246-465),
// 3-D patchify / unpatchify (transpose.cu:128-243) and the VAE latent's per-channel
// scale-shift (vae_kernels.cu:172-206).
//
// The steps are elementwise over the latent: each thread takes 8 consecutive elements as
// 16-byte chunks when every pointer is 16-byte aligned (scalar otherwise), grid-stride over
// one resident wave. The per-element arithmetic is the reference's own expression, written in
// the same order, so nvcc forms the same fused multiply-adds and the results are the
// reference's bit for bit (the tests compare against the reference kernels). Patchify and
// unpatchify are index permutations (exact by construction), written per destination element
// so the stores are coalesced, with 32-bit index arithmetic when the tensor allows it and
// one launch for all batch items (the reference launches once per item).
#include "common.cuh"

namespace anima {
namespace {

constexpr int kSmpBlock = 256;

__device__ __forceinline__ float ldf(const anima_bf16 *p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}
__device__ __forceinline__ void stf(anima_bf16 *p, int64_t i, float f) {
    reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(f);
}

// ------------------------------------------------------------------ CFG + Euler
struct EulerArgs {
    const anima_bf16 *sample, *pos, *neg;
    anima_bf16 *out;
    float cfg, sigma, sigma_next;
    int64_t n;
    bool vec;
};

// transpose.cu:260-275
__device__ __forceinline__ float euler_elem(float s, float np, float nn, const EulerArgs &a) {
    const float noise = nn + a.cfg * (np - nn);
    float result;
    if (a.sigma_next == 0.0f) {
        result = s - a.sigma * noise;
    } else {
        const float denoised = s - a.sigma * noise;
        const float d = (s - denoised) / a.sigma;
        result = s + d * (a.sigma_next - a.sigma);
    }
    return result;
}

__global__ void __launch_bounds__(kSmpBlock) cfg_euler_kernel(EulerArgs a) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nch = a.vec ? a.n >> 3 : 0;
    for (int64_t c = tid; c < nch; c += stride) {
        float s[8], p[8], q[8];
        unpack8(ld_stream(a.sample + c * 8), s);
        unpack8(ld_stream(a.pos + c * 8), p);
        unpack8(ld_stream(a.neg + c * 8), q);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] = euler_elem(s[e], p[e], q[e], a);
        st_vec(a.out + c * 8, pack8(s));
    }
    for (int64_t i = (nch << 3) + tid; i < a.n; i += stride)
        stf(a.out, i, euler_elem(ldf(a.sample, i), ldf(a.pos, i), ldf(a.neg, i), a));
    pdl_launch();
}

// ------------------------------------------------- CFG + Euler ancestral (RF)
struct EulerAArgs {
    const anima_bf16 *sample, *pos, *neg, *rand;
    anima_bf16 *out;
    float cfg, sigma, eta, s_noise, sigma_down_ratio, alpha_ratio, renoise_coeff;
    int64_t n;
    bool vec, renoise;
};

// transpose.cu:318-333
__device__ __forceinline__ float euler_a_elem(float s, float np, float nn, float rn, const EulerAArgs &a) {
    const float noise_pred = nn + a.cfg * (np - nn);
    const float denoised = s - a.sigma * noise_pred;
    float result = a.sigma_down_ratio * s + (1.0f - a.sigma_down_ratio) * denoised;
    if (a.renoise) result = a.alpha_ratio * result + rn * a.s_noise * a.renoise_coeff;
    return result;
}

__global__ void __launch_bounds__(kSmpBlock) cfg_euler_a_kernel(EulerAArgs a) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nch = a.vec ? a.n >> 3 : 0;
    for (int64_t c = tid; c < nch; c += stride) {
        float s[8], p[8], q[8], r[8] = {};
        unpack8(ld_stream(a.sample + c * 8), s);
        unpack8(ld_stream(a.pos + c * 8), p);
        unpack8(ld_stream(a.neg + c * 8), q);
        if (a.renoise) unpack8(ld_stream(a.rand + c * 8), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] = euler_a_elem(s[e], p[e], q[e], r[e], a);
        st_vec(a.out + c * 8, pack8(s));
    }
    for (int64_t i = (nch << 3) + tid; i < a.n; i += stride)
        stf(a.out, i, euler_a_elem(ldf(a.sample, i), ldf(a.pos, i), ldf(a.neg, i),
                                   a.renoise ? ldf(a.rand, i) : 0.0f, a));
    pdl_launch();
}

// ------------------------------------------------------------- CFG + ER-SDE
struct ErSdeArgs {
    anima_bf16 *x;
    const anima_bf16 *pos, *neg;
    anima_bf16 *den_out;
    const anima_bf16 *old_den;
    anima_bf16 *dd_out;
    const anima_bf16 *old_dd, *rand;
    float cfg, sigma, A, B, d_scale, coeff2, u_scale, coeff3, noise_coeff;
    int64_t n;
    bool vec;
};

// transpose.cu:405-439: returns x; den and dd through the references
__device__ __forceinline__ float er_sde_elem(float s, float np, float nn, float old_den, float old_dd, float rn,
                                             const ErSdeArgs &a, float &den, float &dd) {
    const float vel = nn + a.cfg * (np - nn);
    den = s - a.sigma * vel;
    float result = a.A * s + a.B * den;
    dd = 0.0f;
    if (a.old_den != nullptr) {
        dd = (den - old_den) * a.d_scale;
        result += a.coeff2 * dd;
        if (a.old_dd != nullptr) {
            const float du = (dd - old_dd) * a.u_scale;
            result += a.coeff3 * du;
        }
    }
    if (a.noise_coeff > 0.0f && a.rand != nullptr) result += a.noise_coeff * rn;
    return result;
}

__global__ void __launch_bounds__(kSmpBlock) cfg_er_sde_kernel(ErSdeArgs a) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nch = a.vec ? a.n >> 3 : 0;
    const bool want_dd = a.dd_out != nullptr && a.old_den != nullptr;
    const bool use_rand = a.noise_coeff > 0.0f && a.rand != nullptr;
    for (int64_t c = tid; c < nch; c += stride) {
        float s[8], p[8], q[8], od[8] = {}, odd[8] = {}, r[8] = {}, den[8], dd[8];
        unpack8(ld_stream(a.x + c * 8), s);
        unpack8(ld_stream(a.pos + c * 8), p);
        unpack8(ld_stream(a.neg + c * 8), q);
        if (a.old_den) unpack8(ld_stream(a.old_den + c * 8), od);
        if (a.old_den && a.old_dd) unpack8(ld_stream(a.old_dd + c * 8), odd);
        if (use_rand) unpack8(ld_stream(a.rand + c * 8), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[e] = er_sde_elem(s[e], p[e], q[e], od[e], odd[e], r[e], a, den[e], dd[e]);
        st_vec(a.x + c * 8, pack8(s));
        st_vec(a.den_out + c * 8, pack8(den));
        if (want_dd) st_vec(a.dd_out + c * 8, pack8(dd));
    }
    for (int64_t i = (nch << 3) + tid; i < a.n; i += stride) {
        float den, dd;
        const float r = er_sde_elem(ldf(a.x, i), ldf(a.pos, i), ldf(a.neg, i), a.old_den ? ldf(a.old_den, i) : 0.0f,
                                    a.old_den && a.old_dd ? ldf(a.old_dd, i) : 0.0f, use_rand ? ldf(a.rand, i) : 0.0f,
                                    a, den, dd);
        stf(a.x, i, r);
        stf(a.den_out, i, den);
        if (want_dd) stf(a.dd_out, i, dd);
    }
    pdl_launch();
}

// ------------------------------------------------------- patchify / unpatchify
struct PatchArgs {
    const anima_bf16 *src;
    anima_bf16 *dst;
    int C, T, H, W, pT, pH, pW, pe_t, pe_h, pe_w;
    int64_t S, pd;       // tokens per item, patch_dim = C*pT*pH*pW
    int64_t per_item;    // elements per item on the patch side = S * pd
    int64_t vol;         // C*T*H*W, elements per item on the volume side
    int64_t total;       // B * per_item (patchify) or B * C*T*H*W (unpatchify)
};

// transpose.cu:132-163: dst[b, tok, d] = src[b, c, t, h, w], d = ((c*pT + pt)*pH + ph)*pW + pw
template <typename I>
__device__ __forceinline__ void patchify_elem(const PatchArgs &a, I j) {
    const I per_item = (I)a.per_item, pd = (I)a.pd;
    const I b = j / per_item, r = j - b * per_item;
    const I tok = r / pd;
    I d = r - tok * pd;
    const I pw = d % a.pW;
    d /= a.pW;
    const I ph = d % a.pH;
    d /= a.pH;
    const I pt = d % a.pT;
    const I c = d / a.pT;
    const I fw = tok % a.pe_w, fh = (tok / a.pe_w) % a.pe_h, ft = tok / ((I)a.pe_w * a.pe_h);
    const I t = ft * a.pT + pt, h = fh * a.pH + ph, w = fw * a.pW + pw;
    a.dst[j] = a.src[(int64_t)b * a.vol + (((int64_t)c * a.T + t) * a.H + h) * a.W + w];
}

// transpose.cu:191-223: dst[b, c, t, h, w] = src[b, tok, d], d = ((ph*pW + pw)*pT + pt)*C + c
// (the Cosmos output projection's [pH, pW, pT, C] order). Volume positions beyond the last
// whole patch are not written, as in the reference.
template <typename I>
__device__ __forceinline__ void unpatchify_elem(const PatchArgs &a, I j) {
    const I vol = (I)a.vol;
    const I b = j / vol;
    I r = j - b * vol;
    const I w = r % a.W;
    r /= a.W;
    const I h = r % a.H;
    r /= a.H;
    const I t = r % a.T;
    const I c = r / a.T;
    const I ft = t / a.pT, fh = h / a.pH, fw = w / a.pW;
    if (ft >= a.pe_t || fh >= a.pe_h || fw >= a.pe_w) return;
    const I pt = t - ft * a.pT, ph = h - fh * a.pH, pw = w - fw * a.pW;
    const I tok = (ft * a.pe_h + fh) * a.pe_w + fw;
    const I d = ((ph * a.pW + pw) * a.pT + pt) * a.C + c;
    a.dst[j] = a.src[(int64_t)b * a.per_item + (int64_t)tok * a.pd + d];
}

// The DiT's patches (pT = 1, pH = pW = 2, T a multiple of 1, H and W even): one thread per
// (item, token, channel) moves the 2x2 patch as two 4-byte row pieces on the volume side and
// 8 contiguous bytes (patchify: c-major patch order) or 4 channel-strided values (unpatchify)
// on the token side.
template <bool kUnpatch>
__global__ void __launch_bounds__(kSmpBlock) patch_kernel_122(PatchArgs a, int64_t items) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t q = tid; q < items; q += stride) {  // q = (b * S + tok) * C + c
        const int64_t bt = q / a.C;
        const int c = (int)(q - bt * a.C);
        const int64_t b = bt / a.S, tok = bt - b * a.S;
        const int fw = (int)(tok % a.pe_w), fh = (int)((tok / a.pe_w) % a.pe_h), t = (int)(tok / ((int64_t)a.pe_w * a.pe_h));
        const int64_t row0 = (((int64_t)b * a.C + c) * a.T + t) * a.H + 2 * fh;
        uint32_t *v0 = reinterpret_cast<uint32_t *>(kUnpatch ? a.dst : const_cast<anima_bf16 *>(a.src)) +
                       (row0 * a.W + 2 * fw) / 2;
        uint32_t *v1 = v0 + a.W / 2;
        if constexpr (!kUnpatch) {  // d = c*4 + ph*2 + pw
            const uint2 o = make_uint2(*v0, *v1);
            *reinterpret_cast<uint2 *>(a.dst + ((int64_t)b * a.S + tok) * a.pd + 4 * c) = o;
        } else {  // d = (ph*2 + pw)*C + c
            const anima_bf16 *sp = a.src + ((int64_t)b * a.S + tok) * a.pd + c;
            *v0 = (uint32_t)sp[0] | (uint32_t)sp[a.C] << 16;
            *v1 = (uint32_t)sp[2 * a.C] | (uint32_t)sp[3 * a.C] << 16;
        }
    }
    pdl_launch();
}

template <bool kUnpatch>
__global__ void __launch_bounds__(kSmpBlock) patch_kernel(PatchArgs a) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (a.total < 2147483647LL) {
        for (int j = (int)tid; j < (int)a.total; j += (int)stride) {
            if constexpr (kUnpatch) unpatchify_elem<int>(a, j);
            else patchify_elem<int>(a, j);
        }
    } else {
        for (int64_t j = tid; j < a.total; j += stride) {
            if constexpr (kUnpatch) unpatchify_elem<int64_t>(a, j);
            else patchify_elem<int64_t>(a, j);
        }
    }
    pdl_launch();
}

// -------------------------------------------------------- channel scale-shift
struct CssArgs {
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    int C;
    int64_t spatial, n;  // n = B*C*spatial
    bool vec;            // spatial % 8 == 0 and 16-byte aligned x, out
};

// vae_kernels.cu:175-188: x * scale[c] + shift[c]
__device__ __forceinline__ float css_elem(float xv, float sv, float hv) { return xv * sv + hv; }

__global__ void __launch_bounds__(kSmpBlock) channel_scale_shift_kernel(CssArgs a) {
    pdl_wait();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (a.vec) {
        const int64_t nch = a.n >> 3, cpc = a.spatial >> 3;  // chunks per channel plane
        for (int64_t q = tid; q < nch; q += stride) {
            const int c = (int)((q / cpc) % a.C);
            const float sv = ldf(a.scale, c), hv = ldf(a.shift, c);
            float f[8];
            unpack8(ld_stream(a.x + q * 8), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = css_elem(f[e], sv, hv);
            st_vec(a.out + q * 8, pack8(f));
        }
    } else {
        for (int64_t i = tid; i < a.n; i += stride) {
            const int c = (int)((i / a.spatial) % a.C);
            stf(a.out, i, css_elem(ldf(a.x, i), ldf(a.scale, c), ldf(a.shift, c)));
        }
    }
    pdl_launch();
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

// An output may be the same buffer as an input (in place) but not partly overlap it.
bool clash(const void *out, int64_t nb, const void *in, int64_t ib) {
    return in && partial_overlap(out, nb, in, ib);
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_cfg_euler_step_bf16(const anima_bf16 *sample, const anima_bf16 *noise_pos,
                                         const anima_bf16 *noise_neg, anima_bf16 *out, float cfg_scale,
                                         float sigma, float sigma_next, int64_t N, anima_stream_t stream) {
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!sample || !noise_pos || !noise_neg || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(sample) || !bf16_ok(noise_pos) || !bf16_ok(noise_neg) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    if (N > INT64_MAX / 2) return ANIMA_ERR_TOO_LARGE;
    const int64_t nb = N * 2;
    if (clash(out, nb, sample, nb) || clash(out, nb, noise_pos, nb) || clash(out, nb, noise_neg, nb))
        return ANIMA_ERR_OVERLAP;
    EulerArgs a{sample, noise_pos, noise_neg, out, cfg_scale, sigma, sigma_next, N,
                aligned16(sample) && aligned16(noise_pos) && aligned16(noise_neg) && aligned16(out)};
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)cfg_euler_kernel, kSmpBlock, 0, a.vec ? (N + 7) / 8 : N, &err);
    if (err) return err;
    launch(cfg_euler_kernel, grid, kSmpBlock, 0, stream, a);
    return launch_status();
}

extern "C" int anima_cfg_euler_a_rf_step_bf16(const anima_bf16 *sample, const anima_bf16 *noise_pos,
                                              const anima_bf16 *noise_neg, const anima_bf16 *rand_noise,
                                              anima_bf16 *out, float cfg_scale, float sigma, float sigma_next,
                                              float eta, float s_noise, int64_t N, anima_stream_t stream) {
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!sample || !noise_pos || !noise_neg || !out) return ANIMA_ERR_NULL_POINTER;
    // transpose.cu:345-354: the step's coefficients, in the reference's host float arithmetic
    const float downstep_ratio = 1.0f + (sigma_next / sigma - 1.0f) * eta;
    const float sigma_down = sigma_next * downstep_ratio;
    const float alpha_ip1 = 1.0f - sigma_next;
    const float alpha_down = 1.0f - sigma_down;
    const float renoise_sq = sigma_next * sigma_next -
                             sigma_down * sigma_down * alpha_ip1 * alpha_ip1 / (alpha_down * alpha_down);
    const float renoise_coeff = (renoise_sq > 0.0f) ? sqrtf(renoise_sq) : 0.0f;
    const float sigma_down_ratio = sigma_down / sigma;
    const float alpha_ratio = alpha_ip1 / alpha_down;
    const bool renoise = eta > 0.0f && renoise_coeff > 0.0f;
    if (renoise && !rand_noise) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(sample) || !bf16_ok(noise_pos) || !bf16_ok(noise_neg) || !bf16_ok(out) ||
        (rand_noise && !bf16_ok(rand_noise)))
        return ANIMA_ERR_MISALIGNED;
    if (N > INT64_MAX / 2) return ANIMA_ERR_TOO_LARGE;
    const int64_t nb = N * 2;
    if (clash(out, nb, sample, nb) || clash(out, nb, noise_pos, nb) || clash(out, nb, noise_neg, nb) ||
        clash(out, nb, rand_noise, nb))
        return ANIMA_ERR_OVERLAP;
    EulerAArgs a{sample, noise_pos, noise_neg, rand_noise, out, cfg_scale, sigma, eta, s_noise,
                 sigma_down_ratio, alpha_ratio, renoise_coeff, N,
                 aligned16(sample) && aligned16(noise_pos) && aligned16(noise_neg) && aligned16(out) &&
                     (!renoise || aligned16(rand_noise)),
                 renoise};
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)cfg_euler_a_kernel, kSmpBlock, 0, a.vec ? (N + 7) / 8 : N, &err);
    if (err) return err;
    launch(cfg_euler_a_kernel, grid, kSmpBlock, 0, stream, a);
    return launch_status();
}

extern "C" int anima_cfg_er_sde_full_step_bf16(anima_bf16 *x, const anima_bf16 *noise_pos,
                                               const anima_bf16 *noise_neg, anima_bf16 *denoised_out,
                                               const anima_bf16 *old_denoised, anima_bf16 *denoised_d_out,
                                               const anima_bf16 *old_denoised_d, const anima_bf16 *rand_noise,
                                               float cfg_scale, float sigma, float A, float B, float d_scale,
                                               float coeff2, float u_scale, float coeff3, float noise_coeff,
                                               int64_t N, anima_stream_t stream) {
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!x || !noise_pos || !noise_neg || !denoised_out) return ANIMA_ERR_NULL_POINTER;
    const anima_bf16 *ins[] = {noise_pos, noise_neg, old_denoised, old_denoised_d, rand_noise};
    for (const anima_bf16 *p : ins)
        if (p && !bf16_ok(p)) return ANIMA_ERR_MISALIGNED;
    if (!bf16_ok(x) || !bf16_ok(denoised_out) || (denoised_d_out && !bf16_ok(denoised_d_out)))
        return ANIMA_ERR_MISALIGNED;
    if (N > INT64_MAX / 2) return ANIMA_ERR_TOO_LARGE;
    const int64_t nb = N * 2;
    // x is updated in place; the other outputs are separate buffers that overlap nothing
    anima_bf16 *outs[] = {x, denoised_out, denoised_d_out};
    for (anima_bf16 *o : outs) {
        if (!o) continue;
        for (const anima_bf16 *p : ins)
            if (p && (o == x ? partial_overlap(o, nb, p, nb) : overlaps(o, nb, p, nb))) return ANIMA_ERR_OVERLAP;
    }
    if (overlaps(denoised_out, nb, x, nb) || (denoised_d_out && (overlaps(denoised_d_out, nb, x, nb) ||
                                                                 overlaps(denoised_d_out, nb, denoised_out, nb))))
        return ANIMA_ERR_OVERLAP;
    bool vec = aligned16(x) && aligned16(denoised_out) && (!denoised_d_out || aligned16(denoised_d_out));
    for (const anima_bf16 *p : ins) vec = vec && (!p || aligned16(p));
    ErSdeArgs a{x, noise_pos, noise_neg, denoised_out, old_denoised, denoised_d_out, old_denoised_d, rand_noise,
                cfg_scale, sigma, A, B, d_scale, coeff2, u_scale, coeff3, noise_coeff, N, vec};
    int err = ANIMA_OK;
    const unsigned grid = wave_grid((const void *)cfg_er_sde_kernel, kSmpBlock, 0, vec ? (N + 7) / 8 : N, &err);
    if (err) return err;
    launch(cfg_er_sde_kernel, grid, kSmpBlock, 0, stream, a);
    return launch_status();
}

namespace {
template <bool kUnpatch>
int patch_op(const anima_bf16 *src, anima_bf16 *dst, int B, int C, int T, int H, int W, int pT, int pH, int pW,
             cudaStream_t stream) {
    if (B < 0 || C <= 0 || T <= 0 || H <= 0 || W <= 0 || pT <= 0 || pH <= 0 || pW <= 0) return ANIMA_ERR_BAD_SHAPE;
    PatchArgs a{};
    a.src = src;
    a.dst = dst;
    a.C = C, a.T = T, a.H = H, a.W = W, a.pT = pT, a.pH = pH, a.pW = pW;
    a.pe_t = T / pT, a.pe_h = H / pH, a.pe_w = W / pW;
    a.S = (int64_t)a.pe_t * a.pe_h * a.pe_w;
    a.pd = (int64_t)C * pT * pH * pW;
    a.per_item = a.S * a.pd;
    a.vol = (int64_t)C * T * H * W;
    a.total = (int64_t)B * (kUnpatch ? a.vol : a.per_item);
    if (a.total == 0 || a.S == 0) return ANIMA_OK;
    if (!src || !dst) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(src) || !bf16_ok(dst)) return ANIMA_ERR_MISALIGNED;
    const int64_t ns = (int64_t)B * (kUnpatch ? a.per_item : a.vol) * 2, nd = a.total * 2;
    if (overlaps(src, ns, dst, nd)) return ANIMA_ERR_OVERLAP;
    int err = ANIMA_OK;
    // 2x2 spatial patches over whole rows: every row piece is 4-byte aligned when the
    // volume is, and the 8-byte token-side store (patchify) is aligned when the tokens are
    if (pT == 1 && pH == 2 && pW == 2 && H % 2 == 0 && W % 2 == 0 && aligned_to(kUnpatch ? dst : src, 4) &&
        (kUnpatch || aligned_to(dst, 8))) {
        const int64_t items = (int64_t)B * a.S * C;
        const unsigned grid = wave_grid((const void *)patch_kernel_122<kUnpatch>, kSmpBlock, 0, items, &err);
        if (err) return err;
        launch(patch_kernel_122<kUnpatch>, grid, kSmpBlock, 0, stream, a, items);
        return launch_status();
    }
    const unsigned grid = wave_grid((const void *)patch_kernel<kUnpatch>, kSmpBlock, 0, a.total, &err);
    if (err) return err;
    launch(patch_kernel<kUnpatch>, grid, kSmpBlock, 0, stream, a);
    return launch_status();
}
}  // namespace

extern "C" int anima_patchify_3d_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int C, int T, int H, int W,
                                      int pT, int pH, int pW, anima_stream_t stream) {
    return patch_op<false>(src, dst, B, C, T, H, W, pT, pH, pW, stream);
}

extern "C" int anima_unpatchify_3d_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int C, int T, int H, int W,
                                        int pT, int pH, int pW, anima_stream_t stream) {
    return patch_op<true>(src, dst, B, C, T, H, W, pT, pH, pW, stream);
}

extern "C" int anima_channel_scale_shift_bf16(const anima_bf16 *x, const anima_bf16 *scale, const anima_bf16 *shift,
                                              anima_bf16 *out, int B, int C, int spatial, anima_stream_t stream) {
    if (B < 0 || C <= 0 || spatial < 0) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)B * C * spatial;
    if (n == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(out, n * 2, x, n * 2) || overlaps(out, n * 2, scale, (int64_t)C * 2) ||
        overlaps(out, n * 2, shift, (int64_t)C * 2))
        return ANIMA_ERR_OVERLAP;
    CssArgs a{x, scale, shift, out, C, spatial, n, spatial % 8 == 0 && aligned16(x) && aligned16(out)};
    int err = ANIMA_OK;
    const unsigned grid =
        wave_grid((const void *)channel_scale_shift_kernel, kSmpBlock, 0, a.vec ? n / 8 : n, &err);
    if (err) return err;
    launch(channel_scale_shift_kernel, grid, kSmpBlock, 0, stream, a);
    return launch_status();
}
