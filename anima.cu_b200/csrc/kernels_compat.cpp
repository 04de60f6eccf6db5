// kernels_compat.cpp -- the reference's C++ launcher signatures (src/kernels/kernels.h),
// forwarding to the C ABI. Host code only: no kernels live here.
#include "../../include/anima_kernels_compat.h"

#include "../../include/anima_b200.h"

namespace {

thread_local int g_last_error = ANIMA_OK;

inline void record(int status) {
    if (status != ANIMA_OK && g_last_error == ANIMA_OK) g_last_error = status;
}

inline const anima_bf16 *in(const __nv_bfloat16 *p) { return reinterpret_cast<const anima_bf16 *>(p); }
inline anima_bf16 *io(__nv_bfloat16 *p) { return reinterpret_cast<anima_bf16 *>(p); }

}  // namespace

extern "C" int anima_compat_last_error(void) {
    const int e = g_last_error;
    g_last_error = ANIMA_OK;
    return e;
}

void rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *weight, __nv_bfloat16 *out, int N,
                   int D, float eps, cudaStream_t stream) {
    record(anima_rms_norm_bf16(in(x), in(weight), io(out), N, D, eps, stream));
}

void layer_norm_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int N, int D, float eps,
                     cudaStream_t stream) {
    record(anima_layer_norm_bf16(in(x), io(out), N, D, eps, stream));
}

void adaln_layernorm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                          const __nv_bfloat16 *shift, __nv_bfloat16 *out, int N, int D, float eps,
                          cudaStream_t stream) {
    record(anima_adaln_layernorm_bf16(in(x), in(scale), in(shift), io(out), N, D, eps, stream));
}

void residual_gate_adaln_bf16(__nv_bfloat16 *hidden, const __nv_bfloat16 *sub_out,
                              const __nv_bfloat16 *gate, const __nv_bfloat16 *scale,
                              const __nv_bfloat16 *shift, __nv_bfloat16 *normed, int N, int D,
                              float eps, cudaStream_t stream) {
    record(anima_residual_gate_adaln_bf16(io(hidden), in(sub_out), in(gate), in(scale), in(shift),
                                          io(normed), N, D, eps, stream));
}

void gelu_tanh_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream) {
    record(anima_gelu_tanh_bf16(in(x), io(out), N, stream));
}

void gelu_tanh_bias_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out,
                         int64_t N, int D, cudaStream_t stream) {
    record(anima_gelu_tanh_bias_bf16(in(x), in(bias), io(out), N, D, stream));
}

void silu_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream) {
    record(anima_silu_bf16(in(x), io(out), N, stream));
}

void silu_bias_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out, int64_t N,
                    int D, cudaStream_t stream) {
    record(anima_silu_bias_bf16(in(x), in(bias), io(out), N, D, stream));
}

void rope_cosmos_strided_bf16(__nv_bfloat16 *x, const __nv_bfloat16 *cos_freq,
                              const __nv_bfloat16 *sin_freq, int B, int S, int H, int HD,
                              cudaStream_t stream) {
    record(anima_rope_cosmos_strided_bf16(io(x), in(cos_freq), in(sin_freq), B, S, H, HD, stream));
}

void adaln_rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                         const __nv_bfloat16 *shift, __nv_bfloat16 *out, int N, int D, float eps,
                         cudaStream_t stream) {
    record(anima_adaln_rms_norm_bf16(in(x), in(scale), in(shift), io(out), N, D, eps, stream));
}

void add_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, __nv_bfloat16 *out, int64_t N,
              cudaStream_t stream) {
    record(anima_add_bf16(in(a), in(b), io(out), N, stream));
}

void mul_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, __nv_bfloat16 *out, int64_t N,
              cudaStream_t stream) {
    record(anima_mul_bf16(in(a), in(b), io(out), N, stream));
}

void bias_add_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out, int M, int D,
                   cudaStream_t stream) {
    record(anima_bias_add_bf16(in(x), in(bias), io(out), M, D, stream));
}

void scale_shift_bcast_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                            const __nv_bfloat16 *shift, __nv_bfloat16 *out, int M, int D,
                            cudaStream_t stream) {
    record(anima_scale_shift_bcast_bf16(in(x), in(scale), in(shift), io(out), M, D, stream));
}

void residual_gate_bcast_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *y,
                              const __nv_bfloat16 *gate, __nv_bfloat16 *out, int M, int D,
                              cudaStream_t stream) {
    record(anima_residual_gate_bcast_bf16(in(x), in(y), in(gate), io(out), M, D, stream));
}

void gated_gelu_bf16(const __nv_bfloat16 *gate, const __nv_bfloat16 *up, __nv_bfloat16 *out,
                     int64_t N, cudaStream_t stream) {
    record(anima_gated_gelu_bf16(in(gate), in(up), io(out), N, stream));
}

void embedding_lookup_bf16(const __nv_bfloat16 *table, const int *ids, __nv_bfloat16 *out, int T,
                           int D, cudaStream_t stream) {
    // The reference interface carries no vocabulary size, so ids are not range-checked.
    record(anima_embedding_lookup_bf16(in(table), reinterpret_cast<const int32_t *>(ids), io(out), T,
                                       D, 0, nullptr, stream));
}

void rope_standard_bf16(__nv_bfloat16 *x, const float *cos_cache, const float *sin_cache,
                        int total_rows, int T, int D, cudaStream_t stream) {
    record(anima_rope_standard_bf16(io(x), cos_cache, sin_cache, total_rows, T, D, stream));
}

void gemma_rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *weight, __nv_bfloat16 *out,
                         int N, int D, float eps, cudaStream_t stream) {
    record(anima_gemma_rms_norm_bf16(in(x), in(weight), io(out), N, D, eps, stream));
}

void rms_norm_channel_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *gamma, __nv_bfloat16 *out,
                           int B, int C, int spatial, float eps, cudaStream_t stream) {
    record(anima_rms_norm_channel_bf16(in(x), in(gamma), io(out), B, C, spatial, eps, stream));
}

void channel_scale_shift_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale, const __nv_bfloat16 *shift,
                              __nv_bfloat16 *out, int B, int C, int spatial, cudaStream_t stream) {
    record(anima_channel_scale_shift_bf16(in(x), in(scale), in(shift), io(out), B, C, spatial, stream));
}

void scale_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, float scale, int64_t N, cudaStream_t stream) {
    record(anima_scale_bf16(in(x), io(out), scale, N, stream));
}

void f32_to_bf16(const float *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream) {
    record(anima_f32_to_bf16(x, io(out), N, stream));
}

void bf16_to_f32(const __nv_bfloat16 *x, float *out, int64_t N, cudaStream_t stream) {
    record(anima_bf16_to_f32(in(x), out, N, stream));
}

void nearest_upsample_2x_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int C, int H, int W,
                              cudaStream_t stream) {
    record(anima_nearest_upsample_2x_bf16(in(src), io(dst), B, C, H, W, stream));
}

void causal_mask_bf16(__nv_bfloat16 *scores, int num_heads, int T, cudaStream_t stream) {
    record(anima_causal_mask_bf16(io(scores), num_heads, T, stream));
}

void softmax_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int N, int D, cudaStream_t stream) {
    record(anima_softmax_bf16(in(x), io(out), N, D, stream));
}

void softmax_f32_to_bf16(const float *x, __nv_bfloat16 *out, int N, int D, cudaStream_t stream) {
    record(anima_softmax_f32_to_bf16(x, io(out), N, D, stream));
}

void expand_kv_bf16(const __nv_bfloat16 *kv, __nv_bfloat16 *out, int B, int KV_H, int Q_H, int T, int D,
                    cudaStream_t stream) {
    record(anima_expand_kv_bf16(in(kv), io(out), B, KV_H, Q_H, T, D, stream));
}

void head_transpose_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int H, int T, int HD, cudaStream_t stream) {
    record(anima_head_transpose_bf16(in(src), io(dst), H, T, HD, stream));
}

void head_untranspose_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int H, int T, int HD,
                           cudaStream_t stream) {
    record(anima_head_untranspose_bf16(in(src), io(dst), H, T, HD, stream));
}

void head_transpose_batched_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int H, int S, int HD,
                                 cudaStream_t stream) {
    record(anima_head_transpose_batched_bf16(in(src), io(dst), B, H, S, HD, stream));
}

void head_untranspose_batched_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int H, int S, int HD,
                                   cudaStream_t stream) {
    record(anima_head_untranspose_batched_bf16(in(src), io(dst), B, H, S, HD, stream));
}

void pixel_norm_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int B, int C, int spatial, float eps,
                     cudaStream_t stream) {
    record(anima_pixel_norm_bf16(in(x), io(out), B, C, spatial, eps, stream));
}

void patchify_3d_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int C, int T, int H, int W, int pT,
                      int pH, int pW, cudaStream_t stream) {
    record(anima_patchify_3d_bf16(in(src), io(dst), B, C, T, H, W, pT, pH, pW, stream));
}

void unpatchify_3d_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int C, int T, int H, int W, int pT,
                        int pH, int pW, cudaStream_t stream) {
    record(anima_unpatchify_3d_bf16(in(src), io(dst), B, C, T, H, W, pT, pH, pW, stream));
}

void cfg_euler_step_bf16(const __nv_bfloat16 *sample, const __nv_bfloat16 *noise_pos,
                         const __nv_bfloat16 *noise_neg, __nv_bfloat16 *out, float cfg_scale, float sigma,
                         float sigma_next, int64_t N, cudaStream_t stream) {
    record(anima_cfg_euler_step_bf16(in(sample), in(noise_pos), in(noise_neg), io(out), cfg_scale, sigma,
                                     sigma_next, N, stream));
}

void cfg_euler_a_rf_step_bf16(const __nv_bfloat16 *sample, const __nv_bfloat16 *noise_pos,
                              const __nv_bfloat16 *noise_neg, const __nv_bfloat16 *rand_noise,
                              __nv_bfloat16 *out, float cfg_scale, float sigma, float sigma_next, float eta,
                              float s_noise, int64_t N, cudaStream_t stream) {
    record(anima_cfg_euler_a_rf_step_bf16(in(sample), in(noise_pos), in(noise_neg), in(rand_noise), io(out),
                                          cfg_scale, sigma, sigma_next, eta, s_noise, N, stream));
}

void cfg_er_sde_full_step_bf16(__nv_bfloat16 *x, const __nv_bfloat16 *noise_pos, const __nv_bfloat16 *noise_neg,
                               __nv_bfloat16 *denoised_out, const __nv_bfloat16 *old_denoised,
                               __nv_bfloat16 *denoised_d_out, const __nv_bfloat16 *old_denoised_d,
                               const __nv_bfloat16 *rand_noise, float cfg_scale, float sigma, float A, float B,
                               float d_scale, float coeff2, float u_scale, float coeff3, float noise_coeff,
                               int64_t N, cudaStream_t stream) {
    record(anima_cfg_er_sde_full_step_bf16(io(x), in(noise_pos), in(noise_neg), io(denoised_out), in(old_denoised),
                                           io(denoised_d_out), in(old_denoised_d), in(rand_noise), cfg_scale, sigma,
                                           A, B, d_scale, coeff2, u_scale, coeff3, noise_coeff, N, stream));
}
