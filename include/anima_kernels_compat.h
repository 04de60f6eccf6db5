// anima_kernels_compat.h -- the reference's C++ kernel launcher interface, served by the
// B200 library.
//
// libanima_b200.so defines these functions with the exact C++ signatures (and therefore
// the exact mangled symbol names) that TheLegendOfKitty/anima.cu declares in
// src/kernels/kernels.h, so the reference's transformer.cpp, qwen3.cpp, llm_adapter.cpp
// and vae.cpp link against this library without source changes. Default arguments match
// the reference's (eps = 1e-6f, stream = 0). A caller that already includes the
// reference's kernels.h does not need this header; it exists for new callers and as the
// list of what the library serves.
//
// Like the reference, these return void. Errors (argument checks and launch failures)
// are recorded per host thread: anima_compat_last_error() returns the first status
// recorded since the previous call and clears it.
#pragma once

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

// kernels.h:9-11
void rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *weight, __nv_bfloat16 *out, int N,
                   int D, float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:14-16
void layer_norm_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int N, int D, float eps = 1e-6f,
                     cudaStream_t stream = 0);
// kernels.h:19-22
void adaln_layernorm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                          const __nv_bfloat16 *shift, __nv_bfloat16 *out, int N, int D,
                          float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:25-30
void residual_gate_adaln_bf16(__nv_bfloat16 *hidden, const __nv_bfloat16 *sub_out,
                              const __nv_bfloat16 *gate, const __nv_bfloat16 *scale,
                              const __nv_bfloat16 *shift, __nv_bfloat16 *normed, int N, int D,
                              float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:33-36
void gelu_tanh_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream = 0);
void gelu_tanh_bias_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out,
                         int64_t N, int D, cudaStream_t stream = 0);
// kernels.h:39-42
void silu_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream = 0);
void silu_bias_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out,
                    int64_t N, int D, cudaStream_t stream = 0);
// kernels.h:51-53
void rope_cosmos_strided_bf16(__nv_bfloat16 *x, const __nv_bfloat16 *cos_freq,
                              const __nv_bfloat16 *sin_freq, int B, int S, int H, int HD,
                              cudaStream_t stream = 0);
// kernels.h:60-63
void adaln_rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                         const __nv_bfloat16 *shift, __nv_bfloat16 *out, int N, int D,
                         float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:69-71, 78-80
void add_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, __nv_bfloat16 *out, int64_t N,
              cudaStream_t stream = 0);
void mul_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, __nv_bfloat16 *out, int64_t N,
              cudaStream_t stream = 0);
// kernels.h:81-83
void bias_add_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *out, int M, int D,
                   cudaStream_t stream = 0);
// kernels.h:87-92
void scale_shift_bcast_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale,
                            const __nv_bfloat16 *shift, __nv_bfloat16 *out, int M, int D,
                            cudaStream_t stream = 0);
void residual_gate_bcast_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *y,
                              const __nv_bfloat16 *gate, __nv_bfloat16 *out, int M, int D,
                              cudaStream_t stream = 0);
// kernels.h:138-147, 151-153
void gated_gelu_bf16(const __nv_bfloat16 *gate, const __nv_bfloat16 *up, __nv_bfloat16 *out,
                     int64_t N, cudaStream_t stream = 0);
void embedding_lookup_bf16(const __nv_bfloat16 *table, const int *ids, __nv_bfloat16 *out, int T,
                           int D, cudaStream_t stream = 0);
void rope_standard_bf16(__nv_bfloat16 *x, const float *cos_cache, const float *sin_cache,
                        int total_rows, int T, int D, cudaStream_t stream = 0);
void gemma_rms_norm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *weight, __nv_bfloat16 *out,
                         int N, int D, float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:177-180
void rms_norm_channel_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *gamma, __nv_bfloat16 *out,
                           int B, int C, int spatial, float eps = 1e-6f, cudaStream_t stream = 0);
// kernels.h:156-158
void pixel_norm_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int B, int C, int spatial, float eps = 1e-6f,
                     cudaStream_t stream = 0);
// kernels.h:172-174
void nearest_upsample_2x_bf16(const __nv_bfloat16 *in, __nv_bfloat16 *out, int B, int C, int H, int W,
                              cudaStream_t stream = 0);
// kernels.h:189-192
void channel_scale_shift_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *scale, const __nv_bfloat16 *shift,
                              __nv_bfloat16 *out, int B, int C, int spatial, cudaStream_t stream = 0);
// kernels.h:215-223
void patchify_3d_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int C, int T, int H, int W, int pT,
                      int pH, int pW, cudaStream_t stream = 0);
void unpatchify_3d_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int C, int T, int H, int W, int pT,
                        int pH, int pW, cudaStream_t stream = 0);
// kernels.h:75-76
void scale_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, float scale, int64_t N, cudaStream_t stream = 0);
// kernels.h:96-97
void f32_to_bf16(const float *x, __nv_bfloat16 *out, int64_t N, cudaStream_t stream = 0);
void bf16_to_f32(const __nv_bfloat16 *x, float *out, int64_t N, cudaStream_t stream = 0);
// kernels.h:104-117
void causal_mask_bf16(__nv_bfloat16 *scores, int num_heads, int T, cudaStream_t stream = 0);
void softmax_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *out, int N, int D, cudaStream_t stream = 0);
void softmax_f32_to_bf16(const float *x, __nv_bfloat16 *out, int N, int D, cudaStream_t stream = 0);
// kernels.h:148-150
void expand_kv_bf16(const __nv_bfloat16 *kv, __nv_bfloat16 *out, int B, int KV_H, int Q_H, int T, int D,
                    cudaStream_t stream = 0);
// kernels.h:195-212
void head_transpose_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int H, int T, int HD, cudaStream_t stream = 0);
void head_untranspose_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int H, int T, int HD,
                           cudaStream_t stream = 0);
void head_transpose_batched_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int H, int S, int HD,
                                 cudaStream_t stream = 0);
void head_untranspose_batched_bf16(const __nv_bfloat16 *src, __nv_bfloat16 *dst, int B, int H, int S, int HD,
                                   cudaStream_t stream = 0);
// kernels.h:244-276
void cfg_euler_step_bf16(const __nv_bfloat16 *sample, const __nv_bfloat16 *noise_pos,
                         const __nv_bfloat16 *noise_neg, __nv_bfloat16 *out, float cfg_scale, float sigma,
                         float sigma_next, int64_t N, cudaStream_t stream = 0);
void cfg_euler_a_rf_step_bf16(const __nv_bfloat16 *sample, const __nv_bfloat16 *noise_pos,
                              const __nv_bfloat16 *noise_neg, const __nv_bfloat16 *rand_noise,
                              __nv_bfloat16 *out, float cfg_scale, float sigma, float sigma_next, float eta,
                              float s_noise, int64_t N, cudaStream_t stream = 0);
void cfg_er_sde_full_step_bf16(__nv_bfloat16 *x, const __nv_bfloat16 *noise_pos, const __nv_bfloat16 *noise_neg,
                               __nv_bfloat16 *denoised_out, const __nv_bfloat16 *old_denoised,
                               __nv_bfloat16 *denoised_d_out, const __nv_bfloat16 *old_denoised_d,
                               const __nv_bfloat16 *rand_noise, float cfg_scale, float sigma, float A, float B,
                               float d_scale, float coeff2, float u_scale, float coeff3, float noise_coeff,
                               int64_t N, cudaStream_t stream = 0);

extern "C" int anima_compat_last_error(void);
