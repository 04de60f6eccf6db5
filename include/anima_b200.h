/*
 * anima_b200.h -- C ABI of the B200 (sm_100a) fused layer kernels for anima.cu.
 *
 * Every entry point enqueues one kernel (or nothing, for empty inputs) on `stream`
 * and returns without synchronising. The caller owns every buffer; the library
 * allocates no device memory and keeps no per-call state. All pointers are device
 * pointers unless stated otherwise. bf16 tensors are passed as uint16_t bit
 * patterns, row-major and densely packed.
 *
 * Return value: ANIMA_OK (0); a negative ANIMA_ERR_* for an argument the library
 * rejected before touching the GPU; or a positive cudaError_t from the launch.
 * In-place use (input pointer == output pointer) is supported wherever the
 * reference's callers use it; partially overlapping buffers are rejected.
 *
 * Reference: TheLegendOfKitty/anima.cu, src/kernels/kernels.h. Each declaration
 * cites the launcher it replaces. A C++ shim in the same library also exports the
 * reference's exact C++ signatures (see anima_kernels_compat.h), so the reference's
 * model files link against this library unchanged.
 */
#ifndef ANIMA_B200_H
#define ANIMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define ANIMA_API __attribute__((visibility("default")))
#else
#define ANIMA_API
#endif

typedef uint16_t anima_bf16;               /* bf16 bit pattern */
typedef struct CUstream_st *anima_stream_t; /* same type as cudaStream_t */

enum {
    ANIMA_OK = 0,
    ANIMA_ERR_NULL_POINTER = -1,  /* a required pointer is NULL */
    ANIMA_ERR_BAD_SHAPE = -2,     /* a size is negative, zero where it must not be, or odd where it must be even */
    ANIMA_ERR_MISALIGNED = -3,    /* a bf16 pointer is not 2-byte aligned (fp32 / int32: 4-byte) */
    ANIMA_ERR_TOO_LARGE = -4,     /* a size overflows the index arithmetic */
    ANIMA_ERR_OVERLAP = -5,       /* an output partially overlaps an input */
    ANIMA_ERR_NO_DEVICE = -6      /* no current CUDA device could be queried */
};

/* Human-readable name of a status code (static storage, never NULL). */
ANIMA_API const char *anima_status_string(int status);

/* Library version, e.g. "anima_b200 0.1.0 sm_100a". */
ANIMA_API const char *anima_version(void);

/* Bounded waits that ran out on the current device: the kernels that stage data with the TMA
 * unit (the channel norm's tile kernel, the GELU / SiLU table kernel) wait on mbarriers with an
 * iteration limit instead of forever; a CTA whose wait runs out skips its output and counts here. Never expected in
 * normal operation. Writes the count to *count (and clears it when reset != 0); call after
 * synchronizing the streams that ran those kernels. New in this library (the reference's
 * kernels have no waits). */
ANIMA_API int anima_wait_timeouts(unsigned int *count, int reset);

/* ------------------------------------------------------------------ row norms */

/* out[n,:] = x[n,:] * rsqrt(mean(x[n,:]^2) + eps) * weight[:]; weight may be NULL.
 * D even. Replaces rms_norm_bf16, kernels.h:9-11 (rms_norm.cu:118-131). */
ANIMA_API int anima_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight, anima_bf16 *out,
                        int N, int D, float eps, anima_stream_t stream);

/* LayerNorm without affine. Replaces layer_norm_bf16, kernels.h:14-16 (layer_norm.cu:61-72). */
ANIMA_API int anima_layer_norm_bf16(const anima_bf16 *x, anima_bf16 *out, int N, int D, float eps,
                          anima_stream_t stream);

/* out = LayerNorm(x) * (1 + scale[d]) + shift[d], scale/shift broadcast over rows.
 * Replaces adaln_layernorm_bf16, kernels.h:19-22 (layer_norm.cu:127-135). */
ANIMA_API int anima_adaln_layernorm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                               const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                               float eps, anima_stream_t stream);

/* hidden = hidden + sub_out * gate[d] (written back as bf16), then
 * normed = LayerNorm(hidden) * (1 + scale[d]) + shift[d]. The statistics use the
 * unrounded fp32 sum; the normalisation reads the bf16-rounded hidden, as the
 * reference does. Replaces residual_gate_adaln_bf16, kernels.h:25-30 (layer_norm.cu:198-209). */
ANIMA_API int anima_residual_gate_adaln_bf16(anima_bf16 *hidden, const anima_bf16 *sub_out,
                                   const anima_bf16 *gate, const anima_bf16 *scale,
                                   const anima_bf16 *shift, anima_bf16 *normed, int N, int D,
                                   float eps, anima_stream_t stream);

/* out = RMSNorm(x) * (1 + scale[n,d]) + shift[n,d] with per-row scale/shift.
 * Replaces adaln_rms_norm_bf16, kernels.h:60-63 (adaln.cu:58-70). */
ANIMA_API int anima_adaln_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                              const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                              float eps, anima_stream_t stream);

/* out = RMSNorm(x) * (1 + weight[d]). Replaces gemma_rms_norm_bf16, kernels.h:151-153
 * (gemma_ops.cu:170-177). */
ANIMA_API int anima_gemma_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight, anima_bf16 *out,
                              int N, int D, float eps, anima_stream_t stream);

/* -------------------------------------------------------------- elementwise */

/* tanh-GELU. The reference processes floor(N/2) element pairs and leaves an odd last
 * element untouched; so does this. Replaces gelu_tanh_bf16, kernels.h:33 (gelu.cu:66-71).
 * On 16-byte-aligned tensors of 2^20 elements or more it reads a 65536-entry table of the
 * reference's outputs: the first such call on a device fills it and waits for `stream` once
 * (a call captured into a CUDA graph before then uses the table-free kernel; same bits).
 * anima_silu_bf16 likewise. */
ANIMA_API int anima_gelu_tanh_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N,
                         anima_stream_t stream);

/* gelu_tanh(x + bias[i % D]). Replaces gelu_tanh_bias_bf16, kernels.h:34-36 (gelu.cu:73-81). */
ANIMA_API int anima_gelu_tanh_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out,
                              int64_t N, int D, anima_stream_t stream);

/* x / (1 + exp(-x)). Replaces silu_bf16, kernels.h:39 (silu.cu:49-54). */
ANIMA_API int anima_silu_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N, anima_stream_t stream);

/* silu(x + bias[i % D]). Replaces silu_bias_bf16, kernels.h:40-42 (silu.cu:56-64). */
ANIMA_API int anima_silu_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out,
                         int64_t N, int D, anima_stream_t stream);

/* out = a + b. Replaces add_bf16, kernels.h:69-71 (elementwise.cu:55-64). */
ANIMA_API int anima_add_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                   anima_stream_t stream);

/* out = a * b. Replaces mul_bf16, kernels.h:78-80 (elementwise.cu:143-152). */
ANIMA_API int anima_mul_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                   anima_stream_t stream);

/* out[m,d] = x[m,d] + bias[d] on [M, D], D even. Replaces bias_add_bf16
 * (kernels.h:81-83, elementwise.cu:184-213; after every biased Linear, linear.cpp:78).
 * out may alias x. */
ANIMA_API int anima_bias_add_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out, int M, int D,
                        anima_stream_t stream);

/* out[m,d] = x[m,d] * (1 + scale[d]) + shift[d]. Replaces scale_shift_bcast_bf16,
 * kernels.h:87-89 (elementwise.cu:238-247). */
ANIMA_API int anima_scale_shift_bcast_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                 const anima_bf16 *shift, anima_bf16 *out, int M, int D,
                                 anima_stream_t stream);

/* out[m,d] = x[m,d] + y[m,d] * gate[d]. Replaces residual_gate_bcast_bf16, kernels.h:90-92
 * (elementwise.cu:271-280). */
ANIMA_API int anima_residual_gate_bcast_bf16(const anima_bf16 *x, const anima_bf16 *y,
                                   const anima_bf16 *gate, anima_bf16 *out, int M, int D,
                                   anima_stream_t stream);

/* out = gelu_tanh(gate) * up (scalar formula of the reference). Replaces gated_gelu_bf16,
 * kernels.h:138-140 (gemma_ops.cu:24-31). */
ANIMA_API int anima_gated_gelu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out,
                          int64_t N, anima_stream_t stream);

/* --------------------------------------------------------------------- RoPE */

/* In-place Cosmos half-split rotation on x[B*S, H*HD]: for i < HD/2,
 * (x_i, x_{i+HD/2}) <- (x_i c - x_{i+HD/2} s, x_{i+HD/2} c + x_i s), with c, s read
 * from the bf16 tables cos/sin [S, HD] at [s_pos, i]. Replaces rope_cosmos_strided_bf16,
 * kernels.h:51-53 (rope.cu:110-121). */
ANIMA_API int anima_rope_cosmos_strided_bf16(anima_bf16 *x, const anima_bf16 *cos_table,
                                   const anima_bf16 *sin_table, int B, int S, int H, int HD,
                                   anima_stream_t stream);

/* In-place half-split rotation on rows of x[total_rows, D] with t = row % T and fp32
 * tables cos/sin [T, D/2]. Replaces rope_standard_bf16, kernels.h:145-147 (gemma_ops.cu:89-97). */
ANIMA_API int anima_rope_standard_bf16(anima_bf16 *x, const float *cos_table, const float *sin_table,
                             int total_rows, int T, int D, anima_stream_t stream);

/* ------------------------------------------------------------------- gather */

/* out[t,:] = table[ids[t],:], bit-exact. ids outside [0, vocab) produce a zero row and,
 * when bad_id_count is non-NULL, increment *bad_id_count (a device int the caller
 * zeroes). vocab <= 0 disables the check (the reference's behaviour). `out` must not
 * overlap `table` or `ids` (rejected with ANIMA_ERR_OVERLAP; with vocab <= 0 the table's
 * extent is unknown and the caller guarantees it).
 * Replaces embedding_lookup_bf16, kernels.h:142-144 (gemma_ops.cu:47-53), which takes
 * no vocabulary size. */
ANIMA_API int anima_embedding_lookup_bf16(const anima_bf16 *table, const int32_t *ids, anima_bf16 *out,
                                int T, int D, int vocab, int32_t *bad_id_count,
                                anima_stream_t stream);

/* ----------------------------------------------------------- VAE channel norm */

/* NCHW: out[b,c,s] = x[b,c,s] * rsqrt(mean_c x[b,:,s]^2 + eps) * gamma[c], one launch
 * for all B. Replaces rms_norm_channel_bf16, kernels.h:177-180 (vae_kernels.cu:83-98). */
ANIMA_API int anima_rms_norm_channel_bf16(const anima_bf16 *x, const anima_bf16 *gamma, anima_bf16 *out,
                                int B, int C, int spatial, float eps, anima_stream_t stream);

/* ------------------------------------------------ new entry points (additive)
 * These have no single reference launcher: each replaces a short chain of reference
 * calls with one kernel and produces the same bits as that chain (the intermediate
 * bf16 rounding is kept). */

/* out[b,c,s] = x[b,c,s] / sqrt(mean_c x[b,:,s]^2 + eps) on NCHW (no gamma; IEEE sqrt and
 * divide as the reference). Replaces pixel_norm_bf16, kernels.h:156-158 (vae_kernels.cu:15-52).
 * out may alias x. */
ANIMA_API int anima_pixel_norm_bf16(const anima_bf16 *x, anima_bf16 *out, int B, int C, int spatial, float eps,
                         anima_stream_t stream);

/* silu(rms_norm_channel(x)) in one pass: the chain rms_norm_channel_bf16 + silu_bf16 at
 * vae.cpp:148,184 (and :189, :457-458). */
ANIMA_API int anima_rms_norm_channel_silu_bf16(const anima_bf16 *x, const anima_bf16 *gamma,
                                     anima_bf16 *out, int B, int C, int spatial, float eps,
                                     anima_stream_t stream);

/* Per-head RMSNorm with weight followed by the Cosmos rotation, in place on
 * x[B*S, H*HD]: the chain rms_norm_bf16 + rope_cosmos_strided_bf16 at
 * transformer.cpp:350-358. */
ANIMA_API int anima_qk_norm_rope_bf16(anima_bf16 *x, const anima_bf16 *weight,
                            const anima_bf16 *cos_table, const anima_bf16 *sin_table, int B,
                            int S, int H, int HD, float eps, anima_stream_t stream);

/* out = silu(gate) * up with silu rounded to bf16 first: the chain silu_bf16 + mul_bf16 at
 * qwen3.cpp:248-250. out may alias gate or up. */
ANIMA_API int anima_swiglu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out, int64_t N,
                      anima_stream_t stream);

/* out = LayerNorm(x) rounded to bf16, then * (1 + scale[d]) + shift[d]: the chain
 * layer_norm_bf16 + scale_shift_bcast_bf16 at transformer.cpp:563-564. */
ANIMA_API int anima_layer_norm_modulate_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                   const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                                   float eps, anima_stream_t stream);

/* ---- sampler steps and latent I/O (kernels.h:186-190, 215-223, 244-276) ----------------- */

/* Fused CFG + Euler step over N elements: noise = neg + cfg*(pos - neg);
 * out = sample - sigma*noise when sigma_next == 0, else sample + d*(sigma_next - sigma)
 * with d = (sample - denoised)/sigma. Replaces cfg_euler_step_bf16 (transpose.cu:250-291).
 * out may alias sample. */
ANIMA_API int anima_cfg_euler_step_bf16(const anima_bf16 *sample, const anima_bf16 *noise_pos,
                             const anima_bf16 *noise_neg, anima_bf16 *out, float cfg_scale,
                             float sigma, float sigma_next, int64_t N, anima_stream_t stream);

/* Fused CFG + Euler-ancestral rectified-flow step; the coefficients are derived from sigma,
 * sigma_next, eta on the host as the reference does. rand_noise (N(0,1) bf16) is read only
 * when eta > 0 and the re-noise coefficient is positive, and may be NULL otherwise.
 * Replaces cfg_euler_a_rf_step_bf16 (transpose.cu:306-364). out may alias sample. */
ANIMA_API int anima_cfg_euler_a_rf_step_bf16(const anima_bf16 *sample, const anima_bf16 *noise_pos,
                                  const anima_bf16 *noise_neg, const anima_bf16 *rand_noise,
                                  anima_bf16 *out, float cfg_scale, float sigma, float sigma_next,
                                  float eta, float s_noise, int64_t N, anima_stream_t stream);

/* Fused CFG + ER-SDE multi-stage step, x updated in place; writes denoised_out, and
 * denoised_d_out when it and old_denoised are non-NULL. old_denoised, old_denoised_d and
 * rand_noise are nullable exactly as in the reference. Replaces cfg_er_sde_full_step_bf16
 * (transpose.cu:386-465). */
ANIMA_API int anima_cfg_er_sde_full_step_bf16(anima_bf16 *x, const anima_bf16 *noise_pos,
                                   const anima_bf16 *noise_neg, anima_bf16 *denoised_out,
                                   const anima_bf16 *old_denoised, anima_bf16 *denoised_d_out,
                                   const anima_bf16 *old_denoised_d, const anima_bf16 *rand_noise,
                                   float cfg_scale, float sigma, float A, float B, float d_scale,
                                   float coeff2, float u_scale, float coeff3, float noise_coeff,
                                   int64_t N, anima_stream_t stream);

/* [B, C, T, H, W] -> [B, S, C*pT*pH*pW], patch element order (c, pt, ph, pw), S over
 * whole patches only. Replaces patchify_3d_bf16 (transpose.cu:132-185), one launch for all
 * B (the reference launches per item). */
ANIMA_API int anima_patchify_3d_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int C, int T, int H,
                          int W, int pT, int pH, int pW, anima_stream_t stream);

/* [B, S, patch_dim] -> [B, C, T, H, W] with the Cosmos projection's (ph, pw, pt, c) patch
 * element order; volume positions outside whole patches are left unwritten. Replaces
 * unpatchify_3d_bf16 (transpose.cu:191-243). */
ANIMA_API int anima_unpatchify_3d_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int C, int T, int H,
                            int W, int pT, int pH, int pW, anima_stream_t stream);

/* out[b,c,s] = x[b,c,s]*scale[c] + shift[c] on NCHW. Replaces channel_scale_shift_bf16
 * (vae_kernels.cu:174-206; the latent denormalisation, vae.cpp:406). out may alias x. */
ANIMA_API int anima_channel_scale_shift_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                  const anima_bf16 *shift, anima_bf16 *out, int B, int C, int spatial,
                                  anima_stream_t stream);

/* dtype conversions over floor(N/2) element pairs (an odd last element is left untouched,
 * as the reference does): replace f32_to_bf16 and bf16_to_f32, kernels.h:96-97
 * (elementwise.cu:311-352; transformer.cpp:543,622, pipeline.cpp:399-609). */
ANIMA_API int anima_f32_to_bf16(const float *x, anima_bf16 *out, int64_t N, anima_stream_t stream);
ANIMA_API int anima_bf16_to_f32(const anima_bf16 *x, float *out, int64_t N, anima_stream_t stream);

/* out = bf16(x * scale) over floor(N/2) element pairs. Replaces scale_bf16, kernels.h:75-76
 * (elementwise.cu:97-122; the initial noise, pipeline.cpp:519). out may alias x. */
ANIMA_API int anima_scale_bf16(const anima_bf16 *x, anima_bf16 *out, float scale, int64_t N, anima_stream_t stream);

/* [B, C, H, W] -> [B, C, 2H, 2W], each input element repeated 2x2. Replaces
 * nearest_upsample_2x_bf16, kernels.h:172-174 (vae_kernels.cu:98-133; vae.cpp:339). in and
 * out may not overlap. */
ANIMA_API int anima_nearest_upsample_2x_bf16(const anima_bf16 *in, anima_bf16 *out, int B, int C, int H, int W,
                                  anima_stream_t stream);

/* Attention glue of the Qwen3 encoder and the LLM adapter (qwen3.cpp:164-226,
 * llm_adapter.cpp:169-222). Head layout changes: [T, H*HD] <-> [H, T, HD]
 * (head_transpose_bf16 / head_untranspose_bf16, transpose.cu:13-66) and
 * [B*S, H*HD] <-> [B, H, S, HD] (the _batched forms, transpose.cu:68-123). src and dst may
 * not overlap. */
ANIMA_API int anima_head_transpose_bf16(const anima_bf16 *src, anima_bf16 *dst, int H, int T, int HD,
                             anima_stream_t stream);
ANIMA_API int anima_head_untranspose_bf16(const anima_bf16 *src, anima_bf16 *dst, int H, int T, int HD,
                               anima_stream_t stream);
ANIMA_API int anima_head_transpose_batched_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int H, int S,
                                     int HD, anima_stream_t stream);
ANIMA_API int anima_head_untranspose_batched_bf16(const anima_bf16 *src, anima_bf16 *dst, int B, int H, int S,
                                       int HD, anima_stream_t stream);

/* head_transpose_bf16 + rms_norm_bf16 on each head row + rope_standard_bf16 in one pass:
 * dst[h, t, :] = rope(bf16(rms_norm(src[t, h*HD : (h+1)*HD]) * weight[:])), the chain at
 * qwen3.cpp:164-178 for q and k (and llm_adapter.cpp:169-187). weight may be NULL (no
 * weight), cos_table/sin_table ([T, HD/2] fp32) may both be NULL (no rotation). HD = 128
 * runs one fused kernel; other head sizes run the three steps. src and dst may not
 * overlap. No reference counterpart (opt-in). */
ANIMA_API int anima_head_transpose_qk_norm_rope_bf16(const anima_bf16 *src, const anima_bf16 *weight,
                                          const float *cos_table, const float *sin_table, anima_bf16 *dst,
                                          int H, int T, int HD, float eps, anima_stream_t stream);

/* GQA expansion [B, KV_H, T, D] -> [B, Q_H, T, D], q head h reading kv head h / (Q_H / KV_H).
 * Replaces expand_kv_bf16 (gemma_ops.cu:99-127). Q_H must be a multiple of KV_H (the
 * reference reads past kv otherwise); rejected with ANIMA_ERR_BAD_SHAPE. */
ANIMA_API int anima_expand_kv_bf16(const anima_bf16 *kv, anima_bf16 *out, int B, int KV_H, int Q_H, int T,
                        int D, anima_stream_t stream);

/* scores[h, i, j] = bf16(-1e9) for j > i, in place on [num_heads, T, T]. Replaces
 * causal_mask_bf16 (softmax.cu:62-80). */
ANIMA_API int anima_causal_mask_bf16(anima_bf16 *scores, int num_heads, int T, anima_stream_t stream);

/* Row-wise softmax of x[N, D] into out (out may alias x). Replaces softmax_bf16
 * (softmax.cu:8-60,115-122), bit for bit. */
ANIMA_API int anima_softmax_bf16(const anima_bf16 *x, anima_bf16 *out, int N, int D, anima_stream_t stream);

/* causal_mask_bf16 followed by softmax_bf16 on [num_heads, T, T] (qwen3.cpp:205-208) in one
 * pass; wholly masked 16-byte chunks are not read. out may alias scores. No reference
 * counterpart (opt-in). */
ANIMA_API int anima_causal_softmax_bf16(const anima_bf16 *scores, anima_bf16 *out, int num_heads, int T,
                             anima_stream_t stream);

/* Row-wise softmax of fp32 x[N, D] into bf16 out. Replaces softmax_f32_to_bf16
 * (softmax.cu:153-252; the VAE attention, vae.cpp:262), bit for bit. */
ANIMA_API int anima_softmax_f32_to_bf16(const float *x, anima_bf16 *out, int N, int D, anima_stream_t stream);

/* out[b,c,s] = x[b,c,s] + bias[c] on NCHW: the convolution's bias add, the file-local
 * conv_bias_add_kernel launched by causal_conv3d_forward after every biased conv
 * (causal_conv3d.cu:187-195, :247-254, :293-299). The caller runs the conv without its bias
 * and calls this. out may alias x (the reference adds in place). */
ANIMA_API int anima_conv_bias_add_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out,
                            int B, int C, int spatial, anima_stream_t stream);

/* out = (x + bias[c]) + residual in one pass, each sum rounded to bf16: the conv's bias launch
 * followed by add_bf16(out, residual, out) at vae.cpp:190-194 (residual block) and :277-280
 * (attention projection). out may alias x or residual. */
ANIMA_API int anima_conv_bias_residual_add_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                     const anima_bf16 *residual, anima_bf16 *out, int B, int C,
                                     int spatial, anima_stream_t stream);

/* silu(rms_norm_channel(x + bias[c])) in one pass: the conv's bias launch, then
 * rms_norm_channel_bf16 and silu_bf16 (vae.cpp:185-189, a residual block's conv1 into
 * norm2). The biased conv output is not stored. out may alias x. */
ANIMA_API int anima_conv_bias_rms_norm_channel_silu_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                              const anima_bf16 *gamma, anima_bf16 *out, int B, int C,
                                              int spatial, float eps, anima_stream_t stream);

/* adaLN-Zero modulation folded into adaLN LayerNorm. One launch replaces the chain
 *   add_bf16(mod, temb, mod, 3*D); adaln_layernorm_bf16(x, mod + D, mod, out, N, D, eps);
 *   cudaMemcpyAsync(gate, mod + 2*D, 2*D, DeviceToDevice)            (transformer.cpp:404-425)
 * mod = [shift | scale | gate] as the modulation Linear wrote it (before the temb add),
 * temb = [3*D]. out is the chain's normed output and gate_out[D] receives
 * bf16(mod_gate + temb_gate), bit for bit; mod itself is left unchanged. gate_out may not
 * overlap any other argument. */
ANIMA_API int anima_adaln_layernorm_temb_bf16(const anima_bf16 *x, const anima_bf16 *mod,
                                   const anima_bf16 *temb, anima_bf16 *gate_out, anima_bf16 *out,
                                   int N, int D, float eps, anima_stream_t stream);

/* The same fold for the fused residual gate: one launch replaces
 *   add_bf16(mod, temb, mod, 3*D);
 *   residual_gate_adaln_bf16(hidden, sub_out, gate, mod + D, mod, normed, N, D, eps);
 *   cudaMemcpyAsync(gate, mod + 2*D, 2*D, DeviceToDevice)            (transformer.cpp:433-456)
 * gate_in is the previous set's gate (the chain's `gate` buffer before the copy);
 * gate_out receives this set's, so the caller alternates two gate buffers. gate_out may
 * not overlap any other argument. */
ANIMA_API int anima_residual_gate_adaln_temb_bf16(anima_bf16 *hidden, const anima_bf16 *sub_out,
                                       const anima_bf16 *gate_in, const anima_bf16 *mod,
                                       const anima_bf16 *temb, anima_bf16 *gate_out,
                                       anima_bf16 *normed, int N, int D, float eps,
                                       anima_stream_t stream);

/* Timestep embedding on the GPU: writes the flip_sin_to_cos sinusoid of `timestep`
 * (cos of t*f_i in [0, dim/2), sin in [dim/2, dim), f_i = exp(-ln(1e4) i / (dim/2)))
 * as bf16 to sinusoid_out[dim], and, when normed_out is non-NULL, its RMSNorm times
 * norm_weight (nullable) to normed_out[dim]. The reference builds the sinusoid on the
 * host and uploads it (transformer.cpp:182-197) before rms_norm_bf16 (:200). dim even.
 * Not bit-exact with that host loop: exp/cos/sin are correctly rounded here, glibc's fp32
 * functions are not everywhere, so rare elements differ by one bf16 ulp. */
ANIMA_API int anima_timestep_embedding_bf16(float timestep, const anima_bf16 *norm_weight,
                                  anima_bf16 *sinusoid_out, anima_bf16 *normed_out, int dim,
                                  float eps, anima_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ANIMA_B200_H */
