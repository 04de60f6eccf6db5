/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the arithmetic of anima.cu's fused layer kernels
 * (the .cu files under src/kernels) and of the host-side table builders that feed them. It is
 * the checker the parity tests compare the CUDA library against; nothing in the
 * product links or calls it. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load it.
 *
 * bf16 values travel as uint16_t bit patterns. Each function names the
 * reference file:line whose arithmetic it follows. Where the reference's
 * floating-point result depends on its CUDA thread layout (block reductions),
 * the restatement reproduces that layout: per-thread strided partial sums, the
 * warp shfl_down tree (src/cuda_utils.cuh:46-50) and the cross-warp tree
 * through shared memory (src/kernels/layer_norm.cu:7-19).
 *
 * The reference's per-element expressions leave a few fused-multiply-add
 * contractions to nvcc. Those choices are parameters here ("mode" arguments);
 * the parity tests pin them against the reference kernels' own outputs.
 */
#ifndef ANIMA_ORACLE_H
#define ANIMA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 <-> f32, round-to-nearest-even with NaN -> 0x7fff (cuda_bf16 host semantics). */
float    oracle_bf16_to_f32(uint16_t b);
uint16_t oracle_f32_to_bf16(float f);

/* The reference's CTA reduction of per-thread partials (layer_norm.cu:7-19,
 * rms_norm.cu:40-53): nthreads is the launched block size. */
float oracle_ref_block_sum(const float *per_thread, int nthreads);

/* Block size the reference launchers pick for a row of D elements
 * (layer_norm.cu:68-70, rms_norm.cu:126-128). */
int oracle_ref_row_threads(int D);

/* layer_norm.cu:26-72 -- LayerNorm without affine. */
void oracle_layer_norm(const uint16_t *x, uint16_t *out, int N, int D, float eps,
                       int var_mode);

/* layer_norm.cu:83-135 -- LN(x)*(1+scale[d])+shift[d]. */
void oracle_adaln_layernorm(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                            uint16_t *out, int N, int D, float eps, int var_mode);

/* layer_norm.cu:146-209 -- hidden = x + y*gate[d] (in place, bf16);
 * normed = LN(hidden)*(1+scale)+shift. Stats from the fp32 h, pass 2 from bf16(h).
 * sq_mode: 0 fma(h0,h0,h1*h1), 1 fma(h1,h1,h0*h0), 2 h0*h0+h1*h1 unfused. */
void oracle_residual_gate_adaln(uint16_t *hidden, const uint16_t *sub_out,
                                const uint16_t *gate, const uint16_t *scale,
                                const uint16_t *shift, uint16_t *normed, int N, int D,
                                float eps, int sq_mode, int var_mode);

/* rms_norm.cu:9-67,118-131 -- x*rsqrt(mean x^2+eps)*w[d]; weight may be NULL. */
void oracle_rms_norm(const uint16_t *x, const uint16_t *weight, uint16_t *out, int N, int D,
                     float eps);

/* adaln.cu:11-58 -- RMS(x)*(1+scale[n,d])+shift[n,d] with per-row scale/shift. */
void oracle_adaln_rms_norm(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                           uint16_t *out, int N, int D, float eps);

/* gemma_ops.cu:132-177 -- RMS(x)*(1+w[d]), scalar loop, block over D. */
void oracle_gemma_rms_norm(const uint16_t *x, const uint16_t *weight, uint16_t *out, int N,
                           int D, float eps);

/* gelu.cu:12-34 / :37-64 -- tanh GELU, optionally of x+bias[d]. bias may be NULL. */
void oracle_gelu_tanh(const uint16_t *x, const uint16_t *bias, uint16_t *out, int64_t N, int D);

/* silu.cu:7-24 / :26-47 -- x/(1+exp(-x)), optionally of x+bias[d]. bias may be NULL. */
void oracle_silu(const uint16_t *x, const uint16_t *bias, uint16_t *out, int64_t N, int D);

/* gemma_ops.cu:5-22 -- gelu_tanh(gate)*up, scalar formula. */
void oracle_gated_gelu(const uint16_t *gate, const uint16_t *up, uint16_t *out, int64_t N);

/* elementwise.cu:37-53 (add), :125-141 (mul). */
void oracle_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t N);
void oracle_mul(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t N);

/* elementwise.cu:216-236 -- fma(x, 1+scale[d], shift[d]). */
void oracle_bias_add(const uint16_t *x, const uint16_t *bias, uint16_t *out, int M, int D);
void oracle_scale_shift_bcast(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                              uint16_t *out, int M, int D);

/* elementwise.cu:249-269 -- fma(y, gate[d], x). */
void oracle_residual_gate_bcast(const uint16_t *x, const uint16_t *y, const uint16_t *gate,
                                uint16_t *out, int M, int D);

/* rope.cu:72-108 -- in-place half-split rotation on [B*S, H*HD] with bf16 [S,HD] tables. */
void oracle_rope_cosmos_strided(uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                                int B, int S, int H, int HD);

/* gemma_ops.cu:62-87 -- in-place half-split rotation on rows of [rows, D], t = row % T,
 * fp32 tables [T, D/2]. mode_a picks the contraction of x1*c - x2*s, mode_b that of
 * x2*c + x1*s: 0 fma(first product, ., -second), 1 fma(second, ., first), 2 unfused. */
void oracle_rope_standard(uint16_t *x, const float *cos_t, const float *sin_t,
                          int total_rows, int T, int D, int mode_a, int mode_b);

/* gemma_ops.cu:34-45 -- out[t,:] = table[ids[t],:]. Out-of-range ids produce zeros
 * here (the reference does not check them). */
void oracle_embedding_lookup(const uint16_t *table, const int32_t *ids, uint16_t *out, int T,
                             int D, int vocab);

/* vae_kernels.cu:15-52 -- NCHW pixel norm: x / sqrt(mean_c x^2 + eps), no gamma. */
void oracle_pixel_norm(const uint16_t *x, uint16_t *out, int B, int C, int spatial, float eps);

/* vae_kernels.cu:60-98 -- NCHW channel RMSNorm times gamma[c]; sequential sum over c. */
void oracle_rms_norm_channel(const uint16_t *x, const uint16_t *gamma, uint16_t *out, int B,
                             int C, int spatial, float eps);

/* transpose.cu:13-123 -- [B, S, H, HD] -> [B, H, S, HD] (to_heads = 1, head_transpose) or
 * back (to_heads = 0, head_untranspose); B = 1 gives the unbatched launchers. */
void oracle_head_permute(const uint16_t *src, uint16_t *dst, int B, int H, int S, int HD, int to_heads);

/* gemma_ops.cu:99-127 -- out[b, q, :] = kv[b, q / (QH / KVH), :] over [T*D] planes. */
void oracle_expand_kv(const uint16_t *kv, uint16_t *out, int B, int KVH, int QH, int T, int D);

/* softmax.cu:62-80 -- scores[h, i, j] = bf16(-1e9) for j > i, in place. */
void oracle_causal_mask(uint16_t *scores, int H, int T);

/* softmax.cu:8-60,115-122 -- row softmax in the reference CTA's summation order. */
void oracle_softmax(const uint16_t *x, uint16_t *out, int N, int D);

/* softmax.cu:153-252 -- fp32 rows, per-thread running (max, sum) merged along the
 * reference's shuffle trees; bf16 out. */
void oracle_softmax_f32_to_bf16(const float *x, uint16_t *out, int N, int D);

/* causal_conv3d.cu:187-195 -- out[b,c,s] = x + bias[c] (the conv's bias launch, per batch
 * item there); with residual non-NULL, then out = out + residual[b,c,s] as add_bf16
 * (elementwise.cu:37-53) does it at vae.cpp:194 and :280. */
void oracle_conv_bias_add(const uint16_t *x, const uint16_t *bias, const uint16_t *residual,
                          uint16_t *out, int B, int C, int spatial);

/* vae_kernels.cu:174-206 -- out[b,c,s] = x*scale[c] + shift[c] (one fma). */
void oracle_channel_scale_shift(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                                uint16_t *out, int B, int C, int spatial);

/* transpose.cu:132-243 -- 3-D patchify ([B,C,T,H,W] -> [B,S,C*pT*pH*pW], element order
 * c,pt,ph,pw) and unpatchify ([B,S,pd] -> [B,C,T,H,W], element order ph,pw,pt,c; volume
 * positions outside whole patches are left as they are). */
void oracle_patchify_3d(const uint16_t *src, uint16_t *dst, int B, int C, int T, int H, int W,
                        int pT, int pH, int pW);
void oracle_unpatchify_3d(const uint16_t *src, uint16_t *dst, int B, int C, int T, int H, int W,
                          int pT, int pH, int pW);

/* transpose.cu:250-465 -- the fused CFG sampler steps. Products that nvcc fuses into an fma
 * are written as fmaf; in a sum of two products the first product is fused (a choice that
 * small fixtures cannot distinguish from the other: compared within 1 bf16 ulp). The
 * Euler-ancestral coefficients are derived in host float arithmetic as the launcher does
 * (transpose.cu:345-354). Pointers the reference treats as nullable may be NULL here. */
void oracle_cfg_euler_step(const uint16_t *sample, const uint16_t *pos, const uint16_t *neg,
                           uint16_t *out, float cfg, float sigma, float sigma_next, int64_t n);
void oracle_cfg_euler_a_rf_step(const uint16_t *sample, const uint16_t *pos, const uint16_t *neg,
                                const uint16_t *rand_noise, uint16_t *out, float cfg, float sigma,
                                float sigma_next, float eta, float s_noise, int64_t n);
void oracle_cfg_er_sde_full_step(uint16_t *x, const uint16_t *pos, const uint16_t *neg,
                                 uint16_t *den_out, const uint16_t *old_den, uint16_t *dd_out,
                                 const uint16_t *old_dd, const uint16_t *rand_noise, float cfg,
                                 float sigma, float A, float B, float d_scale, float coeff2,
                                 float u_scale, float coeff3, float noise_coeff, int64_t n);

/* transformer.cpp:182-197 -- flip_sin_to_cos sinusoid of one timestep, bf16 [dim]. */
void oracle_timestep_sinusoid(float t, int dim, uint16_t *out);

/* transformer.cpp:213-318 -- Cosmos 3-axis RoPE tables, bf16 [pe_t*pe_h*pe_w, HD]. */
void oracle_cosmos_rope_tables(int pe_t, int pe_h, int pe_w, int HD, uint16_t *cos_out,
                               uint16_t *sin_out);

/* qwen3.cpp:12-23 (theta 1e6) and llm_adapter.cpp:11-22 (theta 1e4) -- fp32 [T, HD/2]. */
void oracle_standard_rope_tables(int T, int HD, float theta, float *cos_out, float *sin_out);

#ifdef __cplusplus
}
#endif

#endif
