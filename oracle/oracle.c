/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY: CPU restatement of anima.cu's fused layer
 * kernels, used as the parity checker. Compiled with -ffp-contract=off so that every
 * fused multiply-add below is one the reference's CUDA source spells out (or that nvcc
 * is known to form there); see oracle.h for the contract and the mode parameters.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ bf16 helpers */

float oracle_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff; /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                      /* round to nearest even */
    return (uint16_t)(u >> 16);
}

#define B2F oracle_bf16_to_f32
#define F2B oracle_f32_to_bf16

/* ------------------------------------------------------- reference reductions */

/* warp_reduce_sum, src/cuda_utils.cuh:46-50: __shfl_down_sync with offsets 16..1;
 * the value that matters is lane 0's. */
static float ref_warp_sum(float v[32]) {
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) v[l] = v[l] + v[l + off];
    return v[0];
}

/* cta_reduce_sum, src/kernels/layer_norm.cu:7-19 (the same tree is inlined at
 * rms_norm.cu:40-53, adaln.cu:418-431, gemma_ops.cu:148-161). */
float oracle_ref_block_sum(const float *per_thread, int nthreads) {
    int nwarps = (nthreads + 31) / 32;
    float warp_sums[32];
    for (int w = 0; w < nwarps; ++w) {
        float v[32];
        for (int l = 0; l < 32; ++l) {
            int t = w * 32 + l;
            v[l] = t < nthreads ? per_thread[t] : 0.0f;
        }
        warp_sums[w] = ref_warp_sum(v);
    }
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = l < nwarps ? warp_sums[l] : 0.0f;
    return ref_warp_sum(v);
}

/* layer_norm.cu:68-70, :132-133, :205-206; rms_norm.cu:126-128; adaln.cu:453-454 */
int oracle_ref_row_threads(int D) {
    int D2 = D / 2;
    int threads = (D2 <= 1024) ? ((D2 + 31) / 32 * 32) : 1024;
    if (threads < 32) threads = 32;
    return threads;
}

/* var = sum_sq/D - mean*mean (layer_norm.cu:49,107,179); mode 0 = contracted to an fma. */
static float ref_var(float q_over_d, float mean, int var_mode) {
    return var_mode == 0 ? fmaf(-mean, mean, q_over_d) : q_over_d - mean * mean;
}

/* ------------------------------------------------------------------ LayerNorm */

/* layer_norm.cu:26-59 */
void oracle_layer_norm(const uint16_t *x, uint16_t *out, int N, int D, float eps,
                       int var_mode) {
    int D2 = D / 2, T = oracle_ref_row_threads(D);
    float *ps = calloc((size_t)T, sizeof(float)), *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        const uint16_t *xr = x + (int64_t)n * D;
        uint16_t *yr = out + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float s = 0.0f, q = 0.0f;
            for (int i = t; i < D2; i += T) {
                float v0 = B2F(xr[2 * i]), v1 = B2F(xr[2 * i + 1]);
                s += v0 + v1;
                q = fmaf(v0, v0, q);
                q = fmaf(v1, v1, q);
            }
            ps[t] = s;
            pq[t] = q;
        }
        float mean = oracle_ref_block_sum(ps, T) / (float)D;
        float var = ref_var(oracle_ref_block_sum(pq, T) / (float)D, mean, var_mode);
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < D2; ++i) {
            float v0 = (B2F(xr[2 * i]) - mean) * inv_std;
            float v1 = (B2F(xr[2 * i + 1]) - mean) * inv_std;
            yr[2 * i] = F2B(v0);
            yr[2 * i + 1] = F2B(v1);
        }
    }
    free(ps);
    free(pq);
}

/* layer_norm.cu:83-125 */
void oracle_adaln_layernorm(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                            uint16_t *out, int N, int D, float eps, int var_mode) {
    int D2 = D / 2, T = oracle_ref_row_threads(D);
    float *ps = calloc((size_t)T, sizeof(float)), *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        const uint16_t *xr = x + (int64_t)n * D;
        uint16_t *yr = out + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float s = 0.0f, q = 0.0f;
            for (int i = t; i < D2; i += T) {
                float v0 = B2F(xr[2 * i]), v1 = B2F(xr[2 * i + 1]);
                s += v0 + v1;
                q += v0 * v0 + v1 * v1; /* bf16 squares are exact: no contraction choice */
            }
            ps[t] = s;
            pq[t] = q;
        }
        float mean = oracle_ref_block_sum(ps, T) / (float)D;
        float var = ref_var(oracle_ref_block_sum(pq, T) / (float)D, mean, var_mode);
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int e = 0; e < 2 * D2; ++e) {
            float xv = B2F(xr[e]), sv = B2F(scale[e]), hv = B2F(shift[e]);
            yr[e] = F2B(fmaf((xv - mean) * inv_std, 1.0f + sv, hv));
        }
    }
    free(ps);
    free(pq);
}

static float sq_pair(float h0, float h1, int sq_mode) {
    switch (sq_mode) {
    case 0: return fmaf(h0, h0, h1 * h1);
    case 1: return fmaf(h1, h1, h0 * h0);
    default: return h0 * h0 + h1 * h1;
    }
}

/* layer_norm.cu:146-196 */
void oracle_residual_gate_adaln(uint16_t *hidden, const uint16_t *sub_out,
                                const uint16_t *gate, const uint16_t *scale,
                                const uint16_t *shift, uint16_t *normed, int N, int D,
                                float eps, int sq_mode, int var_mode) {
    int D2 = D / 2, T = oracle_ref_row_threads(D);
    float *ps = calloc((size_t)T, sizeof(float)), *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        uint16_t *hr = hidden + (int64_t)n * D;
        const uint16_t *yr = sub_out + (int64_t)n * D;
        uint16_t *nr = normed + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float s = 0.0f, q = 0.0f;
            for (int i = t; i < D2; i += T) {
                float h0 = fmaf(B2F(yr[2 * i]), B2F(gate[2 * i]), B2F(hr[2 * i]));
                float h1 = fmaf(B2F(yr[2 * i + 1]), B2F(gate[2 * i + 1]), B2F(hr[2 * i + 1]));
                hr[2 * i] = F2B(h0);
                hr[2 * i + 1] = F2B(h1);
                s += h0 + h1;
                q += sq_pair(h0, h1, sq_mode);
            }
            ps[t] = s;
            pq[t] = q;
        }
        float mean = oracle_ref_block_sum(ps, T) / (float)D;
        float var = ref_var(oracle_ref_block_sum(pq, T) / (float)D, mean, var_mode);
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int e = 0; e < 2 * D2; ++e) {
            float hv = B2F(hr[e]), sv = B2F(scale[e]), shv = B2F(shift[e]);
            nr[e] = F2B(fmaf((hv - mean) * inv_std, 1.0f + sv, shv));
        }
    }
    free(ps);
    free(pq);
}

/* -------------------------------------------------------------------- RMSNorm */

/* rms_norm.cu:9-67 */
void oracle_rms_norm(const uint16_t *x, const uint16_t *weight, uint16_t *out, int N, int D,
                     float eps) {
    int D2 = D / 2, T = oracle_ref_row_threads(D);
    float *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        const uint16_t *xr = x + (int64_t)n * D;
        uint16_t *yr = out + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float q = 0.0f;
            for (int i = t; i < D2; i += T) {
                float v0 = B2F(xr[2 * i]), v1 = B2F(xr[2 * i + 1]);
                q = fmaf(v0, v0, q);
                q = fmaf(v1, v1, q);
            }
            pq[t] = q;
        }
        float rms_inv = 1.0f / sqrtf(oracle_ref_block_sum(pq, T) / (float)D + eps);
        for (int e = 0; e < 2 * D2; ++e) {
            float v = B2F(xr[e]) * rms_inv;
            if (weight) v = v * B2F(weight[e]);
            yr[e] = F2B(v);
        }
    }
    free(pq);
}

/* adaln.cu:11-58 */
void oracle_adaln_rms_norm(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                           uint16_t *out, int N, int D, float eps) {
    int D2 = D / 2, T = oracle_ref_row_threads(D);
    float *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        const uint16_t *xr = x + (int64_t)n * D;
        const uint16_t *sr = scale + (int64_t)n * D, *hr = shift + (int64_t)n * D;
        uint16_t *yr = out + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float q = 0.0f;
            for (int i = t; i < D2; i += T) {
                float v0 = B2F(xr[2 * i]), v1 = B2F(xr[2 * i + 1]);
                q = fmaf(v0, v0, q);
                q = fmaf(v1, v1, q);
            }
            pq[t] = q;
        }
        float rms_inv = 1.0f / sqrtf(oracle_ref_block_sum(pq, T) / (float)D + eps);
        for (int e = 0; e < 2 * D2; ++e) {
            float v = B2F(xr[e]) * rms_inv;
            yr[e] = F2B(fmaf(v, 1.0f + B2F(sr[e]), B2F(hr[e])));
        }
    }
    free(pq);
}

/* gemma_ops.cu:132-177: scalar loop over D, block of min(roundup32(D), 1024) threads */
void oracle_gemma_rms_norm(const uint16_t *x, const uint16_t *weight, uint16_t *out, int N,
                           int D, float eps) {
    int T = (D <= 1024) ? ((D + 31) / 32 * 32) : 1024;
    if (T < 32) T = 32;
    float *pq = calloc((size_t)T, sizeof(float));
    for (int n = 0; n < N; ++n) {
        const uint16_t *xr = x + (int64_t)n * D;
        uint16_t *yr = out + (int64_t)n * D;
        for (int t = 0; t < T; ++t) {
            float q = 0.0f;
            for (int i = t; i < D; i += T) {
                float v = B2F(xr[i]);
                q += v * v;
            }
            pq[t] = q;
        }
        float rms_inv = 1.0f / sqrtf(oracle_ref_block_sum(pq, T) / (float)D + eps);
        for (int i = 0; i < D; ++i) {
            float v = B2F(xr[i]) * rms_inv;
            yr[i] = F2B(v * (1.0f + B2F(weight[i])));
        }
    }
    free(pq);
}

/* ---------------------------------------------------------------- activations */

static const float kSqrt2OverPi = 0.7978845608028654f; /* gelu.cu:8 */
static const float kGeluCoeff = 0.044715f;             /* gelu.cu:9 */

/* gelu.cu:22-31 */
static float gelu_tanh_f(float v) {
    float inner = kSqrt2OverPi * fmaf(kGeluCoeff * (v * v), v, v);
    float half_v = 0.5f * v;
    return fmaf(half_v, tanhf(inner), half_v);
}

/* gelu.cu:12-34 (bias NULL) and :37-64 */
void oracle_gelu_tanh(const uint16_t *x, const uint16_t *bias, uint16_t *out, int64_t N, int D) {
    int64_t N2 = N / 2;
    for (int64_t e = 0; e < 2 * N2; ++e) {
        float v = B2F(x[e]);
        if (bias) v = v + B2F(bias[e % D]);
        out[e] = F2B(gelu_tanh_f(v));
    }
}

/* silu.cu:7-24 (bias NULL) and :26-47 */
void oracle_silu(const uint16_t *x, const uint16_t *bias, uint16_t *out, int64_t N, int D) {
    int64_t N2 = N / 2;
    for (int64_t e = 0; e < 2 * N2; ++e) {
        float v = B2F(x[e]);
        if (bias) v = v + B2F(bias[e % D]);
        out[e] = F2B(v / (1.0f + expf(-v)));
    }
}

/* gemma_ops.cu:5-22: inner = c1*(g + c2*g*g*g), nvcc folds the add into an fma */
void oracle_gated_gelu(const uint16_t *gate, const uint16_t *up, uint16_t *out, int64_t N) {
    for (int64_t i = 0; i < N; ++i) {
        float g = B2F(gate[i]), u = B2F(up[i]);
        float inner = 0.7978845608f * fmaf(0.044715f * g * g, g, g);
        float gelu_g = 0.5f * g * (1.0f + tanhf(inner));
        out[i] = F2B(gelu_g * u);
    }
}

/* ---------------------------------------------------------------- elementwise */

/* elementwise.cu:37-53 */
void oracle_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t N) {
    for (int64_t i = 0; i < N / 2 * 2; ++i) out[i] = F2B(B2F(a[i]) + B2F(b[i]));
}

/* elementwise.cu:125-141 */
void oracle_mul(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t N) {
    for (int64_t i = 0; i < N / 2 * 2; ++i) out[i] = F2B(B2F(a[i]) * B2F(b[i]));
}

/* elementwise.cu:216-236 */
void oracle_scale_shift_bcast(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                              uint16_t *out, int M, int D) {
    int D2 = D / 2;
    for (int64_t m = 0; m < M; ++m)
        for (int d = 0; d < 2 * D2; ++d) {
            int64_t e = m * (2 * D2) + d;
            out[e] = F2B(fmaf(B2F(x[e]), 1.0f + B2F(scale[d]), B2F(shift[d])));
        }
}

/* elementwise.cu:184-213 */
void oracle_bias_add(const uint16_t *x, const uint16_t *bias, uint16_t *out, int M, int D) {
    int D2 = D / 2;
    for (int64_t m = 0; m < M; ++m)
        for (int d = 0; d < 2 * D2; ++d) {
            int64_t e = m * (2 * D2) + d;
            out[e] = F2B(B2F(x[e]) + B2F(bias[d]));
        }
}

/* elementwise.cu:249-269 */
void oracle_residual_gate_bcast(const uint16_t *x, const uint16_t *y, const uint16_t *gate,
                                uint16_t *out, int M, int D) {
    int D2 = D / 2;
    for (int64_t m = 0; m < M; ++m)
        for (int d = 0; d < 2 * D2; ++d) {
            int64_t e = m * (2 * D2) + d;
            out[e] = F2B(fmaf(B2F(y[e]), B2F(gate[d]), B2F(x[e])));
        }
}

/* ----------------------------------------------------------------------- RoPE */

/* rope.cu:72-108. bf16 x bf16 products are exact in fp32, so the rotation has a
 * single rounding whichever way nvcc contracts it. */
void oracle_rope_cosmos_strided(uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                                int B, int S, int H, int HD) {
    int half = HD / 2;
    for (int64_t row = 0; row < (int64_t)B * S; ++row) {
        int s = (int)(row % S);
        for (int h = 0; h < H; ++h) {
            uint16_t *base = x + row * H * HD + (int64_t)h * HD;
            for (int i = 0; i < half; ++i) {
                float xr = B2F(base[i]), xi = B2F(base[i + half]);
                float c = B2F(cos_t[(int64_t)s * HD + i]), sn = B2F(sin_t[(int64_t)s * HD + i]);
                base[i] = F2B(xr * c - xi * sn);
                base[i + half] = F2B(xi * c + xr * sn);
            }
        }
    }
}

static float rot2(float a, float b, float c, float d, int mode, float sign) {
    /* a*b + sign*(c*d), with the contraction choice `mode` */
    switch (mode) {
    case 0: return fmaf(a, b, sign * (c * d));
    case 1: return fmaf(sign * c, d, a * b);
    default: return a * b + sign * (c * d);
    }
}

/* gemma_ops.cu:62-87 */
void oracle_rope_standard(uint16_t *x, const float *cos_t, const float *sin_t,
                          int total_rows, int T, int D, int mode_a, int mode_b) {
    int half = D / 2;
    for (int64_t row = 0; row < total_rows; ++row) {
        int t = (int)(row % T);
        for (int d = 0; d < half; ++d) {
            float c = cos_t[(int64_t)t * half + d], s = sin_t[(int64_t)t * half + d];
            int64_t i1 = row * D + d, i2 = row * D + half + d;
            float x1 = B2F(x[i1]), x2 = B2F(x[i2]);
            float o1 = rot2(x1, c, x2, s, mode_a, -1.0f);
            float o2 = rot2(x2, c, x1, s, mode_b, 1.0f);
            x[i1] = F2B(o1);
            x[i2] = F2B(o2);
        }
    }
}

/* ------------------------------------------------------------------ gather */

/* gemma_ops.cu:34-45 */
void oracle_embedding_lookup(const uint16_t *table, const int32_t *ids, uint16_t *out, int T,
                             int D, int vocab) {
    for (int t = 0; t < T; ++t) {
        int id = ids[t];
        if (id < 0 || id >= vocab)
            memset(out + (int64_t)t * D, 0, (size_t)D * 2);
        else
            memcpy(out + (int64_t)t * D, table + (int64_t)id * D, (size_t)D * 2);
    }
}

/* ------------------------------------------------------------- VAE channel norm */

/* vae_kernels.cu:15-39, launched per batch item at :41-52 (nvcc contracts sum_sq += v*v) */
void oracle_pixel_norm(const uint16_t *x, uint16_t *out, int B, int C, int spatial, float eps) {
    for (int b = 0; b < B; ++b) {
        const uint16_t *xb = x + (int64_t)b * C * spatial;
        uint16_t *ob = out + (int64_t)b * C * spatial;
        for (int s = 0; s < spatial; ++s) {
            float q = 0.0f;
            for (int c = 0; c < C; ++c) {
                float v = B2F(xb[(int64_t)c * spatial + s]);
                q = fmaf(v, v, q);
            }
            float inv = 1.0f / sqrtf(q / (float)C + eps);
            for (int c = 0; c < C; ++c) {
                int64_t i = (int64_t)c * spatial + s;
                ob[i] = F2B(B2F(xb[i]) * inv);
            }
        }
    }
}

/* vae_kernels.cu:60-81, launched per batch item at :83-98 */
void oracle_rms_norm_channel(const uint16_t *x, const uint16_t *gamma, uint16_t *out, int B,
                             int C, int spatial, float eps) {
    for (int b = 0; b < B; ++b) {
        const uint16_t *xb = x + (int64_t)b * C * spatial;
        uint16_t *ob = out + (int64_t)b * C * spatial;
        for (int s = 0; s < spatial; ++s) {
            float q = 0.0f;
            for (int c = 0; c < C; ++c) {
                float v = B2F(xb[(int64_t)c * spatial + s]);
                q += v * v;
            }
            float rms = 1.0f / sqrtf(q / (float)C + eps);
            for (int c = 0; c < C; ++c) {
                int64_t i = (int64_t)c * spatial + s;
                ob[i] = F2B((B2F(xb[i]) * rms) * B2F(gamma[c]));
            }
        }
    }
}

/* ------------------------------------------------------------- host tables */

/* transformer.cpp:182-197 */
void oracle_timestep_sinusoid(float t, int dim, uint16_t *out) {
    int half = dim / 2;
    for (int i = 0; i < half; ++i) {
        float freq = expf(-logf(10000.0f) * (float)i / (float)half);
        float angle = t * freq;
        out[i] = F2B(cosf(angle));
        out[half + i] = F2B(sinf(angle));
    }
}

static void axis_freqs(int dim, float theta, float *freqs) {
    for (int i = 0; i < dim / 2; ++i) freqs[i] = 1.0f / powf(theta, (float)(2 * i) / (float)dim);
}

/* transformer.cpp:213-318 */
void oracle_cosmos_rope_tables(int pe_t, int pe_h, int pe_w, int HD, uint16_t *cos_out,
                               uint16_t *sin_out) {
    int dim_h = (HD / 6) * 2, dim_w = (HD / 6) * 2, dim_t = HD - dim_h - dim_w;
    float h_ntk = powf(4.0f, (float)dim_h / (float)(dim_h - 2));
    float w_ntk = powf(4.0f, (float)dim_w / (float)(dim_w - 2));
    float t_ntk = powf(1.0f, (float)dim_t / (float)(dim_t - 2));
    float *ft = malloc(sizeof(float) * (size_t)(dim_t / 2 + 1));
    float *fh = malloc(sizeof(float) * (size_t)(dim_h / 2 + 1));
    float *fw = malloc(sizeof(float) * (size_t)(dim_w / 2 + 1));
    axis_freqs(dim_t, 10000.0f * t_ntk, ft);
    axis_freqs(dim_h, 10000.0f * h_ntk, fh);
    axis_freqs(dim_w, 10000.0f * w_ntk, fw);
    float *crow = malloc(sizeof(float) * (size_t)HD), *srow = malloc(sizeof(float) * (size_t)HD);
    for (int a = 0; a < pe_t; ++a)
        for (int b = 0; b < pe_h; ++b)
            for (int c = 0; c < pe_w; ++c) {
                int idx = (a * pe_h + b) * pe_w + c, off = 0;
                for (int d = 0; d < dim_t / 2; ++d, ++off) {
                    float ang = (float)a * ft[d];
                    crow[off] = cosf(ang);
                    srow[off] = sinf(ang);
                }
                for (int d = 0; d < dim_h / 2; ++d, ++off) {
                    float ang = (float)b * fh[d];
                    crow[off] = cosf(ang);
                    srow[off] = sinf(ang);
                }
                for (int d = 0; d < dim_w / 2; ++d, ++off) {
                    float ang = (float)c * fw[d];
                    crow[off] = cosf(ang);
                    srow[off] = sinf(ang);
                }
                for (int d = 0; d < off; ++d) {
                    crow[off + d] = crow[d];
                    srow[off + d] = srow[d];
                }
                for (int d = 0; d < HD; ++d) {
                    cos_out[(int64_t)idx * HD + d] = F2B(crow[d]);
                    sin_out[(int64_t)idx * HD + d] = F2B(srow[d]);
                }
            }
    free(ft);
    free(fh);
    free(fw);
    free(crow);
    free(srow);
}

/* qwen3.cpp:12-23, llm_adapter.cpp:11-22 */
void oracle_standard_rope_tables(int T, int HD, float theta, float *cos_out, float *sin_out) {
    int half = HD / 2;
    for (int t = 0; t < T; ++t)
        for (int d = 0; d < half; ++d) {
            float freq = 1.0f / powf(theta, (float)(2 * d) / (float)HD);
            float angle = (float)t * freq;
            cos_out[t * half + d] = cosf(angle);
            sin_out[t * half + d] = sinf(angle);
        }
}

/* ---------------------------------------------------- latent I/O and sampler steps */

/* ------------------------------------------------------------ attention glue */

/* transpose.cu:17-31, 45-59, 71-89, 100-118 */
void oracle_head_permute(const uint16_t *src, uint16_t *dst, int B, int H, int S, int HD, int to_heads) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t t = 0; t < S; ++t)
                for (int64_t d = 0; d < HD; ++d) {
                    int64_t heads = ((b * H + h) * S + t) * HD + d; /* [B, H, S, HD] */
                    int64_t rows = ((b * S + t) * H + h) * HD + d;  /* [B*S, H*HD] */
                    if (to_heads)
                        dst[heads] = src[rows];
                    else
                        dst[rows] = src[heads];
                }
}

/* gemma_ops.cu:101-117 */
void oracle_expand_kv(const uint16_t *kv, uint16_t *out, int B, int KVH, int QH, int T, int D) {
    int ratio = QH / KVH;
    int64_t P = (int64_t)T * D;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t q = 0; q < QH; ++q)
            memcpy(out + (b * QH + q) * P, kv + (b * KVH + q / ratio) * P, (size_t)P * 2);
}

/* softmax.cu:64-73 */
void oracle_causal_mask(uint16_t *scores, int H, int T) {
    uint16_t m = F2B(-1e9f);
    for (int64_t h = 0; h < H; ++h)
        for (int64_t i = 0; i < T; ++i)
            for (int64_t j = i + 1; j < T; ++j) scores[(h * T + i) * T + j] = m;
}

/* cuda_utils.cuh:46-50: a warp's __shfl_down_sync sum tree; the value lane 0 ends with. */
static float shfl_down_sum32(const float *in) {
    float v[32];
    memcpy(v, in, sizeof v);
    for (int o = 16; o > 0; o >>= 1)
        for (int i = 0; i < o; ++i) v[i] = v[i] + v[i + o];
    return v[0];
}

static int softmax_threads(int D) { /* softmax.cu:118-119, :248-249 */
    int t = D <= 1024 ? (D + 31) / 32 * 32 : 1024;
    return t < 32 ? 32 : t;
}

/* softmax.cu:8-60 */
void oracle_softmax(const uint16_t *x, uint16_t *out, int N, int D) {
    int nt = softmax_threads(D), nw = nt / 32;
    float *part = (float *)calloc((size_t)nt, sizeof(float));
    for (int64_t r = 0; r < N; ++r) {
        const uint16_t *xr = x + r * D;
        float mx = -1e30f;
        for (int i = 0; i < D; ++i) mx = fmaxf(mx, B2F(xr[i]));
        for (int t = 0; t < nt; ++t) {
            float acc = 0.0f;
            for (int i = t; i < D; i += nt) acc += expf(B2F(xr[i]) - mx);
            part[t] = acc;
        }
        float warps[32] = {0};
        for (int w = 0; w < nw; ++w) warps[w] = shfl_down_sum32(part + 32 * w);
        float inv = 1.0f / shfl_down_sum32(warps);
        for (int i = 0; i < D; ++i) out[r * D + i] = F2B(expf(B2F(xr[i]) - mx) * inv);
    }
    free(part);
}

/* softmax.cu:160-166 and :185-193 (nvcc contracts a*b + c into one fma there) */
static void online_add(float xi, float *m, float *s) {
    if (xi > *m) {
        *s = fmaf(*s, expf(*m - xi), 1.0f);
        *m = xi;
    } else {
        *s += expf(xi - *m);
    }
}
static void online_merge(float om, float os, float *m, float *s) {
    if (om > *m) {
        *s = fmaf(*s, expf(*m - om), os);
        *m = om;
    } else {
        *s = fmaf(os, expf(om - *m), *s);
    }
}

/* A warp's __shfl_down_sync merge tree over (m, s); lanes whose source is out of range merge
 * with themselves, as the shuffle returns their own value. Result: lane 0. */
static void shfl_down_merge32(float *m, float *s) {
    for (int o = 16; o > 0; o >>= 1) {
        float nm[32], ns[32];
        for (int i = 0; i < 32; ++i) {
            int src = i + o < 32 ? i + o : i;
            nm[i] = m[i];
            ns[i] = s[i];
            online_merge(m[src], s[src], &nm[i], &ns[i]);
        }
        memcpy(m, nm, sizeof nm);
        memcpy(s, ns, sizeof ns);
    }
}

/* softmax.cu:153-245 */
void oracle_softmax_f32_to_bf16(const float *x, uint16_t *out, int N, int D) {
    int nt = softmax_threads(D), nw = nt / 32, D4 = D / 4;
    float *tm = (float *)malloc((size_t)nt * sizeof(float)), *ts = (float *)malloc((size_t)nt * sizeof(float));
    for (int64_t r = 0; r < N; ++r) {
        const float *xr = x + r * D;
        for (int t = 0; t < nt; ++t) {
            float m = -1e30f, s = 0.0f;
            for (int i = t; i < D4; i += nt)
                for (int k = 0; k < 4; ++k) online_add(xr[4 * i + k], &m, &s);
            for (int i = D4 * 4 + t; i < D; i += nt) online_add(xr[i], &m, &s);
            tm[t] = m;
            ts[t] = s;
        }
        float wm[32], ws[32];
        for (int w = 0; w < 32; ++w) {
            wm[w] = -1e30f;
            ws[w] = 0.0f;
        }
        for (int w = 0; w < nw; ++w) {
            float m[32], s[32];
            memcpy(m, tm + 32 * w, sizeof m);
            memcpy(s, ts + 32 * w, sizeof s);
            shfl_down_merge32(m, s);
            wm[w] = m[0];
            ws[w] = s[0];
        }
        shfl_down_merge32(wm, ws);
        float mx = wm[0], inv = 1.0f / ws[0];
        for (int i = 0; i < D; ++i) out[r * D + i] = F2B(expf(xr[i] - mx) * inv);
    }
    free(tm);
    free(ts);
}

/* causal_conv3d.cu:187-195, then elementwise.cu:37-53 when residual is given */
void oracle_conv_bias_add(const uint16_t *x, const uint16_t *bias, const uint16_t *residual,
                          uint16_t *out, int B, int C, int spatial) {
    for (int64_t b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c)
            for (int64_t s = 0; s < spatial; ++s) {
                int64_t e = (b * C + c) * spatial + s;
                uint16_t h = F2B(B2F(x[e]) + B2F(bias[c]));
                out[e] = residual ? F2B(B2F(h) + B2F(residual[e])) : h;
            }
}

/* vae_kernels.cu:174-206 */
void oracle_channel_scale_shift(const uint16_t *x, const uint16_t *scale, const uint16_t *shift,
                                uint16_t *out, int B, int C, int spatial) {
    for (int64_t b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c)
            for (int64_t s = 0; s < spatial; ++s) {
                int64_t e = (b * C + c) * spatial + s;
                out[e] = F2B(fmaf(B2F(x[e]), B2F(scale[c]), B2F(shift[c])));
            }
}

/* transpose.cu:132-185 */
void oracle_patchify_3d(const uint16_t *src, uint16_t *dst, int B, int C, int T, int H, int W,
                        int pT, int pH, int pW) {
    int pe_t = T / pT, pe_h = H / pH, pe_w = W / pW;
    int64_t S = (int64_t)pe_t * pe_h * pe_w, pd = (int64_t)C * pT * pH * pW, vol = (int64_t)C * T * H * W;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t tok = 0; tok < S; ++tok) {
            int64_t fw = tok % pe_w, fh = (tok / pe_w) % pe_h, ft = tok / ((int64_t)pe_w * pe_h);
            for (int c = 0; c < C; ++c)
                for (int pt = 0; pt < pT; ++pt)
                    for (int ph = 0; ph < pH; ++ph)
                        for (int pw = 0; pw < pW; ++pw) {
                            int64_t d = ((int64_t)(c * pT + pt) * pH + ph) * pW + pw;
                            int64_t t = ft * pT + pt, h = fh * pH + ph, w = fw * pW + pw;
                            dst[(b * S + tok) * pd + d] = src[b * vol + (((int64_t)c * T + t) * H + h) * W + w];
                        }
        }
}

/* transpose.cu:191-243 */
void oracle_unpatchify_3d(const uint16_t *src, uint16_t *dst, int B, int C, int T, int H, int W,
                          int pT, int pH, int pW) {
    int pe_t = T / pT, pe_h = H / pH, pe_w = W / pW;
    int64_t S = (int64_t)pe_t * pe_h * pe_w, pd = (int64_t)C * pT * pH * pW, vol = (int64_t)C * T * H * W;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t tok = 0; tok < S; ++tok) {
            int64_t fw = tok % pe_w, fh = (tok / pe_w) % pe_h, ft = tok / ((int64_t)pe_w * pe_h);
            for (int64_t d = 0; d < pd; ++d) {
                int64_t r = d;
                int c = (int)(r % C);
                r /= C;
                int pt = (int)(r % pT);
                r /= pT;
                int pw = (int)(r % pW);
                int ph = (int)(r / pW);
                int64_t t = ft * pT + pt, h = fh * pH + ph, w = fw * pW + pw;
                dst[b * vol + (((int64_t)c * T + t) * H + h) * W + w] = src[(b * S + tok) * pd + d];
            }
        }
}

/* transpose.cu:250-276 */
void oracle_cfg_euler_step(const uint16_t *sample, const uint16_t *pos, const uint16_t *neg,
                           uint16_t *out, float cfg, float sigma, float sigma_next, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float s = B2F(sample[i]), np = B2F(pos[i]), nn = B2F(neg[i]);
        float noise = fmaf(cfg, np - nn, nn), r;
        if (sigma_next == 0.0f) {
            r = fmaf(-sigma, noise, s);
        } else {
            float den = fmaf(-sigma, noise, s);
            float d = (s - den) / sigma;
            r = fmaf(d, sigma_next - sigma, s);
        }
        out[i] = F2B(r);
    }
}

/* transpose.cu:306-364 */
void oracle_cfg_euler_a_rf_step(const uint16_t *sample, const uint16_t *pos, const uint16_t *neg,
                                const uint16_t *rand_noise, uint16_t *out, float cfg, float sigma,
                                float sigma_next, float eta, float s_noise, int64_t n) {
    float downstep_ratio = 1.0f + (sigma_next / sigma - 1.0f) * eta;
    float sigma_down = sigma_next * downstep_ratio;
    float alpha_ip1 = 1.0f - sigma_next;
    float alpha_down = 1.0f - sigma_down;
    float renoise_sq = sigma_next * sigma_next -
                       sigma_down * sigma_down * alpha_ip1 * alpha_ip1 / (alpha_down * alpha_down);
    float renoise_coeff = (renoise_sq > 0.0f) ? sqrtf(renoise_sq) : 0.0f;
    float sdr = sigma_down / sigma, alpha_ratio = alpha_ip1 / alpha_down;
    for (int64_t i = 0; i < n; ++i) {
        float s = B2F(sample[i]), np = B2F(pos[i]), nn = B2F(neg[i]);
        float noise_pred = fmaf(cfg, np - nn, nn);
        float den = fmaf(-sigma, noise_pred, s);
        float r = fmaf(sdr, s, (1.0f - sdr) * den);
        if (eta > 0.0f && renoise_coeff > 0.0f)
            r = fmaf(alpha_ratio, r, B2F(rand_noise[i]) * s_noise * renoise_coeff);
        out[i] = F2B(r);
    }
}

/* transpose.cu:386-465 */
void oracle_cfg_er_sde_full_step(uint16_t *x, const uint16_t *pos, const uint16_t *neg,
                                 uint16_t *den_out, const uint16_t *old_den, uint16_t *dd_out,
                                 const uint16_t *old_dd, const uint16_t *rand_noise, float cfg,
                                 float sigma, float A, float B, float d_scale, float coeff2,
                                 float u_scale, float coeff3, float noise_coeff, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float s = B2F(x[i]), np = B2F(pos[i]), nn = B2F(neg[i]);
        float vel = fmaf(cfg, np - nn, nn);
        float den = fmaf(-sigma, vel, s);
        float r = fmaf(A, s, B * den), dd = 0.0f;
        if (old_den) {
            dd = (den - B2F(old_den[i])) * d_scale;
            r = fmaf(coeff2, dd, r);
            if (old_dd) r = fmaf(coeff3, (dd - B2F(old_dd[i])) * u_scale, r);
        }
        if (noise_coeff > 0.0f && rand_noise) r = fmaf(noise_coeff, B2F(rand_noise[i]), r);
        x[i] = F2B(r);
        den_out[i] = F2B(den);
        if (dd_out && old_den) dd_out[i] = F2B(dd);
    }
}
