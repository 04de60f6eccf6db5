/*
 * hostloop.c -- TEST INFRASTRUCTURE ONLY: the CPU baseline row of the benchmark.
 *
 * A plain host loop of the DiT block chain's ops (fp32 arithmetic on bf16 storage), the
 * way a C++ programmer would write anima.cu's kernels for the CPU: one pass per row with
 * sequential sums, OpenMP over rows (or over elements for the elementwise ops). It is
 * built -O3 -march=native -fopenmp on the machine that runs it (hostloop.py) and timed by
 * bench.py's cpu_baseline leg. It is not a parity checker: its sums run in row order, not
 * in the reference kernels' tree order, so results may differ from the reference by a few
 * bf16 ulp (tests/test_cpu_hostloop.py bounds that against oracle.c).
 *
 * The formulas are the reference kernels' (src/kernels/layer_norm.cu:83-125,146-196,
 * rms_norm.cu:9-67, rope.cu:72-108, gelu.cu:12-34, elementwise.cu:37-53,249-269).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float b2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f2b(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void hostloop_set_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n > 0 ? n : 1);
#else
    (void)n;
#endif
}

int hostloop_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* out = a + b (elementwise.cu:37-53) */
void hostloop_add(const uint16_t *a, const uint16_t *b, uint16_t *out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = f2b(b2f(a[i]) + b2f(b[i]));
}

/* out = LN(x) * (1 + scale) + shift (layer_norm.cu:83-125) */
void hostloop_adaln_layernorm(const uint16_t *x, const uint16_t *scale, const uint16_t *shift, uint16_t *out,
                              int64_t N, int D, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint16_t *xr = x + n * D;
        uint16_t *yr = out + n * D;
        float s = 0.0f, q = 0.0f;
        for (int d = 0; d < D; ++d) {
            const float v = b2f(xr[d]);
            s += v;
            q += v * v;
        }
        const float mean = s / (float)D;
        const float inv = 1.0f / sqrtf(q / (float)D - mean * mean + eps);
        for (int d = 0; d < D; ++d)
            yr[d] = f2b(((b2f(xr[d]) - mean) * inv) * (1.0f + b2f(scale[d])) + b2f(shift[d]));
    }
}

/* hidden += y * gate; normed = LN(hidden) * (1 + scale) + shift (layer_norm.cu:146-196) */
void hostloop_residual_gate_adaln(uint16_t *hidden, const uint16_t *y, const uint16_t *gate, const uint16_t *scale,
                                  const uint16_t *shift, uint16_t *normed, int64_t N, int D, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        uint16_t *hr = hidden + n * D;
        const uint16_t *yr = y + n * D;
        uint16_t *nr = normed + n * D;
        float s = 0.0f, q = 0.0f;
        for (int d = 0; d < D; ++d) {
            const float h = b2f(hr[d]) + b2f(yr[d]) * b2f(gate[d]);
            hr[d] = f2b(h);
            s += h;
            q += h * h;
        }
        const float mean = s / (float)D;
        const float inv = 1.0f / sqrtf(q / (float)D - mean * mean + eps);
        for (int d = 0; d < D; ++d)
            nr[d] = f2b(((b2f(hr[d]) - mean) * inv) * (1.0f + b2f(scale[d])) + b2f(shift[d]));
    }
}

/* out = x * rsqrt(mean(x^2) + eps) * w (rms_norm.cu:9-67), rows of D */
void hostloop_rms_norm(const uint16_t *x, const uint16_t *w, uint16_t *out, int64_t N, int D, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint16_t *xr = x + n * D;
        uint16_t *yr = out + n * D;
        float q = 0.0f;
        for (int d = 0; d < D; ++d) {
            const float v = b2f(xr[d]);
            q += v * v;
        }
        const float r = 1.0f / sqrtf(q / (float)D + eps);
        for (int d = 0; d < D; ++d) yr[d] = f2b(b2f(xr[d]) * r * (w ? b2f(w[d]) : 1.0f));
    }
}

/* Cosmos 3-axis RoPE in place on x[B*S, H*HD], bf16 tables [S, HD] (rope.cu:72-108) */
void hostloop_rope_cosmos(uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t, int B, int S, int H, int HD) {
    const int half = HD / 2;
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)B * S; ++row) {
        const int64_t s = row % S;
        for (int h = 0; h < H; ++h) {
            uint16_t *xp = x + (row * H + h) * HD;
            for (int i = 0; i < half; ++i) {
                const float c = b2f(cos_t[s * HD + i]), sn = b2f(sin_t[s * HD + i]);
                const float a = b2f(xp[i]), b = b2f(xp[i + half]);
                xp[i] = f2b(a * c - b * sn);
                xp[i + half] = f2b(b * c + a * sn);
            }
        }
    }
}

/* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) (gelu.cu:12-34) */
void hostloop_gelu_tanh(const uint16_t *x, uint16_t *out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float v = b2f(x[i]);
        out[i] = f2b(0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v))));
    }
}

/* out = x + y * gate[d] (elementwise.cu:249-269) */
void hostloop_residual_gate_bcast(const uint16_t *x, const uint16_t *y, const uint16_t *gate, uint16_t *out,
                                  int64_t M, int D) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int d = 0; d < D; ++d) out[m * D + d] = f2b(b2f(x[m * D + d]) + b2f(y[m * D + d]) * b2f(gate[d]));
}
