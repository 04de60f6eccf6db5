"""TEST INFRASTRUCTURE ONLY: numpy bindings of liboracle.so (oracle.c), the CPU
restatement of anima.cu's fused layer kernels, plus bf16 helpers and the ulp comparator
the parity tests use. Nothing in the product imports this module.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

P, I32, I64, F32 = c_void_p, c_int, c_int64, c_float

_SIGS = {
    "oracle_layer_norm": (P, P, I32, I32, F32, I32),
    "oracle_adaln_layernorm": (P, P, P, P, I32, I32, F32, I32),
    "oracle_residual_gate_adaln": (P, P, P, P, P, P, I32, I32, F32, I32, I32),
    "oracle_rms_norm": (P, P, P, I32, I32, F32),
    "oracle_adaln_rms_norm": (P, P, P, P, I32, I32, F32),
    "oracle_gemma_rms_norm": (P, P, P, I32, I32, F32),
    "oracle_gelu_tanh": (P, P, P, I64, I32),
    "oracle_silu": (P, P, P, I64, I32),
    "oracle_gated_gelu": (P, P, P, I64),
    "oracle_add": (P, P, P, I64),
    "oracle_mul": (P, P, P, I64),
    "oracle_bias_add": (P, P, P, I32, I32),
    "oracle_channel_scale_shift": (P, P, P, P, I32, I32, I32),
    "oracle_conv_bias_add": (P, P, P, P, I32, I32, I32),
    "oracle_head_permute": (P, P, I32, I32, I32, I32, I32),
    "oracle_expand_kv": (P, P, I32, I32, I32, I32, I32),
    "oracle_causal_mask": (P, I32, I32),
    "oracle_softmax": (P, P, I32, I32),
    "oracle_softmax_f32_to_bf16": (P, P, I32, I32),
    "oracle_patchify_3d": (P, P) + (I32,) * 8,
    "oracle_unpatchify_3d": (P, P) + (I32,) * 8,
    "oracle_cfg_euler_step": (P, P, P, P, F32, F32, F32, I64),
    "oracle_cfg_euler_a_rf_step": (P, P, P, P, P) + (F32,) * 5 + (I64,),
    "oracle_cfg_er_sde_full_step": (P,) * 8 + (F32,) * 9 + (I64,),
    "oracle_scale_shift_bcast": (P, P, P, P, I32, I32),
    "oracle_residual_gate_bcast": (P, P, P, P, I32, I32),
    "oracle_rope_cosmos_strided": (P, P, P, I32, I32, I32, I32),
    "oracle_rope_standard": (P, P, P, I32, I32, I32, I32, I32),
    "oracle_embedding_lookup": (P, P, P, I32, I32, I32),
    "oracle_rms_norm_channel": (P, P, P, I32, I32, I32, F32),
    "oracle_pixel_norm": (P, P, I32, I32, I32, F32),
    "oracle_timestep_sinusoid": (F32, I32, P),
    "oracle_cosmos_rope_tables": (I32, I32, I32, I32, P, P),
    "oracle_standard_rope_tables": (I32, I32, F32, P, P),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE} oracle`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = None
    return lib


lib = _load()

# Contraction choices of the reference build, pinned against the reference kernels'
# own outputs (tests/golden): see oracle.h for what each mode means.
VAR_MODE = 0          # var = fma(-mean, mean, sum_sq/D)
RESID_SQ_MODE = 0     # sum_sq += fma(h0, h0, h1*h1)
ROPE_STD_MODES = (0, 1)  # fma(x1, c, -(x2*s)), fma(x1, s, x2*c)


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16); NaN -> 0x7fff."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def randn_bf16(rng: np.random.Generator, shape, mean=0.0, std=1.0) -> np.ndarray:
    return f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean))


def ulp_ordinal(b) -> np.ndarray:
    """Monotonic integer image of bf16 bit patterns (+0 and -0 both map to 0)."""
    b = np.asarray(b, dtype=np.uint16).astype(np.int32)
    mag = b & 0x7FFF
    return np.where(b & 0x8000, -mag, mag)


def ulp_distance(a, b) -> np.ndarray:
    """Number of bf16 representable steps between two bf16 arrays."""
    return np.abs(ulp_ordinal(a) - ulp_ordinal(b))


def bf16_ulp(x) -> np.ndarray:
    """Spacing of bf16 values at |x| (fp32 input)."""
    ax = np.abs(np.asarray(x, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(ax, np.float32(2.0**-126)))).astype(np.int32)
    return np.ldexp(np.float32(1.0), e - 7).astype(np.float32)


def within_one_ulp(got, want, floor=2.0**-12):
    """True where |got - want| <= one bf16 ulp of max(|want|, floor).

    The floor covers outputs that are small only because of cancellation in an fp32
    expression such as x*(1+scale)+shift: for those the absolute error of any fp32
    evaluation order is set by the operands' magnitude, not by the result's.
    """
    g, w = bf16_to_f32(got), bf16_to_f32(want)
    ref = np.maximum(np.abs(w), np.float32(floor))
    both_nan = np.isnan(g) & np.isnan(w)
    return (np.abs(g - w) <= bf16_ulp(ref)) | both_nan


def _p(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


# ------------------------------------------------------------------ oracle calls
def layer_norm(x, N, D, eps=1e-6):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_layer_norm(_p(x), _p(out), N, D, eps, VAR_MODE)
    return out


def adaln_layernorm(x, scale, shift, N, D, eps=1e-6):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_adaln_layernorm(_p(x), _p(scale), _p(shift), _p(out), N, D, eps, VAR_MODE)
    return out


def residual_gate_adaln(hidden, sub_out, gate, scale, shift, N, D, eps=1e-6, sq_mode=None, var_mode=None):
    h = np.array(hidden, dtype=np.uint16, copy=True)
    normed = np.zeros((N, D), np.uint16)
    lib.oracle_residual_gate_adaln(_p(h), _p(sub_out), _p(gate), _p(scale), _p(shift), _p(normed), N, D,
                                   eps, RESID_SQ_MODE if sq_mode is None else sq_mode,
                                   VAR_MODE if var_mode is None else var_mode)
    return h, normed


def rms_norm(x, weight, N, D, eps=1e-6):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_rms_norm(_p(x), _p(weight), _p(out), N, D, eps)
    return out


def adaln_rms_norm(x, scale, shift, N, D, eps=1e-6):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_adaln_rms_norm(_p(x), _p(scale), _p(shift), _p(out), N, D, eps)
    return out


def gemma_rms_norm(x, weight, N, D, eps=1e-6):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_gemma_rms_norm(_p(x), _p(weight), _p(out), N, D, eps)
    return out


def gelu_tanh(x, bias=None, D=0):
    out = np.array(x, dtype=np.uint16, copy=True)  # an odd last element stays untouched
    lib.oracle_gelu_tanh(_p(x), _p(bias), _p(out), x.size, D)
    return out


def silu(x, bias=None, D=0):
    out = np.array(x, dtype=np.uint16, copy=True)
    lib.oracle_silu(_p(x), _p(bias), _p(out), x.size, D)
    return out


def gated_gelu(gate, up):
    out = np.zeros_like(gate)
    lib.oracle_gated_gelu(_p(gate), _p(up), _p(out), gate.size)
    return out


def add(a, b):
    out = np.array(a, dtype=np.uint16, copy=True)
    lib.oracle_add(_p(a), _p(b), _p(out), a.size)
    return out


def mul(a, b):
    out = np.array(a, dtype=np.uint16, copy=True)
    lib.oracle_mul(_p(a), _p(b), _p(out), a.size)
    return out


def swiglu(gate, up):
    return mul(silu(gate), up)


def bias_add(x, bias, M, D):
    out = np.zeros_like(x)
    lib.oracle_bias_add(_p(x), _p(bias), _p(out), M, D)
    return out


def scale_shift_bcast(x, scale, shift, M, D):
    out = np.zeros((M, D), np.uint16)
    lib.oracle_scale_shift_bcast(_p(x), _p(scale), _p(shift), _p(out), M, D)
    return out


def residual_gate_bcast(x, y, gate, M, D):
    out = np.zeros((M, D), np.uint16)
    lib.oracle_residual_gate_bcast(_p(x), _p(y), _p(gate), _p(out), M, D)
    return out


def rope_cosmos_strided(x, cos_t, sin_t, B, S, H, HD):
    out = np.array(x, dtype=np.uint16, copy=True)
    lib.oracle_rope_cosmos_strided(_p(out), _p(cos_t), _p(sin_t), B, S, H, HD)
    return out


def rope_standard(x, cos_t, sin_t, total_rows, T, D, modes=None):
    out = np.array(x, dtype=np.uint16, copy=True)
    ma, mb = ROPE_STD_MODES if modes is None else modes
    lib.oracle_rope_standard(_p(out), _p(cos_t), _p(sin_t), total_rows, T, D, ma, mb)
    return out


def embedding_lookup(table, ids, T, D, vocab):
    out = np.zeros((T, D), np.uint16)
    lib.oracle_embedding_lookup(_p(table), _p(ids), _p(out), T, D, vocab)
    return out


def rms_norm_channel(x, gamma, B, C, spatial, eps=1e-6):
    out = np.zeros((B, C, spatial), np.uint16)
    lib.oracle_rms_norm_channel(_p(x), _p(gamma), _p(out), B, C, spatial, eps)
    return out


def nearest_upsample_2x(x, B, C, H, W):
    """vae_kernels.cu:98-133: out[b, c, h2, w2] = x[b, c, h2 // 2, w2 // 2]."""
    x = np.asarray(x, np.uint16).reshape(B, C, H, W)
    return np.repeat(np.repeat(x, 2, axis=2), 2, axis=3)


def pixel_norm(x, B, C, spatial, eps=1e-6):
    out = np.zeros((B, C, spatial), np.uint16)
    lib.oracle_pixel_norm(_p(np.ascontiguousarray(x)), _p(out), B, C, spatial, eps)
    return out


def rms_norm_channel_silu(x, gamma, B, C, spatial, eps=1e-6):
    return silu(rms_norm_channel(x, gamma, B, C, spatial, eps).reshape(-1)).reshape(B, C, spatial)


def qk_norm_rope(x, weight, cos_t, sin_t, B, S, H, HD, eps=1e-6):
    normed = rms_norm(x, weight, B * S * H, HD, eps)
    return rope_cosmos_strided(normed, cos_t, sin_t, B, S, H, HD)


def layer_norm_modulate(x, scale, shift, N, D, eps=1e-6):
    return scale_shift_bcast(layer_norm(x, N, D, eps), scale, shift, N, D)


def adaln_layernorm_temb(x, mod, temb, N, D, eps=1e-6):
    """transformer.cpp:404-425: mod += temb, adaLN with shift = mod[:D], scale = mod[D:2D];
    returns (normed, gate = mod[2D:3D])."""
    m = add(mod, temb)
    return adaln_layernorm(x, m[D:2 * D], m[:D], N, D, eps), m[2 * D:]


def residual_gate_adaln_temb(hidden, sub_out, gate_in, mod, temb, N, D, eps=1e-6):
    """transformer.cpp:433-456: mod += temb, residual gate with the previous gate, adaLN with
    this set's shift/scale; returns (hidden, normed, gate = mod[2D:3D])."""
    m = add(mod, temb)
    h, n = residual_gate_adaln(hidden, sub_out, gate_in, m[D:2 * D], m[:D], N, D, eps)
    return h, n, m[2 * D:]


def head_transpose(src, B, H, S, HD):
    """transpose.cu:13-123: [B*S, H*HD] -> [B, H, S, HD]."""
    out = np.zeros((B, H, S, HD), np.uint16)
    lib.oracle_head_permute(_p(np.ascontiguousarray(src)), _p(out), B, H, S, HD, 1)
    return out


def head_untranspose(src, B, H, S, HD):
    """transpose.cu:41-123: [B, H, S, HD] -> [B*S, H*HD]."""
    out = np.zeros((B * S, H * HD), np.uint16)
    lib.oracle_head_permute(_p(np.ascontiguousarray(src)), _p(out), B, H, S, HD, 0)
    return out


def expand_kv(kv, B, KVH, QH, T, D):
    out = np.zeros((B, QH, T, D), np.uint16)
    lib.oracle_expand_kv(_p(np.ascontiguousarray(kv)), _p(out), B, KVH, QH, T, D)
    return out


def causal_mask(scores, H, T):
    out = np.array(scores, np.uint16).reshape(H, T, T)
    lib.oracle_causal_mask(_p(out), H, T)
    return out


def softmax(x, N, D):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_softmax(_p(np.ascontiguousarray(x)), _p(out), N, D)
    return out


def softmax_f32_to_bf16(x, N, D):
    out = np.zeros((N, D), np.uint16)
    lib.oracle_softmax_f32_to_bf16(_p(np.ascontiguousarray(x, np.float32)), _p(out), N, D)
    return out


def conv_bias_add(x, bias, B, C, spatial, residual=None):
    """causal_conv3d.cu:187-195 (+ add_bf16 of the residual, vae.cpp:194)."""
    out = np.zeros_like(x)
    res = None if residual is None else _p(np.ascontiguousarray(residual))
    lib.oracle_conv_bias_add(_p(x), _p(bias), res, _p(out), B, C, spatial)
    return out


def conv_bias_rms_norm_channel_silu(x, bias, gamma, B, C, spatial, eps=1e-6):
    """vae.cpp:185-189: the conv's bias launch, then rms_norm_channel_bf16 and silu_bf16."""
    h = conv_bias_add(x, bias, B, C, spatial)
    return rms_norm_channel_silu(h, gamma, B, C, spatial, eps)


def channel_scale_shift(x, scale, shift, B, C, spatial):
    out = np.zeros_like(x)
    lib.oracle_channel_scale_shift(_p(x), _p(scale), _p(shift), _p(out), B, C, spatial)
    return out


def patchify_3d(src, B, C, T, H, W, pT, pH, pW):
    S = (T // pT) * (H // pH) * (W // pW)
    out = np.zeros((B, S, C * pT * pH * pW), np.uint16)
    lib.oracle_patchify_3d(_p(np.ascontiguousarray(src)), _p(out), B, C, T, H, W, pT, pH, pW)
    return out


def unpatchify_3d(src, B, C, T, H, W, pT, pH, pW, init=None):
    out = np.zeros((B, C, T, H, W), np.uint16) if init is None else np.array(init, np.uint16).reshape(B, C, T, H, W)
    lib.oracle_unpatchify_3d(_p(np.ascontiguousarray(src)), _p(out), B, C, T, H, W, pT, pH, pW)
    return out


def cfg_euler_step(sample, pos, neg, cfg, sigma, sigma_next):
    out = np.zeros_like(sample)
    lib.oracle_cfg_euler_step(_p(sample), _p(pos), _p(neg), _p(out), cfg, sigma, sigma_next, sample.size)
    return out


def cfg_euler_a_rf_step(sample, pos, neg, rand_noise, cfg, sigma, sigma_next, eta, s_noise):
    out = np.zeros_like(sample)
    lib.oracle_cfg_euler_a_rf_step(_p(sample), _p(pos), _p(neg), None if rand_noise is None else _p(rand_noise),
                                   _p(out), cfg, sigma, sigma_next, eta, s_noise, sample.size)
    return out


def cfg_er_sde_full_step(x, pos, neg, old_den, old_dd, rand_noise, cfg, sigma, A, B, d_scale, coeff2, u_scale,
                         coeff3, noise_coeff, want_dd=True):
    """Returns (x, denoised, dd); dd is None unless want_dd and old_den is given."""
    xo, den = np.array(x, np.uint16), np.zeros_like(x)
    dd = np.zeros_like(x) if want_dd else None
    opt = lambda a: None if a is None else _p(a)  # noqa: E731
    lib.oracle_cfg_er_sde_full_step(_p(xo), _p(pos), _p(neg), _p(den), opt(old_den), opt(dd), opt(old_dd),
                                    opt(rand_noise), cfg, sigma, A, B, d_scale, coeff2, u_scale, coeff3, noise_coeff,
                                    x.size)
    return xo, den, (dd if want_dd and old_den is not None else None)


def timestep_sinusoid(t, dim):
    out = np.zeros(dim, np.uint16)
    lib.oracle_timestep_sinusoid(float(t), dim, _p(out))
    return out


def cosmos_rope_tables(pe_t, pe_h, pe_w, HD=128):
    S = pe_t * pe_h * pe_w
    c = np.zeros((S, HD), np.uint16)
    s = np.zeros((S, HD), np.uint16)
    lib.oracle_cosmos_rope_tables(pe_t, pe_h, pe_w, HD, _p(c), _p(s))
    return c, s


def standard_rope_tables(T, HD, theta):
    c = np.zeros((T, HD // 2), np.float32)
    s = np.zeros((T, HD // 2), np.float32)
    lib.oracle_standard_rope_tables(T, HD, theta, _p(c), _p(s))
    return c, s
