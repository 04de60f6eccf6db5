"""Python binding of libanima_b200.so, the B200 (sm_100a) fused layer kernels of anima.cu.

The library's interface is the C ABI in include/anima_b200.h; this module binds it with
ctypes and adds thin wrappers that take torch CUDA tensors (torch supplies device memory
and streams; it is not on the compute path). Every wrapper launches exactly one of the
library's kernels on the current torch stream (or the stream given) and raises
AnimaError on a non-zero status.

There is no fallback: if the shared library is missing or fails to load, importing this
module raises. Build it with `make -C anima.cu_b200` (or __graft_entry__.build()).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_float, c_int, c_int64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libanima_b200.so")

P, I32, I64, F32 = c_void_p, c_int, c_int64, c_float

# name -> argument types (all return int status). Mirrors include/anima_b200.h.
SIGNATURES = {
    "anima_rms_norm_bf16": (P, P, P, I32, I32, F32, P),
    "anima_layer_norm_bf16": (P, P, I32, I32, F32, P),
    "anima_adaln_layernorm_bf16": (P, P, P, P, I32, I32, F32, P),
    "anima_residual_gate_adaln_bf16": (P, P, P, P, P, P, I32, I32, F32, P),
    "anima_adaln_rms_norm_bf16": (P, P, P, P, I32, I32, F32, P),
    "anima_gemma_rms_norm_bf16": (P, P, P, I32, I32, F32, P),
    "anima_gelu_tanh_bf16": (P, P, I64, P),
    "anima_gelu_tanh_bias_bf16": (P, P, P, I64, I32, P),
    "anima_silu_bf16": (P, P, I64, P),
    "anima_silu_bias_bf16": (P, P, P, I64, I32, P),
    "anima_add_bf16": (P, P, P, I64, P),
    "anima_mul_bf16": (P, P, P, I64, P),
    "anima_bias_add_bf16": (P, P, P, I32, I32, P),
    "anima_cfg_euler_step_bf16": (P, P, P, P, F32, F32, F32, I64, P),
    "anima_cfg_euler_a_rf_step_bf16": (P, P, P, P, P) + (F32,) * 5 + (I64, P),
    "anima_cfg_er_sde_full_step_bf16": (P,) * 8 + (F32,) * 9 + (I64, P),
    "anima_patchify_3d_bf16": (P, P) + (I32,) * 8 + (P,),
    "anima_unpatchify_3d_bf16": (P, P) + (I32,) * 8 + (P,),
    "anima_channel_scale_shift_bf16": (P, P, P, P, I32, I32, I32, P),
    "anima_pixel_norm_bf16": (P, P, I32, I32, I32, F32, P),
    "anima_scale_bf16": (P, P, F32, I64, P),
    "anima_f32_to_bf16": (P, P, I64, P),
    "anima_bf16_to_f32": (P, P, I64, P),
    "anima_nearest_upsample_2x_bf16": (P, P, I32, I32, I32, I32, P),
    "anima_head_transpose_bf16": (P, P, I32, I32, I32, P),
    "anima_head_untranspose_bf16": (P, P, I32, I32, I32, P),
    "anima_head_transpose_batched_bf16": (P, P, I32, I32, I32, I32, P),
    "anima_head_untranspose_batched_bf16": (P, P, I32, I32, I32, I32, P),
    "anima_expand_kv_bf16": (P, P, I32, I32, I32, I32, I32, P),
    "anima_head_transpose_qk_norm_rope_bf16": (P, P, P, P, P, I32, I32, I32, F32, P),
    "anima_causal_mask_bf16": (P, I32, I32, P),
    "anima_softmax_bf16": (P, P, I32, I32, P),
    "anima_causal_softmax_bf16": (P, P, I32, I32, P),
    "anima_softmax_f32_to_bf16": (P, P, I32, I32, P),
    "anima_conv_bias_add_bf16": (P, P, P, I32, I32, I32, P),
    "anima_conv_bias_residual_add_bf16": (P, P, P, P, I32, I32, I32, P),
    "anima_conv_bias_rms_norm_channel_silu_bf16": (P, P, P, P, I32, I32, I32, F32, P),
    "anima_scale_shift_bcast_bf16": (P, P, P, P, I32, I32, P),
    "anima_residual_gate_bcast_bf16": (P, P, P, P, I32, I32, P),
    "anima_gated_gelu_bf16": (P, P, P, I64, P),
    "anima_rope_cosmos_strided_bf16": (P, P, P, I32, I32, I32, I32, P),
    "anima_rope_standard_bf16": (P, P, P, I32, I32, I32, P),
    "anima_embedding_lookup_bf16": (P, P, P, I32, I32, I32, P, P),
    "anima_rms_norm_channel_bf16": (P, P, P, I32, I32, I32, F32, P),
    "anima_rms_norm_channel_silu_bf16": (P, P, P, I32, I32, I32, F32, P),
    "anima_qk_norm_rope_bf16": (P, P, P, P, I32, I32, I32, I32, F32, P),
    "anima_swiglu_bf16": (P, P, P, I64, P),
    "anima_layer_norm_modulate_bf16": (P, P, P, P, I32, I32, F32, P),
    "anima_adaln_layernorm_temb_bf16": (P, P, P, P, P, I32, I32, F32, P),
    "anima_residual_gate_adaln_temb_bf16": (P, P, P, P, P, P, P, I32, I32, F32, P),
    "anima_timestep_embedding_bf16": (F32, P, P, P, I32, F32, P),
}

# Status codes (include/anima_b200.h)
ANIMA_OK = 0
ANIMA_ERR_NULL_POINTER = -1
ANIMA_ERR_BAD_SHAPE = -2
ANIMA_ERR_MISALIGNED = -3
ANIMA_ERR_TOO_LARGE = -4
ANIMA_ERR_OVERLAP = -5
ANIMA_ERR_NO_DEVICE = -6


class AnimaError(RuntimeError):
    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed with status {status}: {text}")
        self.status = status


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE}`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = c_int
    lib.anima_status_string.argtypes = [c_int]
    lib.anima_status_string.restype = c_char_p
    lib.anima_version.argtypes = []
    lib.anima_version.restype = c_char_p
    lib.anima_compat_last_error.argtypes = []
    lib.anima_compat_last_error.restype = c_int
    lib.anima_wait_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint), c_int]
    lib.anima_wait_timeouts.restype = c_int
    return lib


lib = _load()


def version() -> str:
    return lib.anima_version().decode()


def status_string(status: int) -> str:
    return lib.anima_status_string(status).decode()


def wait_timeouts(reset: bool = False) -> int:
    """Bounded device waits that ran out on the current device (anima_wait_timeouts); 0 in
    normal operation. Synchronize the streams that ran the kernels first."""
    n = ctypes.c_uint(0)
    st = lib.anima_wait_timeouts(ctypes.byref(n), 1 if reset else 0)
    if st != ANIMA_OK:
        raise AnimaError("anima_wait_timeouts", st, status_string(st))
    return int(n.value)


def call(name: str, *args) -> None:
    """Calls a C entry point with raw arguments and raises on a non-zero status."""
    st = getattr(lib, name)(*args)
    if st != ANIMA_OK:
        raise AnimaError(name, st, status_string(st))


# ------------------------------------------------------------------ torch wrappers
def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream):
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def rms_norm(x, weight, out, N, D, eps=1e-6, stream=None):
    call("anima_rms_norm_bf16", _ptr(x), _ptr(weight), _ptr(out), N, D, eps, _stream(stream))


def layer_norm(x, out, N, D, eps=1e-6, stream=None):
    call("anima_layer_norm_bf16", _ptr(x), _ptr(out), N, D, eps, _stream(stream))


def adaln_layernorm(x, scale, shift, out, N, D, eps=1e-6, stream=None):
    call("anima_adaln_layernorm_bf16", _ptr(x), _ptr(scale), _ptr(shift), _ptr(out), N, D, eps,
         _stream(stream))


def residual_gate_adaln(hidden, sub_out, gate, scale, shift, normed, N, D, eps=1e-6, stream=None):
    call("anima_residual_gate_adaln_bf16", _ptr(hidden), _ptr(sub_out), _ptr(gate), _ptr(scale),
         _ptr(shift), _ptr(normed), N, D, eps, _stream(stream))


def adaln_rms_norm(x, scale, shift, out, N, D, eps=1e-6, stream=None):
    call("anima_adaln_rms_norm_bf16", _ptr(x), _ptr(scale), _ptr(shift), _ptr(out), N, D, eps,
         _stream(stream))


def gemma_rms_norm(x, weight, out, N, D, eps=1e-6, stream=None):
    call("anima_gemma_rms_norm_bf16", _ptr(x), _ptr(weight), _ptr(out), N, D, eps, _stream(stream))


def gelu_tanh(x, out, N, stream=None):
    call("anima_gelu_tanh_bf16", _ptr(x), _ptr(out), N, _stream(stream))


def gelu_tanh_bias(x, bias, out, N, D, stream=None):
    call("anima_gelu_tanh_bias_bf16", _ptr(x), _ptr(bias), _ptr(out), N, D, _stream(stream))


def silu(x, out, N, stream=None):
    call("anima_silu_bf16", _ptr(x), _ptr(out), N, _stream(stream))


def silu_bias(x, bias, out, N, D, stream=None):
    call("anima_silu_bias_bf16", _ptr(x), _ptr(bias), _ptr(out), N, D, _stream(stream))


def add(a, b, out, N, stream=None):
    call("anima_add_bf16", _ptr(a), _ptr(b), _ptr(out), N, _stream(stream))


def mul(a, b, out, N, stream=None):
    call("anima_mul_bf16", _ptr(a), _ptr(b), _ptr(out), N, _stream(stream))


def bias_add(x, bias, out, M, D, stream=None):
    call("anima_bias_add_bf16", _ptr(x), _ptr(bias), _ptr(out), M, D, _stream(stream))


def scale_shift_bcast(x, scale, shift, out, M, D, stream=None):
    call("anima_scale_shift_bcast_bf16", _ptr(x), _ptr(scale), _ptr(shift), _ptr(out), M, D,
         _stream(stream))


def residual_gate_bcast(x, y, gate, out, M, D, stream=None):
    call("anima_residual_gate_bcast_bf16", _ptr(x), _ptr(y), _ptr(gate), _ptr(out), M, D,
         _stream(stream))


def gated_gelu(gate, up, out, N, stream=None):
    call("anima_gated_gelu_bf16", _ptr(gate), _ptr(up), _ptr(out), N, _stream(stream))


def rope_cosmos_strided(x, cos_t, sin_t, B, S, H, HD, stream=None):
    call("anima_rope_cosmos_strided_bf16", _ptr(x), _ptr(cos_t), _ptr(sin_t), B, S, H, HD,
         _stream(stream))


def rope_standard(x, cos_t, sin_t, total_rows, T, D, stream=None):
    call("anima_rope_standard_bf16", _ptr(x), _ptr(cos_t), _ptr(sin_t), total_rows, T, D,
         _stream(stream))


def embedding_lookup(table, ids, out, T, D, vocab=0, bad_id_count=None, stream=None):
    call("anima_embedding_lookup_bf16", _ptr(table), _ptr(ids), _ptr(out), T, D, vocab,
         _ptr(bad_id_count), _stream(stream))


def rms_norm_channel(x, gamma, out, B, C, spatial, eps=1e-6, stream=None):
    call("anima_rms_norm_channel_bf16", _ptr(x), _ptr(gamma), _ptr(out), B, C, spatial, eps,
         _stream(stream))


def rms_norm_channel_silu(x, gamma, out, B, C, spatial, eps=1e-6, stream=None):
    call("anima_rms_norm_channel_silu_bf16", _ptr(x), _ptr(gamma), _ptr(out), B, C, spatial, eps,
         _stream(stream))


def qk_norm_rope(x, weight, cos_t, sin_t, B, S, H, HD, eps=1e-6, stream=None):
    call("anima_qk_norm_rope_bf16", _ptr(x), _ptr(weight), _ptr(cos_t), _ptr(sin_t), B, S, H, HD,
         eps, _stream(stream))


def swiglu(gate, up, out, N, stream=None):
    call("anima_swiglu_bf16", _ptr(gate), _ptr(up), _ptr(out), N, _stream(stream))


def layer_norm_modulate(x, scale, shift, out, N, D, eps=1e-6, stream=None):
    call("anima_layer_norm_modulate_bf16", _ptr(x), _ptr(scale), _ptr(shift), _ptr(out), N, D, eps,
         _stream(stream))


def cfg_euler_step(sample, noise_pos, noise_neg, out, cfg_scale, sigma, sigma_next, N, stream=None):
    call("anima_cfg_euler_step_bf16", _ptr(sample), _ptr(noise_pos), _ptr(noise_neg), _ptr(out), cfg_scale, sigma,
         sigma_next, N, _stream(stream))


def cfg_euler_a_rf_step(sample, noise_pos, noise_neg, rand_noise, out, cfg_scale, sigma, sigma_next, eta, s_noise,
                        N, stream=None):
    call("anima_cfg_euler_a_rf_step_bf16", _ptr(sample), _ptr(noise_pos), _ptr(noise_neg), _ptr(rand_noise),
         _ptr(out), cfg_scale, sigma, sigma_next, eta, s_noise, N, _stream(stream))


def cfg_er_sde_full_step(x, noise_pos, noise_neg, denoised_out, old_denoised, denoised_d_out, old_denoised_d,
                         rand_noise, cfg_scale, sigma, A, B, d_scale, coeff2, u_scale, coeff3, noise_coeff, N,
                         stream=None):
    call("anima_cfg_er_sde_full_step_bf16", _ptr(x), _ptr(noise_pos), _ptr(noise_neg), _ptr(denoised_out),
         _ptr(old_denoised), _ptr(denoised_d_out), _ptr(old_denoised_d), _ptr(rand_noise), cfg_scale, sigma, A, B,
         d_scale, coeff2, u_scale, coeff3, noise_coeff, N, _stream(stream))


def patchify_3d(src, dst, B, C, T, H, W, pT, pH, pW, stream=None):
    call("anima_patchify_3d_bf16", _ptr(src), _ptr(dst), B, C, T, H, W, pT, pH, pW, _stream(stream))


def unpatchify_3d(src, dst, B, C, T, H, W, pT, pH, pW, stream=None):
    call("anima_unpatchify_3d_bf16", _ptr(src), _ptr(dst), B, C, T, H, W, pT, pH, pW, _stream(stream))


def head_transpose(src, dst, H, T, HD, stream=None):
    call("anima_head_transpose_bf16", _ptr(src), _ptr(dst), H, T, HD, _stream(stream))


def head_untranspose(src, dst, H, T, HD, stream=None):
    call("anima_head_untranspose_bf16", _ptr(src), _ptr(dst), H, T, HD, _stream(stream))


def head_transpose_batched(src, dst, B, H, S, HD, stream=None):
    call("anima_head_transpose_batched_bf16", _ptr(src), _ptr(dst), B, H, S, HD, _stream(stream))


def head_untranspose_batched(src, dst, B, H, S, HD, stream=None):
    call("anima_head_untranspose_batched_bf16", _ptr(src), _ptr(dst), B, H, S, HD, _stream(stream))


def head_transpose_qk_norm_rope(src, weight, cos_table, sin_table, dst, H, T, HD, eps=1e-6, stream=None):
    call("anima_head_transpose_qk_norm_rope_bf16", _ptr(src), _ptr(weight), _ptr(cos_table), _ptr(sin_table),
         _ptr(dst), H, T, HD, eps, _stream(stream))


def expand_kv(kv, out, B, KV_H, Q_H, T, D, stream=None):
    call("anima_expand_kv_bf16", _ptr(kv), _ptr(out), B, KV_H, Q_H, T, D, _stream(stream))


def causal_mask(scores, num_heads, T, stream=None):
    call("anima_causal_mask_bf16", _ptr(scores), num_heads, T, _stream(stream))


def softmax(x, out, N, D, stream=None):
    call("anima_softmax_bf16", _ptr(x), _ptr(out), N, D, _stream(stream))


def causal_softmax(scores, out, num_heads, T, stream=None):
    call("anima_causal_softmax_bf16", _ptr(scores), _ptr(out), num_heads, T, _stream(stream))


def softmax_f32_to_bf16(x, out, N, D, stream=None):
    call("anima_softmax_f32_to_bf16", _ptr(x), _ptr(out), N, D, _stream(stream))


def conv_bias_add(x, bias, out, B, C, spatial, stream=None):
    call("anima_conv_bias_add_bf16", _ptr(x), _ptr(bias), _ptr(out), B, C, spatial, _stream(stream))


def conv_bias_residual_add(x, bias, residual, out, B, C, spatial, stream=None):
    call("anima_conv_bias_residual_add_bf16", _ptr(x), _ptr(bias), _ptr(residual), _ptr(out), B, C, spatial,
         _stream(stream))


def conv_bias_rms_norm_channel_silu(x, bias, gamma, out, B, C, spatial, eps=1e-6, stream=None):
    call("anima_conv_bias_rms_norm_channel_silu_bf16", _ptr(x), _ptr(bias), _ptr(gamma), _ptr(out), B, C, spatial,
         eps, _stream(stream))


def scale(x, out, s, N, stream=None):
    call("anima_scale_bf16", _ptr(x), _ptr(out), s, N, _stream(stream))


def f32_to_bf16(x, out, N, stream=None):
    call("anima_f32_to_bf16", _ptr(x), _ptr(out), N, _stream(stream))


def bf16_to_f32(x, out, N, stream=None):
    call("anima_bf16_to_f32", _ptr(x), _ptr(out), N, _stream(stream))


def nearest_upsample_2x(x, out, B, C, H, W, stream=None):
    call("anima_nearest_upsample_2x_bf16", _ptr(x), _ptr(out), B, C, H, W, _stream(stream))


def pixel_norm(x, out, B, C, spatial, eps=1e-6, stream=None):
    call("anima_pixel_norm_bf16", _ptr(x), _ptr(out), B, C, spatial, eps, _stream(stream))


def channel_scale_shift(x, scale, shift, out, B, C, spatial, stream=None):
    call("anima_channel_scale_shift_bf16", _ptr(x), _ptr(scale), _ptr(shift), _ptr(out), B, C, spatial,
         _stream(stream))


def adaln_layernorm_temb(x, mod, temb, gate_out, out, N, D, eps=1e-6, stream=None):
    call("anima_adaln_layernorm_temb_bf16", _ptr(x), _ptr(mod), _ptr(temb), _ptr(gate_out), _ptr(out), N, D,
         eps, _stream(stream))


def residual_gate_adaln_temb(hidden, sub_out, gate_in, mod, temb, gate_out, normed, N, D, eps=1e-6,
                             stream=None):
    call("anima_residual_gate_adaln_temb_bf16", _ptr(hidden), _ptr(sub_out), _ptr(gate_in), _ptr(mod),
         _ptr(temb), _ptr(gate_out), _ptr(normed), N, D, eps, _stream(stream))


def timestep_embedding(t, norm_weight, sinusoid_out, normed_out, dim, eps=1e-6, stream=None):
    call("anima_timestep_embedding_bf16", float(t), _ptr(norm_weight), _ptr(sinusoid_out),
         _ptr(normed_out), dim, eps, _stream(stream))
