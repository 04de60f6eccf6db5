"""TEST INFRASTRUCTURE ONLY: ctypes access to the reference's C++ kernel launchers.

`load_reference()` opens oracle/_ref/libref_kernels.so, the reference's own
src/kernels/*.cu compiled unchanged for sm_100a (oracle/Makefile). It is the GPU-side
oracle of the parity tests and the kernels that `bench.py --impl reference` times.

The launchers have C++ linkage, so they are resolved by their mangled names
(src/kernels/kernels.h). libanima_b200.so exports the same mangled names through its
compatibility shim; `load_launchers(path)` binds either library the same way, which is
how the tests check that the shim forwards correctly.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB_PATH = os.path.join(_HERE, "_ref", "libref_kernels.so")

P, I32, I64, F32 = c_void_p, c_int, c_int64, c_float

# launcher -> (mangled symbol, argument types); kernels.h line ranges in comments.
LAUNCHERS = {
    "rms_norm_bf16": ("_Z13rms_norm_bf16PK13__nv_bfloat16S1_PS_iifP11CUstream_st", (P, P, P, I32, I32, F32, P)),  # :9-11
    "layer_norm_bf16": ("_Z15layer_norm_bf16PK13__nv_bfloat16PS_iifP11CUstream_st", (P, P, I32, I32, F32, P)),  # :14-16
    "adaln_layernorm_bf16": ("_Z20adaln_layernorm_bf16PK13__nv_bfloat16S1_S1_PS_iifP11CUstream_st",
                             (P, P, P, P, I32, I32, F32, P)),  # :19-22
    "residual_gate_adaln_bf16": ("_Z24residual_gate_adaln_bf16P13__nv_bfloat16PKS_S2_S2_S2_S0_iifP11CUstream_st",
                                 (P, P, P, P, P, P, I32, I32, F32, P)),  # :25-30
    "gelu_tanh_bf16": ("_Z14gelu_tanh_bf16PK13__nv_bfloat16PS_lP11CUstream_st", (P, P, I64, P)),  # :33
    "gelu_tanh_bias_bf16": ("_Z19gelu_tanh_bias_bf16PK13__nv_bfloat16S1_PS_liP11CUstream_st",
                            (P, P, P, I64, I32, P)),  # :34-36
    "silu_bf16": ("_Z9silu_bf16PK13__nv_bfloat16PS_lP11CUstream_st", (P, P, I64, P)),  # :39
    "silu_bias_bf16": ("_Z14silu_bias_bf16PK13__nv_bfloat16S1_PS_liP11CUstream_st", (P, P, P, I64, I32, P)),  # :40-42
    "rope_cosmos_strided_bf16": ("_Z24rope_cosmos_strided_bf16P13__nv_bfloat16PKS_S2_iiiiP11CUstream_st",
                                 (P, P, P, I32, I32, I32, I32, P)),  # :51-53
    "scale_bf16": ("_Z10scale_bf16PK13__nv_bfloat16PS_flP11CUstream_st", (P, P, F32, I64, P)),  # :75-76
    "f32_to_bf16": ("_Z11f32_to_bf16PKfP13__nv_bfloat16lP11CUstream_st", (P, P, I64, P)),  # :96
    "bf16_to_f32": ("_Z11bf16_to_f32PK13__nv_bfloat16PflP11CUstream_st", (P, P, I64, P)),  # :97
    "causal_mask_bf16": ("_Z16causal_mask_bf16P13__nv_bfloat16iiP11CUstream_st", (P, I32, I32, P)),  # :104-106
    "softmax_bf16": ("_Z12softmax_bf16PK13__nv_bfloat16PS_iiP11CUstream_st", (P, P, I32, I32, P)),  # :109-111
    "softmax_f32_to_bf16": ("_Z19softmax_f32_to_bf16PKfP13__nv_bfloat16iiP11CUstream_st",
                            (P, P, I32, I32, P)),  # :115-117
    "adaln_rms_norm_bf16": ("_Z19adaln_rms_norm_bf16PK13__nv_bfloat16S1_S1_PS_iifP11CUstream_st",
                            (P, P, P, P, I32, I32, F32, P)),  # :60-63
    "add_bf16": ("_Z8add_bf16PK13__nv_bfloat16S1_PS_lP11CUstream_st", (P, P, P, I64, P)),  # :69-71
    "mul_bf16": ("_Z8mul_bf16PK13__nv_bfloat16S1_PS_lP11CUstream_st", (P, P, P, I64, P)),  # :78-80
    "bias_add_bf16": ("_Z13bias_add_bf16PK13__nv_bfloat16S1_PS_iiP11CUstream_st", (P, P, P, I32, I32, P)),  # :81-83
    "scale_shift_bcast_bf16": ("_Z22scale_shift_bcast_bf16PK13__nv_bfloat16S1_S1_PS_iiP11CUstream_st",
                               (P, P, P, P, I32, I32, P)),  # :87-89
    "residual_gate_bcast_bf16": ("_Z24residual_gate_bcast_bf16PK13__nv_bfloat16S1_S1_PS_iiP11CUstream_st",
                                 (P, P, P, P, I32, I32, P)),  # :90-92
    "gated_gelu_bf16": ("_Z15gated_gelu_bf16PK13__nv_bfloat16S1_PS_lP11CUstream_st", (P, P, P, I64, P)),  # :138-140
    "embedding_lookup_bf16": ("_Z21embedding_lookup_bf16PK13__nv_bfloat16PKiPS_iiP11CUstream_st",
                              (P, P, P, I32, I32, P)),  # :142-144
    "rope_standard_bf16": ("_Z18rope_standard_bf16P13__nv_bfloat16PKfS2_iiiP11CUstream_st",
                           (P, P, P, I32, I32, I32, P)),  # :145-147
    "expand_kv_bf16": ("_Z14expand_kv_bf16PK13__nv_bfloat16PS_iiiiiP11CUstream_st",
                       (P, P, I32, I32, I32, I32, I32, P)),  # :148-150
    "gemma_rms_norm_bf16": ("_Z19gemma_rms_norm_bf16PK13__nv_bfloat16S1_PS_iifP11CUstream_st",
                            (P, P, P, I32, I32, F32, P)),  # :151-153
    "rms_norm_channel_bf16": ("_Z21rms_norm_channel_bf16PK13__nv_bfloat16S1_PS_iiifP11CUstream_st",
                              (P, P, P, I32, I32, I32, F32, P)),  # :177-180
    "nearest_upsample_2x_bf16": ("_Z24nearest_upsample_2x_bf16PK13__nv_bfloat16PS_iiiiP11CUstream_st",
                                 (P, P, I32, I32, I32, I32, P)),  # :172-174
    "pixel_norm_bf16": ("_Z15pixel_norm_bf16PK13__nv_bfloat16PS_iiifP11CUstream_st", (P, P, I32, I32, I32, F32, P)),  # :156-158
    "channel_scale_shift_bf16": ("_Z24channel_scale_shift_bf16PK13__nv_bfloat16S1_S1_PS_iiiP11CUstream_st",
                                 (P, P, P, P, I32, I32, I32, P)),  # :189-192
    "head_transpose_bf16": ("_Z19head_transpose_bf16PK13__nv_bfloat16PS_iiiP11CUstream_st",
                            (P, P, I32, I32, I32, P)),  # :195-197
    "head_untranspose_bf16": ("_Z21head_untranspose_bf16PK13__nv_bfloat16PS_iiiP11CUstream_st",
                              (P, P, I32, I32, I32, P)),  # :200-202
    "head_transpose_batched_bf16": ("_Z27head_transpose_batched_bf16PK13__nv_bfloat16PS_iiiiP11CUstream_st",
                                    (P, P, I32, I32, I32, I32, P)),  # :205-207
    "head_untranspose_batched_bf16": ("_Z29head_untranspose_batched_bf16PK13__nv_bfloat16PS_iiiiP11CUstream_st",
                                      (P, P, I32, I32, I32, I32, P)),  # :210-212
    "patchify_3d_bf16": ("_Z16patchify_3d_bf16PK13__nv_bfloat16PS_iiiiiiiiP11CUstream_st",
                         (P, P) + (I32,) * 8 + (P,)),  # :215-218
    "unpatchify_3d_bf16": ("_Z18unpatchify_3d_bf16PK13__nv_bfloat16PS_iiiiiiiiP11CUstream_st",
                           (P, P) + (I32,) * 8 + (P,)),  # :221-223
    "cfg_euler_step_bf16": ("_Z19cfg_euler_step_bf16PK13__nv_bfloat16S1_S1_PS_ffflP11CUstream_st",
                            (P, P, P, P, F32, F32, F32, I64, P)),  # :244-250
    "cfg_euler_a_rf_step_bf16": ("_Z24cfg_euler_a_rf_step_bf16PK13__nv_bfloat16S1_S1_S1_PS_ffffflP11CUstream_st",
                                 (P, P, P, P, P) + (F32,) * 5 + (I64, P)),  # :253-260
    "cfg_er_sde_full_step_bf16": ("_Z25cfg_er_sde_full_step_bf16P13__nv_bfloat16PKS_S2_S0_S2_S0_S2_S2_ffffffffflP11CUstream_st",
                                  (P,) * 8 + (F32,) * 9 + (I64, P)),  # :264-276
}


class Launchers:
    """Attribute access to the launchers of one library: `L.rms_norm_bf16(...)`."""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing")
        # RTLD_LOCAL: the reference and the B200 library export the same C++ names.
        self.cdll = ctypes.CDLL(path, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        self.path = path
        for name, (sym, argtypes) in LAUNCHERS.items():
            fn = getattr(self.cdll, sym)
            fn.argtypes = list(argtypes)
            fn.restype = None
            setattr(self, name, fn)


def load_launchers(path: str) -> Launchers:
    return Launchers(path)


def load_reference() -> Launchers:
    return Launchers(REF_LIB_PATH)


def reference_available() -> bool:
    return os.path.exists(REF_LIB_PATH)
