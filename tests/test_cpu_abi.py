"""CPU-only checks of the C ABI library: it loads without a GPU, exports every symbol the
public headers declare (the C entry points and the reference-signature C++ launchers),
and rejects invalid arguments with the documented status before touching the GPU (no
call here reaches a kernel launch)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_c_functions():
    text = open(os.path.join(ROOT, "include", "anima_b200.h")).read()
    return sorted(set(re.findall(r"ANIMA_API\s+[\w\s\*]*?\b(anima_\w+)\s*\(", text)))


def _declared_cpp_launchers():
    text = open(os.path.join(ROOT, "include", "anima_kernels_compat.h")).read()
    return sorted(set(re.findall(r"^void\s+(\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_reports_version():
    import anima_b200

    assert anima_b200.version().startswith("anima_b200")
    assert "sm_100a" in anima_b200.version()


def test_every_declared_c_symbol_is_exported():
    import anima_b200

    names = _declared_c_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(anima_b200.lib, n), f"{n} declared in anima_b200.h but not exported"
    # and the Python binding covers every compute entry point
    compute = [n for n in names if n not in ("anima_status_string", "anima_version", "anima_wait_timeouts")]
    assert sorted(compute) == sorted(anima_b200.SIGNATURES)


def test_every_reference_launcher_is_exported_with_the_reference_mangling():
    """The shim must export the exact mangled C++ names of src/kernels/kernels.h."""
    import anima_b200
    import refkernels

    declared = _declared_cpp_launchers()
    assert sorted(declared) == sorted(refkernels.LAUNCHERS)
    out = subprocess.run(["nm", "-D", "--defined-only", anima_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for name, (mangled, _) in refkernels.LAUNCHERS.items():
        assert mangled in exported, f"{name}: {mangled} not exported"
    # the reference build exports the same names (so the shim is a drop-in for them)
    if refkernels.reference_available():
        ref_out = subprocess.run(["nm", "-D", "--defined-only", refkernels.REF_LIB_PATH], capture_output=True,
                                 text=True, check=True).stdout
        ref_exported = {line.split()[-1] for line in ref_out.splitlines() if " T " in line}
        for name, (mangled, _) in refkernels.LAUNCHERS.items():
            assert mangled in ref_exported, f"reference build lacks {mangled}"


def test_internal_symbols_are_hidden():
    import anima_b200

    out = subprocess.run(["nm", "-D", "--defined-only", anima_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert not any("sm_count" in s or "allow_dynamic_smem" in s for s in exported)


# ------------------------------------------------------------ argument validation
X, Y, Z = 0x10000, 0x20000, 0x30000  # never dereferenced: every call below fails validation


@pytest.mark.parametrize("call,status", [
    (("anima_rms_norm_bf16", None, None, Z, 4, 128, 1e-6, None), -1),
    (("anima_rms_norm_bf16", X, None, Z, 4, 127, 1e-6, None), -2),
    (("anima_rms_norm_bf16", X, None, Z, -1, 128, 1e-6, None), -2),
    (("anima_rms_norm_bf16", X, None, Z, 4, 0, 1e-6, None), -2),
    (("anima_rms_norm_bf16", X + 1, None, Z, 4, 128, 1e-6, None), -3),
    (("anima_rms_norm_bf16", X, None, X + 2, 4, 128, 1e-6, None), -5),
    (("anima_layer_norm_bf16", X, None, 4, 128, 1e-6, None), -1),
    (("anima_adaln_layernorm_bf16", X, None, Y, Z, 4, 128, 1e-6, None), -1),
    (("anima_residual_gate_adaln_bf16", X, Y, Z, Z, Z, X, 4, 128, 1e-6, None), -5),
    (("anima_residual_gate_adaln_bf16", X, X + 2, Z, Z, Z, Y, 4, 128, 1e-6, None), -5),
    (("anima_gelu_tanh_bf16", X, None, 10, None), -1),
    (("anima_gelu_tanh_bf16", X, Y, -4, None), -2),
    (("anima_gelu_tanh_bias_bf16", X, Y, Z, 10, 3, None), -2),
    (("anima_silu_bf16", X + 1, Y, 10, None), -3),
    (("anima_add_bf16", X, Y, X + 2, 100, None), -5),
    (("anima_mul_bf16", X, None, Z, 100, None), -1),
    (("anima_scale_shift_bcast_bf16", X, Y, Z, X, 4, 7, None), -2),
    (("anima_bias_add_bf16", X, None, X, 4, 8, None), -1),
    (("anima_cfg_euler_step_bf16", X, Y, None, Z, 1.0, 0.5, 0.2, 100, None), -1),
    (("anima_cfg_euler_step_bf16", X, Y, Z, X + 2, 1.0, 0.5, 0.2, 100, None), -5),
    (("anima_cfg_euler_a_rf_step_bf16", X, Y, Z, None, X, 1.0, 0.8, 0.5, 1.0, 1.0, 100, None), -1),
    (("anima_cfg_er_sde_full_step_bf16", X, Y, Z, X + 4, None, None, None, None) + (1.0,) * 9 + (100, None), -5),
    (("anima_patchify_3d_bf16", X, Y, 1, 4, 1, 8, 8, 1, 0, 2, None), -2),
    (("anima_unpatchify_3d_bf16", X, X + 8, 1, 4, 1, 8, 8, 1, 2, 2, None), -5),
    (("anima_channel_scale_shift_bf16", X, Y, Z, X + 2, 1, 4, 16, None), -5),
    (("anima_bias_add_bf16", X, Y, Z, 4, 7, None), -2),
    (("anima_bias_add_bf16", X, Y, X + 2, 4, 8, None), -5),
    (("anima_residual_gate_bcast_bf16", X, Y, None, X, 4, 8, None), -1),
    (("anima_rope_cosmos_strided_bf16", X, Y, Z, 1, 4, 2, 7, None), -2),
    (("anima_rope_cosmos_strided_bf16", X, X, Z, 1, 4, 2, 8, None), -5),
    (("anima_rope_standard_bf16", X, Y + 2, Z, 4, 2, 8, None), -3),
    (("anima_rope_standard_bf16", X, Y, Z, 4, 0, 8, None), -2),
    (("anima_embedding_lookup_bf16", X, Y + 1, Z, 4, 8, 10, None, None), -3),
    (("anima_embedding_lookup_bf16", None, Y, Z, 4, 8, 10, None, None), -1),
    (("anima_embedding_lookup_bf16", X, Y, X + 0x40, 4, 8, 10, None, None), -5),  # out inside the table
    (("anima_rms_norm_channel_bf16", X, Y, Z, 1, 0, 16, 1e-6, None), -2),
    (("anima_rms_norm_channel_silu_bf16", X, None, Z, 1, 4, 16, 1e-6, None), -1),
    (("anima_pixel_norm_bf16", X, X + 2, 1, 4, 16, 1e-6, None), -5),
    (("anima_f32_to_bf16", X + 2, Y, 16, None), -3),
    (("anima_scale_bf16", X, X + 2, 0.5, 16, None), -5),
    (("anima_bf16_to_f32", X, X + 8, 16, None), -5),
    (("anima_nearest_upsample_2x_bf16", X, X + 32, 1, 2, 4, 4, None), -5),
    (("anima_nearest_upsample_2x_bf16", X, None, 1, 2, 4, 4, None), -1),
    (("anima_pixel_norm_bf16", X, Y + 1, 1, 4, 16, 1e-6, None), -3),
    (("anima_head_transpose_bf16", X, X + 64, 4, 8, 16, None), -5),
    (("anima_head_untranspose_batched_bf16", X, None, 1, 4, 8, 16, None), -1),
    (("anima_head_transpose_qk_norm_rope_bf16", X, Y, Z, None, X + 0x100000, 4, 8, 128, 1e-6, None), -1),
    (("anima_head_transpose_qk_norm_rope_bf16", X, Y, None, None, X + 0x800, 4, 8, 128, 1e-6, None), -5),
    (("anima_head_transpose_qk_norm_rope_bf16", X, Y, Z + 2, Z + 0x1002, X + 0x100000, 4, 8, 128, 1e-6, None), -3),
    (("anima_expand_kv_bf16", X, Y, 1, 3, 8, 4, 16, None), -2),
    (("anima_expand_kv_bf16", X, Y + 1, 1, 2, 8, 4, 16, None), -3),
    (("anima_causal_mask_bf16", None, 2, 8, None), -1),
    (("anima_causal_mask_bf16", X, -1, 8, None), -2),
    (("anima_softmax_bf16", X + 1, Y, 4, 16, None), -3),
    (("anima_softmax_bf16", X, X + 2, 4, 16, None), -5),
    (("anima_causal_softmax_bf16", X, None, 2, 8, None), -1),
    (("anima_softmax_f32_to_bf16", X + 2, Y, 4, 16, None), -3),
    (("anima_softmax_f32_to_bf16", X, X + 8, 4, 16, None), -5),
    (("anima_conv_bias_add_bf16", X, Y, Z, 1, 0, 16, None), -2),
    (("anima_conv_bias_add_bf16", X, Y, X + 2, 1, 4, 16, None), -5),
    (("anima_conv_bias_add_bf16", X, Z + 2, Z, 1, 4, 16, None), -5),
    (("anima_conv_bias_residual_add_bf16", X, Y, None, Z, 1, 4, 16, None), -1),
    (("anima_conv_bias_residual_add_bf16", X, Y, Z + 1, Z, 1, 4, 16, None), -3),
    (("anima_conv_bias_rms_norm_channel_silu_bf16", X, Y + 1, Z, X, 1, 4, 16, 1e-6, None), -3),
    (("anima_conv_bias_rms_norm_channel_silu_bf16", X, None, Z, X, 1, 4, 16, 1e-6, None), -1),
    (("anima_qk_norm_rope_bf16", X, None, Y, Z, 1, 4, 2, 128, 1e-6, None), -1),
    (("anima_swiglu_bf16", X, Y, Z + 1, 10, None), -3),
    (("anima_layer_norm_modulate_bf16", X, Y, Z, X + 4, 4, 128, 1e-6, None), -5),
    (("anima_adaln_layernorm_temb_bf16", X, Y, Z, None, X + 0x8000, 4, 128, 1e-6, None), -1),
    (("anima_adaln_layernorm_temb_bf16", X, Y, Z, Y + 2, X + 0x8000, 4, 128, 1e-6, None), -5),
    (("anima_adaln_layernorm_temb_bf16", X, Y, Z, X + 0x8100, X + 0x8000, 4, 128, 1e-6, None), -5),
    (("anima_residual_gate_adaln_temb_bf16", X, Y, Z, Z + 0x1000, Z + 0x2000, Z, X + 0x8000, 4, 128, 1e-6, None), -5),
    (("anima_residual_gate_adaln_temb_bf16", X, Y, Z, Z + 0x1000, Z + 0x2000, Z + 0x3000, X + 0x8000, 4, 127, 1e-6, None), -2),
    (("anima_timestep_embedding_bf16", 1.0, None, X, None, 255, 1e-6, None), -2),
    (("anima_timestep_embedding_bf16", 1.0, None, None, None, 256, 1e-6, None), -1),
    (("anima_timestep_embedding_bf16", 1.0, None, X, X, 256, 1e-6, None), -5),
])
def test_invalid_arguments_are_rejected(call, status):
    import anima_b200

    name, *args = call
    assert getattr(anima_b200.lib, name)(*args) == status
    with pytest.raises(anima_b200.AnimaError) as e:
        anima_b200.call(name, *args)
    assert e.value.status == status


@pytest.mark.parametrize("call", [
    ("anima_rms_norm_bf16", None, None, None, 0, 128, 1e-6, None),
    ("anima_layer_norm_bf16", None, None, 0, 2048, 1e-6, None),
    ("anima_gelu_tanh_bf16", None, None, 1, None),   # floor(1/2) pairs: nothing to do
    ("anima_add_bf16", None, None, None, 0, None),
    ("anima_scale_shift_bcast_bf16", None, None, None, None, 0, 2048, None),
    ("anima_rope_cosmos_strided_bf16", None, None, None, 0, 16, 16, 128, None),
    ("anima_embedding_lookup_bf16", None, None, None, 0, 1024, 0, None, None),
    ("anima_rms_norm_channel_bf16", None, None, None, 0, 512, 64, 1e-6, None),
])
def test_empty_inputs_are_a_no_op(call):
    import anima_b200

    name, *args = call
    assert getattr(anima_b200.lib, name)(*args) == 0


def test_status_strings():
    import anima_b200

    for code in range(-6, 1):
        assert anima_b200.status_string(code)
    assert "NULL" in anima_b200.status_string(-1)


def test_compat_shim_records_errors_per_thread():
    """The reference-signature launchers return void; their argument errors land in
    anima_compat_last_error() (read-and-clear), never in exit()."""
    import ctypes

    import anima_b200
    import refkernels

    shim = refkernels.load_launchers(anima_b200.LIB_PATH)
    assert anima_b200.lib.anima_compat_last_error() == 0
    shim.rms_norm_bf16(None, None, None, 4, 128, 1e-6, None)
    shim.layer_norm_bf16(X, Y, 4, 127, 1e-6, None)  # a second error does not overwrite the first
    assert anima_b200.lib.anima_compat_last_error() == -1
    assert anima_b200.lib.anima_compat_last_error() == 0
    assert isinstance(shim.cdll, ctypes.CDLL)
