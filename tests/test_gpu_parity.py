"""Parity of the B200 kernels (called through the C ABI) with
  (1) the reference's own CUDA kernels, compiled unchanged for sm_100a -- expected
      bit-exact, since the B200 kernels reproduce the reference's reduction order and
      per-element expressions; and
  (2) the CPU restatement in oracle/ -- within one bf16 ulp of the result, judged at
      max(|result|, 2^-12) (the CPU's 1/sqrtf and libm tanhf/expf differ from the GPU's
      rsqrtf/tanhf/expf in the last fp32 bits).
Edge cases follow what the reference's callers exercise: in-place aliasing, N = 1, widths
outside the fast paths (generic kernels), unaligned sub-buffers, odd lengths, tails.
"""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import (assert_bit_exact, assert_bit_exact_or_reference_race, assert_one_ulp, dev, empty_bf16, fresh_run,
                      host, stream_ptr)

pytestmark = pytest.mark.gpu

ORACLE_MAX_ELEMS = 1 << 21  # the CPU restatement runs on inputs up to this size


def _modvec(rng, D, std=0.1):
    return O.randn_bf16(rng, D, std=std)


def _weight(rng, D):
    return O.randn_bf16(rng, D, mean=1.0, std=0.02)


ROW_SHAPES = [(1, 2048), (37, 2048), (4096, 2048), (5, 1024), (300, 1024), (1, 128), (2049, 128),
              (3, 64), (17, 256), (9, 512), (3, 96), (4, 2050), (2, 4096), (2, 6)]


# ---------------------------------------------------------------- row norms
@pytest.mark.parametrize("N,D", ROW_SHAPES)
@pytest.mark.parametrize("weighted", [True, False])
def test_rms_norm(anima, ref, rng, N, D, weighted):
    x = O.randn_bf16(rng, (N, D))
    w = _weight(rng, D) if weighted else None
    dx = dev(x)
    dw = dev(w) if weighted else None
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.rms_norm(dx, dw, out, N, D, 1e-6)
    ref.rms_norm_bf16(dx.data_ptr(), dw.data_ptr() if weighted else None, out_ref.data_ptr(), N, D, 1e-6, stream_ptr())
    # in place, as the DiT QK norm calls it (transformer.cpp:350)
    xi = dev(x)
    anima.rms_norm(xi, dw, xi, N, D, 1e-6)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "rms_norm vs reference")
    assert_bit_exact(host(xi), host(out_ref), "rms_norm in place")
    if N * D <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.rms_norm(x, w, N, D), "rms_norm vs oracle")


@pytest.mark.parametrize("N,D", ROW_SHAPES)
def test_layer_norm(anima, ref, rng, N, D):
    x = O.randn_bf16(rng, (N, D), mean=0.3)
    dx = dev(x)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.layer_norm(dx, out, N, D, 1e-6)
    ref.layer_norm_bf16(dx.data_ptr(), out_ref.data_ptr(), N, D, 1e-6, stream_ptr())
    xi = dev(x)
    anima.layer_norm(xi, xi, N, D, 1e-6)  # in place (transformer.cpp:563)
    torch.cuda.synchronize()
    lazy = lambda: O.layer_norm(x, N, D)  # noqa: E731
    again = fresh_run(lambda r: ref.layer_norm_bf16(dx.data_ptr(), r.data_ptr(), N, D, 1e-6, stream_ptr()), (N, D))
    assert_bit_exact_or_reference_race(host(out), host(out_ref), lazy, "layer_norm vs reference", again)
    assert_bit_exact_or_reference_race(host(xi), host(out_ref), lazy, "layer_norm in place", again)
    if N * D <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.layer_norm(x, N, D), "layer_norm vs oracle")


@pytest.mark.parametrize("N,D", ROW_SHAPES)
def test_adaln_layernorm(anima, ref, rng, N, D):
    x = O.randn_bf16(rng, (N, D))
    sc, sh = _modvec(rng, D), _modvec(rng, D)
    dx, dsc, dsh = dev(x), dev(sc), dev(sh)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.adaln_layernorm(dx, dsc, dsh, out, N, D, 1e-6)
    ref.adaln_layernorm_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), out_ref.data_ptr(), N, D, 1e-6,
                             stream_ptr())
    torch.cuda.synchronize()
    again = fresh_run(lambda r: ref.adaln_layernorm_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), r.data_ptr(),
                                                         N, D, 1e-6, stream_ptr()), (N, D))
    assert_bit_exact_or_reference_race(host(out), host(out_ref), lambda: O.adaln_layernorm(x, sc, sh, N, D),
                                       "adaln_layernorm vs reference", again)
    if N * D <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.adaln_layernorm(x, sc, sh, N, D), "adaln_layernorm vs oracle")


@pytest.mark.parametrize("N,D", ROW_SHAPES)
def test_residual_gate_adaln(anima, ref, rng, N, D):
    x, y = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D))
    g, sc, sh = _modvec(rng, D), _modvec(rng, D), _modvec(rng, D)
    dg, dsc, dsh, dy = dev(g), dev(sc), dev(sh), dev(y)
    h, h_ref = dev(x), dev(x)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.residual_gate_adaln(h, dy, dg, dsc, dsh, out, N, D, 1e-6)
    ref.residual_gate_adaln_bf16(h_ref.data_ptr(), dy.data_ptr(), dg.data_ptr(), dsc.data_ptr(), dsh.data_ptr(),
                                 out_ref.data_ptr(), N, D, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(h), host(h_ref), "residual_gate_adaln hidden vs reference")
    hid = empty_bf16((N, D))

    def again_launch(r):  # the hidden state is updated in place: start from x each run
        hid.copy_(dev(x))
        ref.residual_gate_adaln_bf16(hid.data_ptr(), dy.data_ptr(), dg.data_ptr(), dsc.data_ptr(), dsh.data_ptr(),
                                     r.data_ptr(), N, D, 1e-6, stream_ptr())
    again = fresh_run(again_launch, (N, D))
    assert_bit_exact_or_reference_race(host(out), host(out_ref), lambda: O.residual_gate_adaln(x, y, g, sc, sh, N, D)[1],
                                       "residual_gate_adaln normed vs reference", again)
    if N * D <= ORACLE_MAX_ELEMS:
        oh, on = O.residual_gate_adaln(x, y, g, sc, sh, N, D)
        assert_bit_exact(host(h), oh, "residual_gate_adaln hidden vs oracle")
        assert_one_ulp(host(out), on, "residual_gate_adaln normed vs oracle")


# adaLN-Zero modulation folded into the norms (transformer.cpp:404-456): each fused call
# against the reference's own chain add_bf16 + norm + gate copy, on the same buffers.
TEMB_SHAPES = [(64, 2048), (37, 1024), (5, 512), (16, 96), (3, 130)]


def _temb_inputs(rng, D, offset):
    """mod [3D] as the modulation Linear writes it and temb [3D]; `offset` elements into a
    larger buffer so that offset 1 exercises the 2-byte-aligned (generic) path."""
    mod, temb = _modvec(rng, 3 * D), _modvec(rng, 3 * D)
    mbuf, tbuf = torch.zeros(3 * D + 8, dtype=torch.int16, device="cuda"), torch.zeros(
        3 * D + 8, dtype=torch.int16, device="cuda")
    mbuf[offset:offset + 3 * D] = dev(mod)
    tbuf[offset:offset + 3 * D] = dev(temb)
    return mod, temb, mbuf, tbuf, mbuf[offset:offset + 3 * D], tbuf[offset:offset + 3 * D]


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("N,D", TEMB_SHAPES)
def test_adaln_layernorm_temb_matches_reference_chain(anima, ref, rng, N, D, offset):
    x = O.randn_bf16(rng, (N, D))
    mod, temb, mbuf, tbuf, dm, dt = _temb_inputs(rng, D, offset)
    dx = dev(x)
    out, gate = empty_bf16((N, D)), empty_bf16(D)
    mod_before = host(dm).copy()
    anima.adaln_layernorm_temb(dx, dm, dt, gate, out, N, D, 1e-6)
    # reference chain: mod += temb in place, adaLN, gate copy. Its bf16x2 loads need 4-byte
    # alignment, so it always gets fresh (aligned) copies of mod and temb.
    m, t_ref = dev(mod), dev(temb)
    out_ref = empty_bf16((N, D))
    ref.add_bf16(m.data_ptr(), t_ref.data_ptr(), m.data_ptr(), 3 * D, stream_ptr())
    ref.adaln_layernorm_bf16(dx.data_ptr(), m.data_ptr() + 2 * D, m.data_ptr(), out_ref.data_ptr(), N, D, 1e-6,
                             stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact_or_reference_race(host(out), host(out_ref), lambda: O.adaln_layernorm_temb(x, mod, temb, N, D)[0],
                                       "adaln_layernorm_temb normed vs reference chain")
    assert_bit_exact(host(gate), host(m)[2 * D:], "adaln_layernorm_temb gate vs reference chain")
    assert np.array_equal(host(dm), mod_before), "mod must be left unchanged"
    if N * D <= ORACLE_MAX_ELEMS:
        on, og = O.adaln_layernorm_temb(x, mod, temb, N, D)
        assert_one_ulp(host(out), on, "adaln_layernorm_temb vs oracle")
        assert_bit_exact(host(gate), og, "adaln_layernorm_temb gate vs oracle")


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("N,D", TEMB_SHAPES)
def test_residual_gate_adaln_temb_matches_reference_chain(anima, ref, rng, N, D, offset):
    x, y = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D))
    g_prev = _modvec(rng, D)
    mod, temb, mbuf, tbuf, dm, dt = _temb_inputs(rng, D, offset)
    dy, dgp = dev(y), dev(g_prev)
    h, normed, gate = dev(x), empty_bf16((N, D)), empty_bf16(D)
    anima.residual_gate_adaln_temb(h, dy, dgp, dm, dt, gate, normed, N, D, 1e-6)
    # reference chain with one gate buffer, on fresh (4-byte aligned) copies
    m, t_ref, h_ref, gate_ref = dev(mod), dev(temb), dev(x), dev(g_prev)
    normed_ref = empty_bf16((N, D))
    ref.add_bf16(m.data_ptr(), t_ref.data_ptr(), m.data_ptr(), 3 * D, stream_ptr())
    ref.residual_gate_adaln_bf16(h_ref.data_ptr(), dy.data_ptr(), gate_ref.data_ptr(), m.data_ptr() + 2 * D,
                                 m.data_ptr(), normed_ref.data_ptr(), N, D, 1e-6, stream_ptr())
    gate_ref.copy_(m[2 * D:])
    torch.cuda.synchronize()
    assert_bit_exact(host(h), host(h_ref), "residual_gate_adaln_temb hidden vs reference chain")
    assert_bit_exact_or_reference_race(
        host(normed), host(normed_ref), lambda: O.residual_gate_adaln_temb(x, y, g_prev, mod, temb, N, D)[1],
        "residual_gate_adaln_temb normed vs reference chain")
    assert_bit_exact(host(gate), host(gate_ref), "residual_gate_adaln_temb gate vs reference chain")
    if N * D <= ORACLE_MAX_ELEMS:
        oh, on, og = O.residual_gate_adaln_temb(x, y, g_prev, mod, temb, N, D)
        assert_bit_exact(host(h), oh, "residual_gate_adaln_temb hidden vs oracle")
        assert_one_ulp(host(normed), on, "residual_gate_adaln_temb normed vs oracle")
        assert_bit_exact(host(gate), og, "residual_gate_adaln_temb gate vs oracle")


@pytest.mark.parametrize("N,D", [(1, 2048), (65, 2048), (7, 128), (3, 96)])
def test_adaln_rms_norm(anima, ref, rng, N, D):
    x = O.randn_bf16(rng, (N, D))
    sc, sh = O.randn_bf16(rng, (N, D), std=0.1), O.randn_bf16(rng, (N, D), std=0.1)
    dx, dsc, dsh = dev(x), dev(sc), dev(sh)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.adaln_rms_norm(dx, dsc, dsh, out, N, D, 1e-6)
    ref.adaln_rms_norm_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), out_ref.data_ptr(), N, D, 1e-6,
                            stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "adaln_rms_norm vs reference")
    assert_one_ulp(host(out), O.adaln_rms_norm(x, sc, sh, N, D), "adaln_rms_norm vs oracle")


@pytest.mark.parametrize("N,D", [(4, 1024), (3, 2048), (5, 100)])
def test_gemma_rms_norm(anima, ref, rng, N, D):
    x, w = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, D, std=0.1)
    dx, dw = dev(x), dev(w)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.gemma_rms_norm(dx, dw, out, N, D, 1e-6)
    ref.gemma_rms_norm_bf16(dx.data_ptr(), dw.data_ptr(), out_ref.data_ptr(), N, D, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "gemma_rms_norm vs reference")
    assert_one_ulp(host(out), O.gemma_rms_norm(x, w, N, D), "gemma_rms_norm vs oracle")


def test_row_norm_unaligned_subbuffer(anima, ref, rng):
    """Row blocks that start 2 or 4 bytes into an allocation take the generic path.

    The reference kernels load bf16 pairs (4-byte accesses, layer_norm.cu:99), so they
    are only ever given 4-byte-aligned pointers here; the 2-byte offset is checked
    against the CPU restatement alone.
    """
    N, D = 8, 2048
    base = O.randn_bf16(rng, N * D + 8)
    d = dev(base)
    scv, shv = _modvec(rng, D), _modvec(rng, D)
    sc, sh = dev(scv), dev(shv)
    from anima_b200 import call

    for off in (2, 4):  # bytes
        e = off // 2
        out, out_ref = empty_bf16(N * D + 8), empty_bf16(N * D + 8)
        call("anima_adaln_layernorm_bf16", d.data_ptr() + off, sc.data_ptr(), sh.data_ptr(), out.data_ptr() + off, N,
             D, 1e-6, stream_ptr())
        if off % 4 == 0:
            ref.adaln_layernorm_bf16(d.data_ptr() + off, sc.data_ptr(), sh.data_ptr(), out_ref.data_ptr() + off, N, D,
                                     1e-6, stream_ptr())
        torch.cuda.synchronize()
        got = host(out)[e:e + N * D]
        want = O.adaln_layernorm(np.ascontiguousarray(base[e:e + N * D]), scv, shv, N, D)
        if off % 4 == 0:
            assert_bit_exact_or_reference_race(got, host(out_ref)[e:e + N * D], lambda: want,
                                               f"adaln at +{off} B vs reference")
        assert_one_ulp(got, want, f"adaln at +{off} B vs oracle")


# ---------------------------------------------------------------- elementwise
FLAT_SIZES = [2, 8, 9, 1000, 4097, 8 * 8192 * 9 + 6, 1 << 20]


@pytest.mark.parametrize("N", FLAT_SIZES)
@pytest.mark.parametrize("op", ["gelu_tanh", "silu"])
def test_unary(anima, ref, rng, N, op):
    x = O.randn_bf16(rng, N, std=2.0)
    dx = dev(x)
    out, out_ref = dev(np.zeros(N, np.uint16)), dev(np.zeros(N, np.uint16))
    getattr(anima, op)(dx, out, N)
    getattr(ref, op + "_bf16")(dx.data_ptr(), out_ref.data_ptr(), N, stream_ptr())
    xi = dev(x)
    getattr(anima, op)(xi, xi, N)  # in place (vae.cpp:184, llm_adapter.cpp:301)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), f"{op} vs reference")
    got_inplace = host(xi)
    assert_bit_exact(got_inplace[: N // 2 * 2], host(out_ref)[: N // 2 * 2], f"{op} in place")
    if N % 2:
        assert got_inplace[-1] == x[-1], "odd last element must stay untouched, as in the reference"
    if N <= ORACLE_MAX_ELEMS:
        want = getattr(O, op)(x)
        assert_one_ulp(host(out)[: N // 2 * 2], want[: N // 2 * 2], f"{op} vs oracle")


@pytest.mark.parametrize("op", ["gelu_tanh", "silu"])
def test_unary_extreme_inputs(anima, ref, op):
    """Saturation, overflow of exp and tiny values go through the same arithmetic."""
    v = np.array([0.0, -0.0, 1e-30, -1e-30, 3.0, -3.0, 8.0, -8.0, 20.0, -20.0, 88.0, -88.0, 100.0, -100.0,
                  3.0e38, -3.0e38, np.inf, -np.inf], np.float32)
    x = O.f32_to_bf16(np.concatenate([v, np.linspace(-12, 12, 4096, dtype=np.float32)]))
    N = x.size
    dx = dev(x)
    out, out_ref = empty_bf16(N), empty_bf16(N)
    getattr(anima, op)(dx, out, N)
    getattr(ref, op + "_bf16")(dx.data_ptr(), out_ref.data_ptr(), N, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), f"{op} extremes vs reference")


@pytest.mark.parametrize("op", ["gelu_tanh", "silu"])
@pytest.mark.parametrize("reps", [1, 8, 9, 513])
def test_unary_exhaustive(anima, ref, op, reps):
    """GELU and SiLU map one bf16 input to one bf16 output, so all 65536 inputs (both
    zeros, subnormals, Inf, every NaN payload) settle parity completely. 131072 elements
    take the table-free kernel (approximation + exact-formula fallback); 2^20 and more take
    the shared-memory table kernel, whose table the exact formula filled (from 2^26, as at
    reps = 513, its TMA-fed form); the extra 6 elements at odd reps exercise the scalar tail."""
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = np.tile(np.concatenate([x, x[::-1]]), reps)  # both halves of a bf16 pair see every value
    if reps > 1 and reps % 2:
        x = np.concatenate([x, x[:6]])
    dx = dev(x)
    n = x.size
    out, out_ref = empty_bf16(n), empty_bf16(n)
    getattr(anima, op)(dx, out, n)
    getattr(ref, op + "_bf16")(dx.data_ptr(), out_ref.data_ptr(), n, stream_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(host(out), host(out_ref)), f"{op}: {int((host(out) != host(out_ref)).sum())} of {n} differ"
    if reps == 513:  # in place, as the DiT FFN calls it (llm_adapter.cpp:301), through the TMA-fed form
        xi = dev(x)
        getattr(anima, op)(xi, xi, n)
        torch.cuda.synchronize()
        assert np.array_equal(host(xi), host(out_ref)), f"{op} in place"
    assert anima.wait_timeouts() == 0


def test_swiglu_exhaustive_gate(anima, ref, rng):
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    u = O.randn_bf16(rng, x.size)
    dg, du = dev(x), dev(u)
    out = empty_bf16(x.size)
    anima.swiglu(dg, du, out, x.size)
    gr = dev(x)
    ref.silu_bf16(gr.data_ptr(), gr.data_ptr(), x.size, stream_ptr())
    ref.mul_bf16(gr.data_ptr(), du.data_ptr(), gr.data_ptr(), x.size, stream_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(host(out), host(gr))


@pytest.mark.parametrize("op", ["gelu_tanh_bias", "silu_bias"])
@pytest.mark.parametrize("M,D", [(3, 6144), (1000, 8), (7, 10)])
def test_unary_bias(anima, ref, rng, op, M, D):
    x, b = O.randn_bf16(rng, (M, D)), O.randn_bf16(rng, D, std=0.5)
    dx, db = dev(x), dev(b)
    N = M * D
    out, out_ref = empty_bf16(N), empty_bf16(N)
    getattr(anima, op)(dx, db, out, N, D)
    getattr(ref, op + "_bf16")(dx.data_ptr(), db.data_ptr(), out_ref.data_ptr(), N, D, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), f"{op} vs reference")
    base = op.replace("_bias", "")
    assert_one_ulp(host(out), getattr(O, base)(x.reshape(-1), b, D), f"{op} vs oracle")


@pytest.mark.parametrize("N", [2, 6144, 4097, 512 * 3072, 1 << 22])
@pytest.mark.parametrize("op", ["add", "mul"])
def test_binary(anima, ref, rng, N, op):
    a, b = O.randn_bf16(rng, N), O.randn_bf16(rng, N)
    da, db = dev(a), dev(b)
    out, out_ref = empty_bf16(N), empty_bf16(N)
    getattr(anima, op)(da, db, out, N)
    getattr(ref, op + "_bf16")(da.data_ptr(), db.data_ptr(), out_ref.data_ptr(), N, stream_ptr())
    ai = dev(a)
    getattr(anima, op)(ai, db, ai, N)  # out == a (qwen3.cpp:249, transformer.cpp:408)
    torch.cuda.synchronize()
    assert_bit_exact(host(out)[: N // 2 * 2], host(out_ref)[: N // 2 * 2], f"{op} vs reference")
    assert_bit_exact(host(ai)[: N // 2 * 2], host(out_ref)[: N // 2 * 2], f"{op} in place")
    if N <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out)[: N // 2 * 2], getattr(O, op)(a, b)[: N // 2 * 2], f"{op} vs oracle")


def test_binary_unaligned(anima, ref, rng):
    """Unaligned sub-buffers take the scalar path. The reference's bf16-pair loads need
    4-byte alignment (elementwise.cu:45-49), so it only sees the 4-byte offset."""
    N = 10001
    a, b = O.randn_bf16(rng, N + 2), O.randn_bf16(rng, N + 2)
    da, db = dev(a), dev(b)
    from anima_b200 import call

    for off in (2, 4):
        e = off // 2
        out, out_ref = empty_bf16(N + 2), empty_bf16(N + 2)
        call("anima_add_bf16", da.data_ptr() + off, db.data_ptr(), out.data_ptr() + off, N - 1, stream_ptr())
        if off % 4 == 0:
            ref.add_bf16(da.data_ptr() + off, db.data_ptr(), out_ref.data_ptr() + off, N - 1, stream_ptr())
        torch.cuda.synchronize()
        n = (N - 1) // 2 * 2
        got = host(out)[e:e + n]
        if off % 4 == 0:
            assert_bit_exact(got, host(out_ref)[e:e + n], f"add at +{off} B vs reference")
        assert_bit_exact(got, O.add(np.ascontiguousarray(a[e:e + n]), np.ascontiguousarray(b[:n])),
                         f"add at +{off} B vs oracle")


@pytest.mark.parametrize("N", [8, 512 * 3072, 4099])
def test_swiglu_matches_reference_chain(anima, ref, rng, N):
    g, u = O.randn_bf16(rng, N, std=2.0), O.randn_bf16(rng, N)
    dg, du = dev(g), dev(u)
    out = empty_bf16(N)
    anima.swiglu(dg, du, out, N)
    gr = dev(g)  # qwen3.cpp:248-250: silu in place, then mul into the gate buffer
    ref.silu_bf16(gr.data_ptr(), gr.data_ptr(), N, stream_ptr())
    ref.mul_bf16(gr.data_ptr(), du.data_ptr(), gr.data_ptr(), N, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out)[: N // 2 * 2], host(gr)[: N // 2 * 2], "swiglu vs silu+mul")


@pytest.mark.parametrize("N", [1, 9, 100003])
def test_gated_gelu(anima, ref, rng, N):
    g, u = O.randn_bf16(rng, N, std=2.0), O.randn_bf16(rng, N)
    dg, du = dev(g), dev(u)
    out, out_ref = empty_bf16(N), empty_bf16(N)
    anima.gated_gelu(dg, du, out, N)
    ref.gated_gelu_bf16(dg.data_ptr(), du.data_ptr(), out_ref.data_ptr(), N, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "gated_gelu vs reference")
    assert_one_ulp(host(out), O.gated_gelu(g, u), "gated_gelu vs oracle")


@pytest.mark.parametrize("M,D", [(1, 2048), (300, 2048), (7, 1024), (3, 96), (5, 10), (4096, 3072)])
def test_bias_add(anima, ref, rng, M, D):
    x, b = O.randn_bf16(rng, (M, D)), _modvec(rng, D, std=1.0)
    dx, db = dev(x), dev(b)
    out, out_ref = empty_bf16((M, D)), empty_bf16((M, D))
    anima.bias_add(dx, db, out, M, D)
    ref.bias_add_bf16(dx.data_ptr(), db.data_ptr(), out_ref.data_ptr(), M, D, stream_ptr())
    xi = dev(x)
    anima.bias_add(xi, db, xi, M, D)  # in place (linear.cpp:78)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "bias_add vs reference")
    assert_bit_exact(host(xi), host(out_ref), "bias_add in place")
    if M * D <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out), O.bias_add(x, b, M, D), "bias_add vs oracle")


@pytest.mark.parametrize("M,D", [(1, 2048), (8192, 2048), (33, 96), (5, 10)])
def test_scale_shift_bcast(anima, ref, rng, M, D):
    x, sc, sh = O.randn_bf16(rng, (M, D)), _modvec(rng, D), _modvec(rng, D)
    dx, dsc, dsh = dev(x), dev(sc), dev(sh)
    out, out_ref = empty_bf16((M, D)), empty_bf16((M, D))
    anima.scale_shift_bcast(dx, dsc, dsh, out, M, D)
    ref.scale_shift_bcast_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), out_ref.data_ptr(), M, D, stream_ptr())
    xi = dev(x)
    anima.scale_shift_bcast(xi, dsc, dsh, xi, M, D)  # in place (transformer.cpp:564)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "scale_shift_bcast vs reference")
    assert_bit_exact(host(xi), host(out_ref), "scale_shift_bcast in place")
    if M * D <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out), O.scale_shift_bcast(x, sc, sh, M, D), "scale_shift_bcast vs oracle")


@pytest.mark.parametrize("M,D", [(1, 2048), (8192, 2048), (33, 96), (5, 10)])
def test_residual_gate_bcast(anima, ref, rng, M, D):
    x, y, g = O.randn_bf16(rng, (M, D)), O.randn_bf16(rng, (M, D)), _modvec(rng, D)
    dx, dy, dg = dev(x), dev(y), dev(g)
    out, out_ref = empty_bf16((M, D)), empty_bf16((M, D))
    anima.residual_gate_bcast(dx, dy, dg, out, M, D)
    ref.residual_gate_bcast_bf16(dx.data_ptr(), dy.data_ptr(), dg.data_ptr(), out_ref.data_ptr(), M, D, stream_ptr())
    xi = dev(x)
    anima.residual_gate_bcast(xi, dy, dg, xi, M, D)  # out == x (transformer.cpp:464)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "residual_gate_bcast vs reference")
    assert_bit_exact(host(xi), host(out_ref), "residual_gate_bcast in place")
    if M * D <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out), O.residual_gate_bcast(x, y, g, M, D), "residual_gate_bcast vs oracle")


# ---------------------------------------------------------------- RoPE
@pytest.mark.parametrize("B,pe,H,HD", [(2, (1, 32, 32), 16, 128), (1, (1, 8, 8), 16, 128), (3, (1, 4, 6), 2, 64),
                                       (2, (1, 3, 5), 3, 12)])
def test_rope_cosmos_strided(anima, ref, rng, B, pe, H, HD):
    S = pe[0] * pe[1] * pe[2]
    cos_t, sin_t = O.cosmos_rope_tables(*pe, HD=HD)
    x = O.randn_bf16(rng, (B * S, H * HD))
    dc, ds = dev(cos_t), dev(sin_t)
    a, r = dev(x), dev(x)
    anima.rope_cosmos_strided(a, dc, ds, B, S, H, HD)
    ref.rope_cosmos_strided_bf16(r.data_ptr(), dc.data_ptr(), ds.data_ptr(), B, S, H, HD, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(a), host(r), "rope_cosmos_strided vs reference")
    assert_bit_exact(host(a), O.rope_cosmos_strided(x, cos_t, sin_t, B, S, H, HD), "rope_cosmos_strided vs oracle")


@pytest.mark.parametrize("heads,T,HD,theta", [(16, 512, 128, 1e6), (8, 512, 128, 1e6), (16, 77, 64, 1e4),
                                              (2, 5, 20, 1e4)])
def test_rope_standard(anima, ref, rng, heads, T, HD, theta):
    cos_t, sin_t = O.standard_rope_tables(T, HD, theta)
    rows = heads * T
    x = O.randn_bf16(rng, (rows, HD))
    dc, ds = dev(cos_t), dev(sin_t)
    a, r = dev(x), dev(x)
    anima.rope_standard(a, dc, ds, rows, T, HD)
    ref.rope_standard_bf16(r.data_ptr(), dc.data_ptr(), ds.data_ptr(), rows, T, HD, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(a), host(r), "rope_standard vs reference")
    assert_one_ulp(host(a), O.rope_standard(x, cos_t, sin_t, rows, T, HD), "rope_standard vs oracle")


@pytest.mark.parametrize("B,pe,H,HD", [(2, (1, 32, 32), 16, 128), (1, (1, 3, 5), 4, 128), (2, (1, 4, 4), 2, 64)])
def test_qk_norm_rope_matches_reference_chain(anima, ref, rng, B, pe, H, HD):
    S = pe[0] * pe[1] * pe[2]
    cos_t, sin_t = O.cosmos_rope_tables(*pe, HD=HD)
    x, w = O.randn_bf16(rng, (B * S, H * HD)), _weight(rng, HD)
    dc, ds, dw = dev(cos_t), dev(sin_t), dev(w)
    a, r = dev(x), dev(x)
    anima.qk_norm_rope(a, dw, dc, ds, B, S, H, HD, 1e-6)
    ref.rms_norm_bf16(r.data_ptr(), dw.data_ptr(), r.data_ptr(), B * S * H, HD, 1e-6, stream_ptr())
    ref.rope_cosmos_strided_bf16(r.data_ptr(), dc.data_ptr(), ds.data_ptr(), B, S, H, HD, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(a), host(r), "qk_norm_rope vs rms_norm + rope_cosmos_strided")


# ---------------------------------------------------------------- gather
def test_embedding_lookup_qwen3(anima, ref, rng):
    V, D, T = 151936, 1024, 512
    table = O.randn_bf16(rng, (V, D), std=0.02)
    ids = rng.integers(0, V, T, dtype=np.int32)
    ids[:4] = [0, V - 1, 7, 7]
    dt, di = dev(table), dev(ids)
    out, out_ref = empty_bf16((T, D)), empty_bf16((T, D))
    anima.embedding_lookup(dt, di, out, T, D, V)
    ref.embedding_lookup_bf16(dt.data_ptr(), di.data_ptr(), out_ref.data_ptr(), T, D, stream_ptr())
    torch.cuda.synchronize()
    got = host(out)
    assert_bit_exact(got, host(out_ref), "embedding_lookup vs reference")
    assert np.array_equal(got, table[ids]), "embedding_lookup vs table[ids]"


@pytest.mark.parametrize("D", [1024, 64, 6])
def test_embedding_lookup_bad_ids(anima, rng, D):
    V, T = 100, 9
    table = O.randn_bf16(rng, (V, D))
    ids = np.array([0, 99, 100, -1, 5, 2**31 - 1, -(2**31), 50, 100], np.int32)
    dt, di = dev(table), dev(ids)
    out = dev(np.full((T, D), 0x3F80, np.uint16))
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    anima.embedding_lookup(dt, di, out, T, D, V, bad)
    torch.cuda.synchronize()
    got = host(out)
    assert int(bad.item()) == 5
    want = O.embedding_lookup(table, ids, T, D, V)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- VAE channel norm
@pytest.mark.parametrize("B,C,H,W", [(1, 512, 32, 32), (2, 96, 16, 16), (1, 128, 8, 12), (1, 100, 5, 7),
                                     (3, 16, 4, 4), (1, 1536, 8, 8), (2, 100, 5, 8), (1, 3, 16, 16),
                                     (1, 4000, 2, 4), (1, 64, 160, 160), (1, 65, 8, 8), (2, 512, 10, 12)])
def test_rms_norm_channel(anima, ref, rng, B, C, H, W):
    sp = H * W
    x, g = O.randn_bf16(rng, (B, C, sp)), _weight(rng, C)
    dx, dg = dev(x), dev(g)
    out, out_ref = empty_bf16((B, C, sp)), empty_bf16((B, C, sp))
    anima.rms_norm_channel(dx, dg, out, B, C, sp, 1e-6)
    ref.rms_norm_channel_bf16(dx.data_ptr(), dg.data_ptr(), out_ref.data_ptr(), B, C, sp, 1e-6, stream_ptr())
    xi = dev(x)
    anima.rms_norm_channel(xi, dg, xi, B, C, sp, 1e-6)  # in place (vae.cpp:148)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "rms_norm_channel vs reference")
    assert_bit_exact(host(xi), host(out_ref), "rms_norm_channel in place")
    if x.size <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.rms_norm_channel(x, g, B, C, sp), "rms_norm_channel vs oracle")


@pytest.mark.parametrize("B,C,H,W", [(1, 512, 32, 32), (1, 96, 10, 10), (2, 100, 5, 8), (1, 64, 160, 160),
                                     (2, 128, 64, 64), (2, 512, 10, 12)])
def test_pixel_norm(anima, ref, rng, B, C, H, W):
    """vae_kernels.cu:15-52 through each channel-norm kernel: cluster (few tiles), tile (many),
    per-pixel (spatial % 8 != 0)."""
    sp = H * W
    x = O.randn_bf16(rng, (B, C, sp))
    dx = dev(x)
    out, out_ref = empty_bf16((B, C, sp)), empty_bf16((B, C, sp))
    anima.pixel_norm(dx, out, B, C, sp, 1e-6)
    ref.pixel_norm_bf16(dx.data_ptr(), out_ref.data_ptr(), B, C, sp, 1e-6, stream_ptr())
    xi = dev(x)
    anima.pixel_norm(xi, xi, B, C, sp, 1e-6)  # in place
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "pixel_norm vs reference")
    assert_bit_exact(host(xi), host(out_ref), "pixel_norm in place")
    if x.size <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.pixel_norm(x, B, C, sp), "pixel_norm vs oracle")


# Large fused-SiLU tensors (>= 2^24 elements) at C = 128 / 256 that end in a partial tile,
# with several images (B > 1) in one launch.
CN_LARGE_SHAPES = [(2, 128, 260, 260), (3, 256, 150, 152)]


@pytest.mark.parametrize("B,C,H,W", [(1, 512, 32, 32), (1, 96, 10, 10), (2, 100, 5, 8), (1, 256, 64, 64),
                                     (1, 64, 160, 160), (1, 128, 150, 132), (2, 256, 100, 104),
                                     (1, 512, 150, 132), (1, 512, 96, 96)] + CN_LARGE_SHAPES)
def test_rms_norm_channel_silu_matches_reference_chain(anima, ref, rng, B, C, H, W):
    """Through the cluster kernel (few tiles), the TMA tile kernel (many tiles; three shapes end
    in a partial tile, which the TMA loads fill with zeros; CN_LARGE_SHAPES at full size) and,
    for few tiles of a large tensor at C = 512, the TMA norm followed by the SiLU table
    kernel."""
    sp = H * W
    x, g = O.randn_bf16(rng, (B, C, sp)), _weight(rng, C)
    dx, dg = dev(x), dev(g)
    out = empty_bf16((B, C, sp))
    anima.rms_norm_channel_silu(dx, dg, out, B, C, sp, 1e-6)
    r = dev(x)  # vae.cpp:148 then :184
    ref.rms_norm_channel_bf16(r.data_ptr(), dg.data_ptr(), r.data_ptr(), B, C, sp, 1e-6, stream_ptr())
    ref.silu_bf16(r.data_ptr(), r.data_ptr(), B * C * sp, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "rms_norm_channel_silu vs rms_norm_channel + silu")
    assert anima.wait_timeouts() == 0


# ---------------------------------------------------------------- fused LN + modulate
@pytest.mark.parametrize("N,D", [(1024, 2048), (3, 96)])
def test_layer_norm_modulate_matches_reference_chain(anima, ref, rng, N, D):
    x, sc, sh = O.randn_bf16(rng, (N, D)), _modvec(rng, D), _modvec(rng, D)
    dx, dsc, dsh = dev(x), dev(sc), dev(sh)
    out = empty_bf16((N, D))
    anima.layer_norm_modulate(dx, dsc, dsh, out, N, D, 1e-6)
    r = dev(x)  # transformer.cpp:563-564, both in place
    ref.layer_norm_bf16(r.data_ptr(), r.data_ptr(), N, D, 1e-6, stream_ptr())
    ref.scale_shift_bcast_bf16(r.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), r.data_ptr(), N, D, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact_or_reference_race(host(out), host(r), lambda: O.layer_norm_modulate(x, sc, sh, N, D),
                                       "layer_norm_modulate vs layer_norm + scale_shift_bcast")


# ---------------------------------------------------------------- timestep embedding
@pytest.mark.parametrize("dim", [256, 2048])
def test_timestep_embedding(anima, ref, rng, dim):
    w = _weight(rng, dim)
    dw = dev(w)
    ts = list(rng.uniform(0.0, 1.0, 12).astype(np.float32) * np.float32(1000.0)) + [0.0, 1.0, 999.0, 0.0313]
    for t in ts:
        sin_out, normed = empty_bf16(dim), empty_bf16(dim)
        anima.timestep_embedding(float(t), dw, sin_out, normed, dim, 1e-6)
        normed_ref = empty_bf16(dim)
        ref.rms_norm_bf16(sin_out.data_ptr(), dw.data_ptr(), normed_ref.data_ptr(), 1, dim, 1e-6, stream_ptr())
        torch.cuda.synchronize()
        # the host loop of transformer.cpp:182-197, restated in oracle.c
        assert_one_ulp(host(sin_out), O.timestep_sinusoid(t, dim), f"sinusoid t={t}")
        assert_bit_exact(host(normed), host(normed_ref), f"timestep rms_norm t={t}")


# ---------------------------------------------------------------- sampler steps and latent I/O
# transpose.cu:128-465, vae_kernels.cu:174-206. The reference kernels use 2-byte accesses, so
# they also take the offset (unaligned) buffers.
def _bf_at(a, offset):
    """a on the device, `offset` elements into a larger buffer (offset 1: 2-byte aligned)."""
    buf = torch.zeros(a.size + 8, dtype=torch.int16, device="cuda")
    buf[offset:offset + a.size] = dev(a.reshape(-1))
    return buf[offset:offset + a.size]


@pytest.mark.parametrize("B,C,sp", [(1, 16, 128 * 128), (2, 16, 4096 + 3), (1, 3, 10), (3, 5, 8)])
def test_channel_scale_shift(anima, ref, rng, B, C, sp):
    x = O.randn_bf16(rng, (B, C, sp))
    sc, sh = O.randn_bf16(rng, C, mean=1.0, std=0.3), O.randn_bf16(rng, C, std=0.5)
    dx, dsc, dsh = dev(x), dev(sc), dev(sh)
    out, out_ref = empty_bf16((B, C, sp)), empty_bf16((B, C, sp))
    anima.channel_scale_shift(dx, dsc, dsh, out, B, C, sp)
    ref.channel_scale_shift_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), out_ref.data_ptr(), B, C, sp,
                                 stream_ptr())
    xi = dev(x)
    anima.channel_scale_shift(xi, dsc, dsh, xi, B, C, sp)  # in place (vae.cpp:406)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "channel_scale_shift vs reference")
    assert_bit_exact(host(xi), host(out_ref), "channel_scale_shift in place")
    assert_bit_exact(host(out), O.channel_scale_shift(x, sc, sh, B, C, sp).reshape(-1), "channel_scale_shift vs oracle")


# ---------------------------------------------------------------- VAE conv epilogue
# The vectorised path (spatial % 8 == 0) at several grid-stride depths, the scalar path
# (spatial % 8 != 0), and for the fused norm each of its three kernels: cluster (few tiles),
# tile (many tiles) and the per-pixel kernel.
CONV_SHAPES = [(1, 512, 32, 32), (1, 96, 10, 10), (2, 100, 5, 8), (1, 256, 64, 64), (1, 64, 160, 160),
               (1, 128, 256, 256), (2, 3, 3, 6), (2, 256, 100, 104), (1, 512, 150, 132), (1, 512, 96, 96)]


def _ref_conv_bias(ref, dx, db, B, C, sp):
    """The reference's bias launch (causal_conv3d.cu:187-195) stores bf16(x + bias[c]). That
    kernel is file-local to causal_conv3d_forward, so the reference side runs the same
    per-element sum through add_bf16 (elementwise.cu:37-53: fp32 add, RNE) with the bias
    broadcast over each channel plane."""
    bexp = db.view(1, C, 1).expand(B, C, sp).contiguous()
    out = empty_bf16((B, C, sp))
    ref.add_bf16(dx.data_ptr(), bexp.data_ptr(), out.data_ptr(), B * C * sp, stream_ptr())
    return out


@pytest.mark.parametrize("B,C,H,W", CONV_SHAPES)
def test_conv_bias_add(anima, ref, rng, B, C, H, W):
    sp = H * W
    x, b = O.randn_bf16(rng, (B, C, sp)), O.randn_bf16(rng, C, std=0.5)
    dx, db = dev(x), dev(b)
    out = empty_bf16((B, C, sp))
    anima.conv_bias_add(dx, db, out, B, C, sp)
    r = _ref_conv_bias(ref, dx, db, B, C, sp)
    xi = dev(x)
    anima.conv_bias_add(xi, db, xi, B, C, sp)  # in place (causal_conv3d.cu:253)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "conv_bias_add vs reference")
    assert_bit_exact(host(xi), host(r), "conv_bias_add in place")
    if x.size <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out), O.conv_bias_add(x, b, B, C, sp), "conv_bias_add vs oracle")


@pytest.mark.parametrize("B,C,H,W", CONV_SHAPES)
def test_conv_bias_residual_add_matches_reference_chain(anima, ref, rng, B, C, H, W):
    sp = H * W
    x, b, res = O.randn_bf16(rng, (B, C, sp)), O.randn_bf16(rng, C, std=0.5), O.randn_bf16(rng, (B, C, sp))
    dx, db, dres = dev(x), dev(b), dev(res)
    out = empty_bf16((B, C, sp))
    anima.conv_bias_residual_add(dx, db, dres, out, B, C, sp)
    r = _ref_conv_bias(ref, dx, db, B, C, sp)  # vae.cpp:190 then :194
    ref.add_bf16(r.data_ptr(), dres.data_ptr(), r.data_ptr(), B * C * sp, stream_ptr())
    xi, ri = dev(x), dev(res)
    anima.conv_bias_residual_add(xi, db, dres, xi, B, C, sp)  # out aliases x
    anima.conv_bias_residual_add(dx, db, ri, ri, B, C, sp)  # out aliases the residual
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "conv_bias_residual_add vs bias + add_bf16")
    assert_bit_exact(host(xi), host(r), "conv_bias_residual_add, out = x")
    assert_bit_exact(host(ri), host(r), "conv_bias_residual_add, out = residual")
    if x.size <= ORACLE_MAX_ELEMS:
        assert_bit_exact(host(out), O.conv_bias_add(x, b, B, C, sp, residual=res), "conv_bias_residual_add vs oracle")


@pytest.mark.parametrize("B,C,H,W", CONV_SHAPES + CN_LARGE_SHAPES)
def test_conv_bias_rms_norm_channel_silu_matches_reference_chain(anima, ref, rng, B, C, H, W):
    sp = H * W
    x, b, g = O.randn_bf16(rng, (B, C, sp)), O.randn_bf16(rng, C, std=0.5), _weight(rng, C)
    dx, db, dg = dev(x), dev(b), dev(g)
    out = empty_bf16((B, C, sp))
    anima.conv_bias_rms_norm_channel_silu(dx, db, dg, out, B, C, sp, 1e-6)
    r = _ref_conv_bias(ref, dx, db, B, C, sp)  # vae.cpp:185, then :188-189
    ref.rms_norm_channel_bf16(r.data_ptr(), dg.data_ptr(), r.data_ptr(), B, C, sp, 1e-6, stream_ptr())
    ref.silu_bf16(r.data_ptr(), r.data_ptr(), B * C * sp, stream_ptr())
    xi = dev(x)
    anima.conv_bias_rms_norm_channel_silu(xi, db, dg, xi, B, C, sp, 1e-6)  # in place
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "conv_bias_rms_norm_channel_silu vs bias + rms_norm_channel + silu")
    assert_bit_exact(host(xi), host(r), "conv_bias_rms_norm_channel_silu in place")
    assert anima.wait_timeouts() == 0


PATCH_SHAPES = [(1, 16, 1, 128, 128, 1, 2, 2), (2, 4, 3, 8, 6, 1, 2, 2), (1, 3, 4, 6, 9, 2, 3, 3),
                (1, 2, 1, 5, 7, 1, 2, 2), (2, 16, 2, 16, 16, 2, 2, 2)]


@pytest.mark.parametrize("shape", PATCH_SHAPES)
def test_patchify_3d(anima, ref, rng, shape):
    B, C, T, H, W, pT, pH, pW = shape
    S, pd = (T // pT) * (H // pH) * (W // pW), C * pT * pH * pW
    x = O.randn_bf16(rng, (B, C, T, H, W))
    dx = dev(x)
    out, out_ref = torch.zeros((B, S, pd), dtype=torch.int16, device="cuda"), torch.zeros(
        (B, S, pd), dtype=torch.int16, device="cuda")
    anima.patchify_3d(dx, out, *shape)
    ref.patchify_3d_bf16(dx.data_ptr(), out_ref.data_ptr(), *shape, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "patchify_3d vs reference")
    assert_bit_exact(host(out), O.patchify_3d(x, *shape), "patchify_3d vs oracle")


@pytest.mark.parametrize("shape", PATCH_SHAPES)
def test_unpatchify_3d(anima, ref, rng, shape):
    B, C, T, H, W, pT, pH, pW = shape
    S, pd = (T // pT) * (H // pH) * (W // pW), C * pT * pH * pW
    p = O.randn_bf16(rng, (B, S, pd))
    fill = O.randn_bf16(rng, (B, C, T, H, W))  # positions outside whole patches keep this
    dp = dev(p)
    out, out_ref = dev(fill), dev(fill)
    anima.unpatchify_3d(dp, out, *shape)
    ref.unpatchify_3d_bf16(dp.data_ptr(), out_ref.data_ptr(), *shape, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "unpatchify_3d vs reference")
    assert_bit_exact(host(out), O.unpatchify_3d(p, *shape, init=fill), "unpatchify_3d vs oracle")


SAMPLER_N = [262144, 1000003, 4 * 1024 * 1024]


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("sigma_next", [0.0, 0.61])
@pytest.mark.parametrize("N", SAMPLER_N)
def test_cfg_euler_step(anima, ref, rng, N, sigma_next, offset):
    s, p, q = (O.randn_bf16(rng, N) for _ in range(3))
    ds, dp, dq = _bf_at(s, offset), _bf_at(p, offset), _bf_at(q, offset)
    args = (4.5, 0.73, sigma_next, N)
    out = _bf_at(np.zeros(N, np.uint16), offset)
    anima.cfg_euler_step(ds, dp, dq, out, *args)
    out_ref = _bf_at(np.zeros(N, np.uint16), offset)
    ref.cfg_euler_step_bf16(ds.data_ptr(), dp.data_ptr(), dq.data_ptr(), out_ref.data_ptr(), *args, stream_ptr())
    xi = _bf_at(s, offset)
    anima.cfg_euler_step(xi, dp, dq, xi, *args)  # in place (pipeline.cpp:433)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "cfg_euler_step vs reference")
    assert_bit_exact(host(xi), host(out_ref), "cfg_euler_step in place")
    if N <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.cfg_euler_step(s, p, q, 4.5, 0.73, sigma_next), "cfg_euler_step vs oracle")


@pytest.mark.parametrize("eta", [0.0, 1.0, 0.5])
@pytest.mark.parametrize("N", SAMPLER_N)
def test_cfg_euler_a_rf_step(anima, ref, rng, N, eta):
    s, p, q, r = (O.randn_bf16(rng, N) for _ in range(4))
    ds, dp, dq, dr = dev(s), dev(p), dev(q), dev(r)
    args = (3.5, 0.8, 0.55, eta, 1.0, N)
    out, out_ref = empty_bf16(N), empty_bf16(N)
    anima.cfg_euler_a_rf_step(ds, dp, dq, dr, out, *args)
    ref.cfg_euler_a_rf_step_bf16(ds.data_ptr(), dp.data_ptr(), dq.data_ptr(), dr.data_ptr(), out_ref.data_ptr(), *args,
                                 stream_ptr())
    xi = dev(s)
    anima.cfg_euler_a_rf_step(xi, dp, dq, dr, xi, *args)  # in place (pipeline.cpp:426)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "cfg_euler_a_rf_step vs reference")
    assert_bit_exact(host(xi), host(out_ref), "cfg_euler_a_rf_step in place")
    if N <= ORACLE_MAX_ELEMS:
        assert_one_ulp(host(out), O.cfg_euler_a_rf_step(s, p, q, r, 3.5, 0.8, 0.55, eta, 1.0),
                       "cfg_euler_a_rf_step vs oracle")


# (old_denoised, old_denoised_d, rand_noise, noise_coeff, denoised_d_out) as pipeline.cpp:400-418 passes them
ER_SDE_CASES = [(False, False, False, 0.0, False), (True, False, False, 0.0, True), (True, True, True, 0.3, True),
                (True, True, False, 0.0, True), (False, False, True, 0.25, False), (True, False, True, 0.2, False)]


@pytest.mark.parametrize("case", ER_SDE_CASES)
@pytest.mark.parametrize("N", [262144, 1000003])
def test_cfg_er_sde_full_step(anima, ref, rng, N, case):
    use_od, use_odd, use_rand, noise_coeff, use_ddo = case
    x, p, q, od, odd, rn = (O.randn_bf16(rng, N) for _ in range(6))
    dp, dq = dev(p), dev(q)
    dod, dodd, drn = (dev(a) if u else None for a, u in ((od, use_od), (odd, use_odd), (rn, use_rand)))
    coeffs = (4.0, 0.7, 0.93, 0.051, 1.7, 0.02, 2.3, 0.004, noise_coeff, N)
    outs = {}
    for who in ("anima", "ref"):
        dx, den = dev(x), torch.zeros(N, dtype=torch.int16, device="cuda")
        ddo = torch.zeros(N, dtype=torch.int16, device="cuda") if use_ddo else None
        if who == "anima":
            anima.cfg_er_sde_full_step(dx, dp, dq, den, dod, ddo, dodd, drn, *coeffs)
        else:
            P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
            ref.cfg_er_sde_full_step_bf16(dx.data_ptr(), dp.data_ptr(), dq.data_ptr(), den.data_ptr(), P(dod), P(ddo),
                                          P(dodd), P(drn), *coeffs, stream_ptr())
        outs[who] = (dx, den, ddo)
    torch.cuda.synchronize()
    for k, name in enumerate(("x", "denoised", "denoised_d")):
        if outs["anima"][k] is not None:
            assert_bit_exact(host(outs["anima"][k]), host(outs["ref"][k]), f"cfg_er_sde {name} vs reference")
    ox, oden, odd_o = O.cfg_er_sde_full_step(x, p, q, od if use_od else None, odd if use_odd else None,
                                            rn if use_rand else None, *coeffs[:-1], want_dd=use_ddo)
    assert_one_ulp(host(outs["anima"][0]), ox, "cfg_er_sde x vs oracle")
    assert_one_ulp(host(outs["anima"][1]), oden, "cfg_er_sde denoised vs oracle")
    if odd_o is not None:
        assert_one_ulp(host(outs["anima"][2]), odd_o, "cfg_er_sde denoised_d vs oracle")


# ---------------------------------------------------------------- random row shapes
def _random_row_shapes(n=24, seed=7):
    r = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        D = int(2 * r.integers(1, 2049))          # any even width up to 4096
        if r.random() < 0.4:
            D = int(64 * r.integers(1, 33))        # the segment widths
        N = int(r.integers(1, max(2, min(3000, (1 << 22) // D))))
        out.append((N, D))
    return out


@pytest.mark.parametrize("N,D", _random_row_shapes())
def test_row_norms_random_shapes(anima, ref, rng, N, D):
    """Every row norm against the reference kernel on a seeded sweep of (N, D)."""
    x, y = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D))
    w, g, sc, sh = _weight(rng, D), _modvec(rng, D), _modvec(rng, D), _modvec(rng, D)
    dx, dy, dw, dg, dsc, dsh = dev(x), dev(y), dev(w), dev(g), dev(sc), dev(sh)
    S = stream_ptr()
    pairs = []
    o, r_ = empty_bf16((N, D)), empty_bf16((N, D))
    anima.rms_norm(dx, dw, o, N, D, 1e-6)
    ref.rms_norm_bf16(dx.data_ptr(), dw.data_ptr(), r_.data_ptr(), N, D, 1e-6, S)
    pairs.append(("rms_norm", o, r_, None, None))

    def ref_ln(r):
        ref.layer_norm_bf16(dx.data_ptr(), r.data_ptr(), N, D, 1e-6, S)

    def ref_ada(r):
        ref.adaln_layernorm_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), r.data_ptr(), N, D, 1e-6, S)

    hid = empty_bf16((N, D))

    def ref_resgate(r, hidden=None):  # the hidden state is updated in place: start from x each run
        if hidden is None:
            hidden = hid
            hidden.copy_(dx)
        ref.residual_gate_adaln_bf16(hidden.data_ptr(), dy.data_ptr(), dg.data_ptr(), dsc.data_ptr(), dsh.data_ptr(),
                                     r.data_ptr(), N, D, 1e-6, S)

    o, r_ = empty_bf16((N, D)), empty_bf16((N, D))
    anima.layer_norm(dx, o, N, D, 1e-6)
    ref_ln(r_)
    pairs.append(("layer_norm", o, r_, lambda: O.layer_norm(x, N, D), fresh_run(ref_ln, (N, D))))
    o, r_ = empty_bf16((N, D)), empty_bf16((N, D))
    anima.adaln_layernorm(dx, dsc, dsh, o, N, D, 1e-6)
    ref_ada(r_)
    pairs.append(("adaln_layernorm", o, r_, lambda: O.adaln_layernorm(x, sc, sh, N, D), fresh_run(ref_ada, (N, D))))
    h, hr = dev(x), dev(x)
    o, r_ = empty_bf16((N, D)), empty_bf16((N, D))
    anima.residual_gate_adaln(h, dy, dg, dsc, dsh, o, N, D, 1e-6)
    ref_resgate(r_, hr)
    pairs += [("residual_gate_adaln hidden", h, hr, None, None),
              ("residual_gate_adaln normed", o, r_, lambda: O.residual_gate_adaln(x, y, g, sc, sh, N, D)[1],
               fresh_run(ref_resgate, (N, D)))]
    torch.cuda.synchronize()
    for name, got, want, oracle_fn, rerun in pairs:  # layer_norm.cu's kernels: see assert_bit_exact_or_reference_race
        if oracle_fn is None:
            assert_bit_exact(host(got), host(want), f"{name} [{N}, {D}] vs reference")
        else:
            assert_bit_exact_or_reference_race(host(got), host(want), oracle_fn, f"{name} [{N}, {D}] vs reference",
                                               rerun)


# ---------------------------------------------------------------- conversions, VAE upsample
@pytest.mark.parametrize("N", [1 << 20, 1001, 2, 1])
def test_f32_bf16_conversions(anima, ref, rng, N):
    """elementwise.cu:311-352 over floor(N/2) pairs (an odd last element stays as it was), with
    zeros, subnormals, Inf and NaN among the inputs."""
    x = (rng.standard_normal(N) * 100).astype(np.float32)
    special = np.array([0.0, -0.0, 1e-40, -1e-45, np.inf, -np.inf, np.nan, 3.0e38], np.float32)
    x[: min(N, special.size)] = special[: min(N, special.size)]
    dx = torch.from_numpy(x).cuda()
    b, b_ref = torch.full((N,), 7, dtype=torch.int16, device="cuda"), torch.full((N,), 7, dtype=torch.int16, device="cuda")
    anima.f32_to_bf16(dx, b, N)
    ref.f32_to_bf16(dx.data_ptr(), b_ref.data_ptr(), N, stream_ptr())
    f, f_ref = torch.full((N,), 5.0, device="cuda"), torch.full((N,), 5.0, device="cuda")
    anima.bf16_to_f32(b_ref, f, N)
    ref.bf16_to_f32(b_ref.data_ptr(), f_ref.data_ptr(), N, stream_ptr())
    torch.cuda.synchronize()
    assert host(b).tobytes() == host(b_ref).tobytes(), "f32_to_bf16 vs reference"
    assert f.cpu().numpy().tobytes() == f_ref.cpu().numpy().tobytes(), "bf16_to_f32 vs reference"


def test_f32_to_bf16_unaligned(anima, rng):
    """A 4-byte-offset fp32 input (scalar path) against the oracle; the reference's float2 loads
    would be misaligned there, so it is not run."""
    N = 4098
    x = (rng.standard_normal(N + 1) * 10).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    out = torch.zeros(N, dtype=torch.int16, device="cuda")
    anima.f32_to_bf16(dx[1:], out, N)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), O.f32_to_bf16(x[1:]), "f32_to_bf16 (unaligned) vs oracle")


@pytest.mark.parametrize("B,C,H,W", [(1, 512, 64, 64), (2, 3, 5, 7), (1, 4, 5, 8), (1, 1, 1, 1)])
def test_nearest_upsample_2x(anima, ref, rng, B, C, H, W):
    x = O.randn_bf16(rng, (B, C, H, W))
    dx = dev(x)
    out, out_ref = empty_bf16((B, C, 2 * H, 2 * W)), empty_bf16((B, C, 2 * H, 2 * W))
    anima.nearest_upsample_2x(dx, out, B, C, H, W)
    ref.nearest_upsample_2x_bf16(dx.data_ptr(), out_ref.data_ptr(), B, C, H, W, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "nearest_upsample_2x vs reference")
    assert_bit_exact(host(out), O.nearest_upsample_2x(x, B, C, H, W), "nearest_upsample_2x vs oracle")


@pytest.mark.parametrize("N", [1 << 20, 4097, 9, 2])
def test_scale(anima, ref, rng, N):
    """elementwise.cu:97-122 (pipeline.cpp:519: the initial noise times sigma_0)."""
    x = O.randn_bf16(rng, N, std=2.0)
    dx = dev(x)
    out, out_ref = dev(np.full(N, 3, np.uint16)), dev(np.full(N, 3, np.uint16))
    anima.scale(dx, out, 14.614642, N)
    ref.scale_bf16(dx.data_ptr(), out_ref.data_ptr(), 14.614642, N, stream_ptr())
    xi = dev(x)
    anima.scale(xi, xi, 14.614642, N)  # in place, as pipeline.cpp:519
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "scale vs reference")
    assert_bit_exact(host(xi)[: N // 2 * 2], host(out_ref)[: N // 2 * 2], "scale in place")
