"""The benchmark's CPU baseline (oracle/hostloop.c, a plain host loop) computes the same ops
as the reference: checked against the CPU restatement (oracle.c) on small inputs. Its sums
run in row order instead of the reference kernels' tree order, so a few elements may differ
by a bf16 ulp or two; the bar is <= 2 ulp (with the comparator's small-value floor) on every
element and bit-equality on most."""
import numpy as np
import pytest

import hostloop
import oracle as O


@pytest.fixture(scope="module")
def L():
    lib = hostloop.load()
    lib.hostloop_set_threads(2)
    return lib


def _close(got, want, exact_frac=0.97):
    got, want = got.reshape(-1), want.reshape(-1)
    d = np.abs(O.bf16_to_f32(got).astype(np.float64) - O.bf16_to_f32(want).astype(np.float64))
    tol = 2 * np.maximum(O.bf16_ulp(O.bf16_to_f32(want)), 2.0 ** -12 / 128)
    assert (d <= tol).all(), f"{int((d > tol).sum())} elements beyond 2 ulp"
    assert (got == want).mean() >= exact_frac


A = lambda a: a.ctypes.data  # noqa: E731


def test_hostloop_row_norms(L):
    rng = np.random.default_rng(3)
    N, D = 12, 2048
    x, y = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D))
    sc, sh, g = (O.randn_bf16(rng, D, std=0.1) for _ in range(3))
    out = np.empty_like(x)
    L.hostloop_adaln_layernorm(A(x), A(sc), A(sh), A(out), N, D, np.float32(1e-6))
    _close(out, O.adaln_layernorm(x, sc, sh, N, D))
    h = x.copy()
    L.hostloop_residual_gate_adaln(A(h), A(y), A(g), A(sc), A(sh), A(out), N, D, np.float32(1e-6))
    wh, wn = O.residual_gate_adaln(x, y, g, sc, sh, N, D)
    _close(h, wh, exact_frac=1.0)
    _close(out, wn)
    q = O.randn_bf16(rng, (N * 16, 128))
    w = O.randn_bf16(rng, 128, mean=1.0, std=0.02)
    oq = np.empty_like(q)
    L.hostloop_rms_norm(A(q), A(w), A(oq), N * 16, 128, np.float32(1e-6))
    _close(oq, O.rms_norm(q, w, N * 16, 128))


def test_hostloop_elementwise_and_rope(L):
    rng = np.random.default_rng(4)
    B, pe, H, HD = 1, (1, 4, 4), 16, 128
    S = pe[0] * pe[1] * pe[2]
    x = O.randn_bf16(rng, (B * S, H * HD))
    ct, st = O.cosmos_rope_tables(*pe, HD=HD)
    xr = x.copy()
    L.hostloop_rope_cosmos(A(xr), A(ct), A(st), B, S, H, HD)
    _close(xr, O.rope_cosmos_strided(x, ct, st, B, S, H, HD), exact_frac=0.9)
    f = O.randn_bf16(rng, 1 << 14)
    of = np.empty_like(f)
    L.hostloop_gelu_tanh(A(f), A(of), f.size)
    _close(of, O.gelu_tanh(f), exact_frac=0.99)
    a, b = O.randn_bf16(rng, 4096), O.randn_bf16(rng, 4096)
    oa = np.empty_like(a)
    L.hostloop_add(A(a), A(b), A(oa), a.size)
    _close(oa, O.add(a, b), exact_frac=1.0)
    M, D = 8, 512
    xm, ym, gm = O.randn_bf16(rng, (M, D)), O.randn_bf16(rng, (M, D)), O.randn_bf16(rng, D, std=0.1)
    om = np.empty_like(xm)
    L.hostloop_residual_gate_bcast(A(xm), A(ym), A(gm), A(om), M, D)
    _close(om, O.residual_gate_bcast(xm, ym, gm, M, D))
