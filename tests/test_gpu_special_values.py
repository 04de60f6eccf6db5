"""Special values inside rows: +-Inf, NaN, values whose squares overflow fp32, all-zero rows,
subnormals. Every kernel must produce what the reference's kernel produces on the same bits
(NaN compared as NaN, whatever its payload), through the statistics as well as the epilogue.
"""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import dev, empty_bf16, host, stream_ptr

pytestmark = pytest.mark.gpu


def _same(got, want, what):
    got, want = np.asarray(got).reshape(-1), np.asarray(want).reshape(-1)
    nan_g = (got & 0x7FFF) > 0x7F80
    nan_w = (want & 0x7FFF) > 0x7F80
    bad = ~((got == want) | (nan_g & nan_w))
    assert not bad.any(), f"{what}: {int(bad.sum())} of {got.size} differ (first at {int(np.nonzero(bad)[0][0])})"


def _rows(rng, N, D):
    """N rows of N(0,1) with special values planted in some of them."""
    x = O.randn_bf16(rng, (N, D))
    sp = O.f32_to_bf16(np.array([np.inf, -np.inf, np.nan, 3.0e38, -3.0e38, 0.0, -0.0, 1e-40, 2.0e19], np.float32))
    x[1, 5] = sp[0]             # +Inf
    x[2, 7] = sp[1]             # -Inf
    x[3, 0] = sp[2]             # NaN
    x[4, :] = sp[5]             # an all-zero row
    x[5, 3] = sp[3]             # its square overflows
    x[6, 1:4] = sp[8]           # 2e19: squares sum past fp32
    x[7, 9] = sp[7]             # subnormal
    x[8, ::2] = sp[6]           # negative zeros
    return x


@pytest.mark.parametrize("D", [2048, 128, 96])
def test_row_norms_with_special_values(anima, ref, rng, D):
    N = 16
    x, y = _rows(rng, N, D), O.randn_bf16(rng, (N, D))
    w = O.randn_bf16(rng, D, mean=1.0, std=0.02)
    sc, sh, g = (O.randn_bf16(rng, D, std=0.1) for _ in range(3))
    dx, dy, dw, dsc, dsh, dg = dev(x), dev(y), dev(w), dev(sc), dev(sh), dev(g)
    s = stream_ptr()

    def rms():
        r = empty_bf16((N, D))
        ref.rms_norm_bf16(dx.data_ptr(), dw.data_ptr(), r.data_ptr(), N, D, 1e-6, s)
        return [r]

    def ln():
        r = empty_bf16((N, D))
        ref.layer_norm_bf16(dx.data_ptr(), r.data_ptr(), N, D, 1e-6, s)
        return [r]

    def ada():
        r = empty_bf16((N, D))
        ref.adaln_layernorm_bf16(dx.data_ptr(), dsc.data_ptr(), dsh.data_ptr(), r.data_ptr(), N, D, 1e-6, s)
        return [r]

    def resgate():
        hr, r = dev(x), empty_bf16((N, D))
        ref.residual_gate_adaln_bf16(hr.data_ptr(), dy.data_ptr(), dg.data_ptr(), dsc.data_ptr(), dsh.data_ptr(),
                                     r.data_ptr(), N, D, 1e-6, s)
        return [hr, r]

    o1, o2, o3, o4 = (empty_bf16((N, D)) for _ in range(4))
    h = dev(x)
    anima.rms_norm(dx, dw, o1, N, D, 1e-6)
    anima.layer_norm(dx, o2, N, D, 1e-6)
    anima.adaln_layernorm(dx, dsc, dsh, o3, N, D, 1e-6)
    anima.residual_gate_adaln(h, dy, dg, dsc, dsh, o4, N, D, 1e-6)
    # layer_norm.cu's kernels can race in their own reduction helper (see
    # gpu_util.assert_bit_exact_or_reference_race): a mismatch there gets one fresh reference run
    for name, ours, run_ref, racy in (("rms_norm", [o1], rms, False), ("layer_norm", [o2], ln, True),
                                      ("adaln_layernorm", [o3], ada, True),
                                      ("residual_gate_adaln", [h, o4], resgate, True)):
        theirs = run_ref()
        torch.cuda.synchronize()
        if racy and any(not np.array_equal(host(a), host(b)) for a, b in zip(ours, theirs)):
            theirs = run_ref()
            torch.cuda.synchronize()
        for a, b in zip(ours, theirs):
            _same(host(a), host(b), f"{name} D={D}")


def test_softmax_and_channel_norm_with_special_values(anima, ref, rng):
    N, D = 16, 512
    x = _rows(rng, N, D)
    dx = dev(x)
    o, r = empty_bf16((N, D)), empty_bf16((N, D))
    anima.softmax(dx, o, N, D)
    ref.softmax_bf16(dx.data_ptr(), r.data_ptr(), N, D, stream_ptr())
    B, C, sp = 1, 16, 512  # the same values as 16 channels of 512 pixels
    gm = dev(O.randn_bf16(rng, C, mean=1.0, std=0.02))
    co, cr = empty_bf16((B, C, sp)), empty_bf16((B, C, sp))
    anima.rms_norm_channel(dx, gm, co, B, C, sp, 1e-6)
    ref.rms_norm_channel_bf16(dx.data_ptr(), gm.data_ptr(), cr.data_ptr(), B, C, sp, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    _same(host(o), host(r), "softmax")
    _same(host(co), host(cr), "rms_norm_channel")


def test_activations_and_rope_with_special_values(anima, ref, rng):
    S, H, HD = 16, 4, 128
    x = _rows(rng, S, H * HD)
    ct, st = O.cosmos_rope_tables(1, 4, 4, HD=HD)
    dc, ds = dev(ct), dev(st)
    a, b = dev(x), dev(x)
    anima.rope_cosmos_strided(a, dc, ds, 1, S, H, HD)
    ref.rope_cosmos_strided_bf16(b.data_ptr(), dc.data_ptr(), ds.data_ptr(), 1, S, H, HD, stream_ptr())
    dx = dev(x)
    g, gr = empty_bf16(x.shape), empty_bf16(x.shape)
    anima.gelu_tanh(dx, g, x.size)
    ref.gelu_tanh_bf16(dx.data_ptr(), gr.data_ptr(), x.size, stream_ptr())
    torch.cuda.synchronize()
    _same(host(a), host(b), "rope_cosmos_strided")
    _same(host(g), host(gr), "gelu_tanh")
