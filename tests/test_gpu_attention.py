"""Parity of the attention glue (head transposes, GQA expansion, causal mask, softmax) with
the reference's own kernels (transpose.cu, gemma_ops.cu, softmax.cu), compiled unchanged for
sm_100a, and with the CPU restatement. Shapes: the Qwen3 encoder's (16 q / 8 kv heads of 128
at seq 512), the adapter's, and widths that take the scalar paths, rows longer than the
reference's 1024-thread CTA, and short rows that pack several per warp.
"""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bit_exact, assert_one_ulp, dev, empty_bf16, host, stream_ptr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,H,S,HD", [(1, 16, 512, 128), (1, 8, 512, 128), (2, 4, 7, 64), (1, 3, 5, 6), (3, 2, 9, 20)])
def test_head_transpose_roundtrip(anima, ref, rng, B, H, S, HD):
    x = O.randn_bf16(rng, (B * S, H * HD))
    dx = dev(x)
    heads, heads_ref = empty_bf16((B, H, S, HD)), empty_bf16((B, H, S, HD))
    back, back_ref = empty_bf16((B * S, H * HD)), empty_bf16((B * S, H * HD))
    if B == 1:  # qwen3.cpp:164-166 and :226
        anima.head_transpose(dx, heads, H, S, HD)
        ref.head_transpose_bf16(dx.data_ptr(), heads_ref.data_ptr(), H, S, HD, stream_ptr())
        anima.head_untranspose(heads, back, H, S, HD)
        ref.head_untranspose_bf16(heads_ref.data_ptr(), back_ref.data_ptr(), H, S, HD, stream_ptr())
    else:
        anima.head_transpose_batched(dx, heads, B, H, S, HD)
        ref.head_transpose_batched_bf16(dx.data_ptr(), heads_ref.data_ptr(), B, H, S, HD, stream_ptr())
        anima.head_untranspose_batched(heads, back, B, H, S, HD)
        ref.head_untranspose_batched_bf16(heads_ref.data_ptr(), back_ref.data_ptr(), B, H, S, HD, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(heads), host(heads_ref), "head transpose vs reference")
    assert_bit_exact(host(back), host(back_ref), "head untranspose vs reference")
    assert_bit_exact(host(back), x, "untranspose(transpose(x)) == x")
    assert_bit_exact(host(heads), O.head_transpose(x, B, H, S, HD), "head transpose vs oracle")


@pytest.mark.parametrize("B,KVH,QH,T,D", [(1, 8, 16, 512, 128), (2, 2, 6, 5, 12), (1, 1, 4, 3, 7)])
def test_expand_kv(anima, ref, rng, B, KVH, QH, T, D):
    kv = O.randn_bf16(rng, (B, KVH, T, D))
    dkv = dev(kv)
    out, out_ref = empty_bf16((B, QH, T, D)), empty_bf16((B, QH, T, D))
    anima.expand_kv(dkv, out, B, KVH, QH, T, D)  # qwen3.cpp:183-184
    ref.expand_kv_bf16(dkv.data_ptr(), out_ref.data_ptr(), B, KVH, QH, T, D, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "expand_kv vs reference")
    assert_bit_exact(host(out), O.expand_kv(kv, B, KVH, QH, T, D), "expand_kv vs oracle")


@pytest.mark.parametrize("H,T", [(16, 512), (3, 37), (2, 8), (1, 1)])
def test_causal_mask(anima, ref, rng, H, T):
    s = O.randn_bf16(rng, (H, T, T))
    mine, theirs = dev(s), dev(s)
    anima.causal_mask(mine, H, T)  # qwen3.cpp:205, in place
    ref.causal_mask_bf16(theirs.data_ptr(), H, T, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(mine), host(theirs), "causal_mask vs reference")
    assert_bit_exact(host(mine), O.causal_mask(s, H, T), "causal_mask vs oracle")


SOFTMAX_SHAPES = [(16 * 512, 512), (64, 1024), (33, 100), (5, 8), (3, 1), (7, 1030), (4, 3000), (40, 72), (9, 257)]


@pytest.mark.parametrize("N,D", SOFTMAX_SHAPES)
def test_softmax(anima, ref, rng, N, D):
    x = O.randn_bf16(rng, (N, D), std=3.0)
    dx = dev(x)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.softmax(dx, out, N, D)
    ref.softmax_bf16(dx.data_ptr(), out_ref.data_ptr(), N, D, stream_ptr())
    xi = dev(x)
    anima.softmax(xi, xi, N, D)  # in place (qwen3.cpp:208)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "softmax vs reference")
    assert_bit_exact(host(xi), host(out_ref), "softmax in place")
    if N * D <= 1 << 20:
        assert_one_ulp(host(out), O.softmax(x, N, D), "softmax vs oracle")


def test_softmax_unaligned_rows(anima, ref, rng):
    """A 2-byte-offset base (scalar path) gives the same bits."""
    N, D = 12, 512
    x = O.randn_bf16(rng, (N * D + 1,))
    dx = dev(x)
    out = empty_bf16((N * D + 1,))
    out_ref = empty_bf16((N * D,))
    anima.softmax(dx[1:], out[1:], N, D)
    ref.softmax_bf16(dx[1:].data_ptr(), out_ref.data_ptr(), N, D, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out[1:]), host(out_ref), "softmax on an unaligned base")


@pytest.mark.parametrize("H,T", [(16, 512), (2, 100), (3, 1030), (4, 9)])
def test_causal_softmax_matches_reference_chain(anima, ref, rng, H, T):
    s = O.randn_bf16(rng, (H, T, T), std=3.0)
    ds = dev(s)
    out = empty_bf16((H, T, T))
    anima.causal_softmax(ds, out, H, T)
    r = dev(s)  # qwen3.cpp:205-208, both in place
    ref.causal_mask_bf16(r.data_ptr(), H, T, stream_ptr())
    ref.softmax_bf16(r.data_ptr(), r.data_ptr(), H * T, T, stream_ptr())
    si = dev(s)
    anima.causal_softmax(si, si, H, T)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "causal_softmax vs causal_mask + softmax")
    assert_bit_exact(host(si), host(r), "causal_softmax in place")


F32_SHAPES = [(512, 512), (7, 100), (3, 1032), (2, 4096), (1, 33), (1, 1031)]


@pytest.mark.parametrize("N,D", F32_SHAPES)
def test_softmax_f32_to_bf16(anima, ref, rng, N, D):
    """vae.cpp:262. The reference loads every row as float4s (softmax.cu:159), so it is only
    handed rows that are 16-byte aligned: D % 4 == 0, or a single row."""
    assert D % 4 == 0 or N == 1, "the reference's float4 loads would be misaligned"
    x = (rng.standard_normal((N, D)) * 4.0).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    anima.softmax_f32_to_bf16(dx, out, N, D)
    ref.softmax_f32_to_bf16(dx.data_ptr(), out_ref.data_ptr(), N, D, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "softmax_f32_to_bf16 vs reference")
    assert_one_ulp(host(out), O.softmax_f32_to_bf16(x, N, D), "softmax_f32_to_bf16 vs oracle")


@pytest.mark.parametrize("N,D", [(6, 33), (5, 1031)])
def test_softmax_f32_to_bf16_ragged_rows(anima, rng, N, D):
    """Rows that are not 16-byte aligned take the scalar loads (the reference's float4 loads
    would be misaligned there, so only the oracle checks these)."""
    x = (rng.standard_normal((N, D)) * 4.0).astype(np.float32)
    out = empty_bf16((N, D))
    anima.softmax_f32_to_bf16(torch.from_numpy(x).cuda(), out, N, D)
    torch.cuda.synchronize()
    assert_one_ulp(host(out), O.softmax_f32_to_bf16(x, N, D), "softmax_f32_to_bf16 (ragged rows) vs oracle")


@pytest.mark.parametrize("H,T,HD,weight,rope", [(16, 512, 128, True, True), (8, 512, 128, True, True),
                                                (3, 7, 128, False, True), (4, 33, 128, True, False),
                                                (4, 9, 64, True, True)])
def test_head_transpose_qk_norm_rope_matches_reference_chain(anima, ref, rng, H, T, HD, weight, rope):
    """qwen3.cpp:164-178 (rope=False: llm_adapter.cpp:169-177 without tables); HD = 64 takes
    the three-step path."""
    x = O.randn_bf16(rng, (T, H * HD))
    w = O.randn_bf16(rng, HD, mean=1.0, std=0.02)
    cs, sn = O.standard_rope_tables(T, HD, 1e6)
    dx, dw = dev(x), dev(w)
    dc, ds = torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda()
    out = empty_bf16((H, T, HD))
    anima.head_transpose_qk_norm_rope(dx, dw if weight else None, dc if rope else None, ds if rope else None,
                                      out, H, T, HD, 1e-6)
    r = empty_bf16((H, T, HD))
    s = stream_ptr()
    ref.head_transpose_bf16(dx.data_ptr(), r.data_ptr(), H, T, HD, s)
    ref.rms_norm_bf16(r.data_ptr(), dw.data_ptr() if weight else None, r.data_ptr(), H * T, HD, 1e-6, s)
    if rope:
        ref.rope_standard_bf16(r.data_ptr(), dc.data_ptr(), ds.data_ptr(), H * T, T, HD, s)
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(r), "head_transpose_qk_norm_rope vs head_transpose + rms_norm + rope_standard")
