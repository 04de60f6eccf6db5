"""Parity at BASELINE.json's own configurations, full size: every row kernel at the DiT's
8192 rows (config 2: 4096 tokens x CFG 2) and 18432 rows (config 5: 9216 tokens x CFG 2),
Cosmos RoPE on config 5's (1, 96, 96) grid, and the VAE channel RMSNorm, alone and fused with
SiLU, at config 4's four NCHW shapes. Each is checked bit for bit against the reference's
own kernels run on the same device buffers (the CPU restatement is too slow at these sizes;
the smaller cases of test_gpu_parity.py pin both against it). Inputs are generated on the
device: N(0,1) activations, N(0,0.1) modulation vectors, 1+N(0,0.02) weights."""
import pytest
import torch

import oracle as O
from gpu_util import assert_bit_exact, assert_bit_exact_or_reference_race, empty_bf16, fresh_run, host, stream_ptr

pytestmark = pytest.mark.gpu


def _randn(shape, seed, mean=0.0, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = torch.randn(shape, generator=g, device="cuda") * std + mean
    return t.to(torch.bfloat16).view(torch.int16)


ROWS = [8192, 18432]


@pytest.mark.parametrize("N", ROWS)
def test_row_norms_at_dit_rows(anima, ref, N):
    D = 2048
    x, y = _randn((N, D), 1), _randn((N, D), 2)
    sc, sh, g = _randn(D, 3, std=0.1), _randn(D, 4, std=0.1), _randn(D, 5, std=0.1)
    w = _randn(D, 6, mean=1.0, std=0.02)
    out, out_ref = empty_bf16((N, D)), empty_bf16((N, D))
    P = lambda t: t.data_ptr()  # noqa: E731
    xs = host(x)
    hx = lambda: host(x)  # noqa: E731

    anima.adaln_layernorm(x, sc, sh, out, N, D, 1e-6)
    ref.adaln_layernorm_bf16(P(x), P(sc), P(sh), P(out_ref), N, D, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact_or_reference_race(
        host(out), host(out_ref), lambda: O.adaln_layernorm(xs, host(sc), host(sh), N, D), "adaln_layernorm",
        fresh_run(lambda r: ref.adaln_layernorm_bf16(P(x), P(sc), P(sh), P(r), N, D, 1e-6, stream_ptr()), (N, D)))

    anima.layer_norm(x, out, N, D, 1e-6)
    ref.layer_norm_bf16(P(x), P(out_ref), N, D, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact_or_reference_race(
        host(out), host(out_ref), lambda: O.layer_norm(xs, N, D), "layer_norm",
        fresh_run(lambda r: ref.layer_norm_bf16(P(x), P(r), N, D, 1e-6, stream_ptr()), (N, D)))

    anima.rms_norm(x, w, out, N, D, 1e-6)
    ref.rms_norm_bf16(P(x), P(w), P(out_ref), N, D, 1e-6, stream_ptr())
    # the per-head QK norm on the same tensor viewed as [N*16, 128] rows, in place
    q, q_ref = x.clone(), x.clone()
    w128 = w[:128].contiguous()
    anima.rms_norm(q, w128, q, N * 16, 128, 1e-6)
    ref.rms_norm_bf16(P(q_ref), P(w128), P(q_ref), N * 16, 128, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), "rms_norm D=2048")
    assert_bit_exact(host(q), host(q_ref), "rms_norm D=128 (QK norm) in place")

    h, h_ref = x.clone(), x.clone()
    anima.residual_gate_adaln(h, y, g, sc, sh, out, N, D, 1e-6)
    ref.residual_gate_adaln_bf16(P(h_ref), P(y), P(g), P(sc), P(sh), P(out_ref), N, D, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(h), host(h_ref), "residual_gate_adaln hidden")
    assert_bit_exact_or_reference_race(
        host(out), host(out_ref), lambda: O.residual_gate_adaln(hx(), host(y), host(g), host(sc), host(sh), N, D)[1],
        "residual_gate_adaln normed",
        fresh_run(lambda r, hid=h_ref: (hid.copy_(x), ref.residual_gate_adaln_bf16(  # hidden from x each run
            P(hid), P(y), P(g), P(sc), P(sh), P(r), N, D, 1e-6, stream_ptr())), (N, D)))


def test_rope_cosmos_cfg5_grid(anima, ref):
    """Config 5: 1536x1536 image -> (1, 96, 96) patch grid, 9216 tokens x CFG 2."""
    pe, B, H, HD = (1, 96, 96), 2, 16, 128
    S = pe[0] * pe[1] * pe[2]
    cos_t, sin_t = O.cosmos_rope_tables(*pe, HD=HD)
    dc = torch.from_numpy(cos_t.view("int16")).cuda()
    ds = torch.from_numpy(sin_t.view("int16")).cuda()
    x = _randn((B * S, H * HD), 7)
    r = x.clone()
    anima.rope_cosmos_strided(x, dc, ds, B, S, H, HD)
    ref.rope_cosmos_strided_bf16(r.data_ptr(), dc.data_ptr(), ds.data_ptr(), B, S, H, HD, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(x), host(r), "rope_cosmos_strided at (1, 96, 96)")


@pytest.mark.parametrize("C,HW", [(512, 128), (512, 256), (256, 512), (128, 1024)])
def test_channel_norm_at_vae_shapes(anima, ref, C, HW):
    """Config 4: the VAE decoder's channel RMSNorm (vae.cpp:148) and its fused SiLU
    (vae.cpp:184) against the reference's rms_norm_channel_bf16 and silu_bf16."""
    sp = HW * HW
    x = _randn((1, C, sp), 8)
    gm = _randn(C, 9, mean=1.0, std=0.02)
    out, out_ref = empty_bf16((1, C, sp)), empty_bf16((1, C, sp))
    P = lambda t: t.data_ptr()  # noqa: E731
    anima.rms_norm_channel(x, gm, out, 1, C, sp, 1e-6)
    ref.rms_norm_channel_bf16(P(x), P(gm), P(out_ref), 1, C, sp, 1e-6, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), f"rms_norm_channel [{C}, {HW}^2]")
    anima.rms_norm_channel_silu(x, gm, out, 1, C, sp, 1e-6)
    ref.silu_bf16(P(out_ref), P(out_ref), C * sp, stream_ptr())
    torch.cuda.synchronize()
    assert_bit_exact(host(out), host(out_ref), f"rms_norm_channel + silu [{C}, {HW}^2]")
