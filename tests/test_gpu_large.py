"""Maximum sizes: every kernel family on a tensor of more than 2^31 elements (about 4 GB of
bf16), where any 32-bit element index would wrap. The input is a small base block tiled
along the leading dimension, so the exact output is known: each tile must equal the
kernel's own result on the base block, which the parity tests pin bit for bit to the
reference kernels. Comparisons stay on the device.
"""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import dev

pytestmark = pytest.mark.gpu

BIG = (1 << 31) + 4096  # elements per large tensor


def _tile(base, reps):
    return base.repeat(reps, *([1] * (base.dim() - 1))).contiguous()


def _same_tiles(big, base_out, reps):
    v = big.view(reps, *base_out.shape)
    return bool(torch.equal(v, base_out.unsqueeze(0).expand_as(v)))


@pytest.fixture
def free_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_gelu_silu_beyond_2g_elements(anima, rng, free_memory):
    base = dev(O.randn_bf16(rng, 1 << 20))  # 1 Mi elements, N(0,1)
    reps = -(-BIG // base.numel())
    for name in ("gelu_tanh", "silu"):
        out_base = torch.empty_like(base)
        getattr(anima, name)(base, out_base, base.numel())
        x = _tile(base, reps)
        getattr(anima, name)(x, x, x.numel())  # in place, 2^31 + 2^20 elements
        torch.cuda.synchronize()
        assert x.numel() > 2**31
        assert _same_tiles(x, out_base, reps), f"{name}: a tile beyond 2^31 elements differs"
        del x


def test_add_and_broadcast_ops_beyond_2g_elements(anima, rng, free_memory):
    D = 2048
    a, b = dev(O.randn_bf16(rng, (512, D))), dev(O.randn_bf16(rng, (512, D)))
    g = dev(O.randn_bf16(rng, D, std=0.1))
    reps = -(-BIG // a.numel())
    M = 512 * reps
    out_add, out_rg, out_ba = torch.empty_like(a), torch.empty_like(a), torch.empty_like(a)
    anima.add(a, b, out_add, a.numel())
    anima.residual_gate_bcast(a, b, g, out_rg, 512, D)
    anima.bias_add(a, g, out_ba, 512, D)
    xa, xb = _tile(a, reps), _tile(b, reps)
    o = torch.empty_like(xa)
    anima.add(xa, xb, o, xa.numel())
    torch.cuda.synchronize()
    assert _same_tiles(o, out_add, reps), "add beyond 2^31 elements"
    anima.residual_gate_bcast(xa, xb, g, o, M, D)
    torch.cuda.synchronize()
    assert _same_tiles(o, out_rg, reps), "residual_gate_bcast beyond 2^31 elements"
    anima.bias_add(xa, g, o, M, D)
    torch.cuda.synchronize()
    assert _same_tiles(o, out_ba, reps), "bias_add beyond 2^31 elements"


@pytest.mark.parametrize("D", [2048, 128])
def test_row_norms_beyond_2g_elements(anima, rng, free_memory, D):
    rows = 64
    x = dev(O.randn_bf16(rng, (rows, D)))
    sc, sh, w = (dev(O.randn_bf16(rng, D, std=0.1)) for _ in range(3))
    reps = -(-BIG // x.numel())
    N = rows * reps
    ref_rms, ref_ada = torch.empty_like(x), torch.empty_like(x)
    anima.rms_norm(x, w, ref_rms, rows, D, 1e-6)
    anima.adaln_layernorm(x, sc, sh, ref_ada, rows, D, 1e-6)
    big = _tile(x, reps)
    out = torch.empty_like(big)
    anima.rms_norm(big, w, out, N, D, 1e-6)
    torch.cuda.synchronize()
    assert _same_tiles(out, ref_rms, reps), f"rms_norm D={D} beyond 2^31 elements"
    anima.adaln_layernorm(big, sc, sh, out, N, D, 1e-6)
    torch.cuda.synchronize()
    assert _same_tiles(out, ref_ada, reps), f"adaln_layernorm D={D} beyond 2^31 elements"


def test_residual_gate_adaln_beyond_2g_elements(anima, rng, free_memory):
    rows, D = 64, 2048
    h, y = dev(O.randn_bf16(rng, (rows, D))), dev(O.randn_bf16(rng, (rows, D)))
    g, sc, sh = (dev(O.randn_bf16(rng, D, std=0.1)) for _ in range(3))
    reps = -(-((1 << 30) + 4096) // h.numel())  # two inputs and two outputs of 2^30+ elements: 8.6 GB
    ref_h, ref_n = h.clone(), torch.empty_like(h)
    anima.residual_gate_adaln(ref_h, y, g, sc, sh, ref_n, rows, D, 1e-6)
    bh, by = _tile(h, reps), _tile(y, reps)
    bn = torch.empty_like(bh)
    anima.residual_gate_adaln(bh, by, g, sc, sh, bn, rows * reps, D, 1e-6)
    torch.cuda.synchronize()
    assert _same_tiles(bh, ref_h, reps) and _same_tiles(bn, ref_n, reps), "residual_gate_adaln at 2^30+ elements"


def test_rope_cosmos_beyond_2g_elements(anima, rng, free_memory):
    S, H, HD = 64, 16, 128
    ct, st = O.cosmos_rope_tables(1, 8, 8, HD=HD)
    c, s = dev(ct), dev(st)
    x = dev(O.randn_bf16(rng, (S, H * HD)))  # one batch item
    reps = -(-BIG // x.numel())
    ref = x.clone()
    anima.rope_cosmos_strided(ref, c, s, 1, S, H, HD)
    big = _tile(x, reps)  # reps batch items, each the same sequence
    anima.rope_cosmos_strided(big, c, s, reps, S, H, HD)
    torch.cuda.synchronize()
    assert _same_tiles(big, ref, reps), "rope_cosmos_strided beyond 2^31 elements"


def test_sampler_step_beyond_2g_elements(anima, rng, free_memory):
    n = 1 << 20
    s, p, q = (dev(O.randn_bf16(rng, n)) for _ in range(3))
    reps = -(-BIG // n)
    ref = torch.empty_like(s)
    anima.cfg_euler_step(s, p, q, ref, 4.5, 0.73, 0.61, n)
    bs = _tile(s, reps)
    bp, bq = _tile(p, reps), _tile(q, reps)
    anima.cfg_euler_step(bs, bp, bq, bs, 4.5, 0.73, 0.61, bs.numel())
    torch.cuda.synchronize()
    assert _same_tiles(bs, ref, reps), "cfg_euler_step beyond 2^31 elements"


def test_conv_bias_beyond_2g_elements(anima, rng, free_memory):
    C, sp = 64, 4096
    x, b, r = dev(O.randn_bf16(rng, (C, sp))), dev(O.randn_bf16(rng, C, std=0.5)), dev(O.randn_bf16(rng, (C, sp)))
    reps = -(-BIG // x.numel())  # batch items, each the same image
    ref_add, ref_res = torch.empty_like(x), torch.empty_like(x)
    anima.conv_bias_add(x, b, ref_add, 1, C, sp)
    anima.conv_bias_residual_add(x, b, r, ref_res, 1, C, sp)
    big = _tile(x.view(1, C, sp), reps)
    anima.conv_bias_add(big, b, big, reps, C, sp)  # in place
    torch.cuda.synchronize()
    assert big.numel() > 2**31
    assert _same_tiles(big, ref_add.view(1, C, sp), reps), "conv_bias_add beyond 2^31 elements"
    del big
    big = _tile(x.view(1, C, sp), reps)
    anima.conv_bias_residual_add(big, b, _tile(r.view(1, C, sp), reps), big, reps, C, sp)
    torch.cuda.synchronize()
    assert _same_tiles(big, ref_res.view(1, C, sp), reps), "conv_bias_residual_add beyond 2^31 elements"


def test_softmax_beyond_2g_elements(anima, rng, free_memory):
    N, D = 64, 512
    x = dev(O.randn_bf16(rng, (N, D), std=3.0))
    reps = -(-BIG // x.numel())
    ref = torch.empty_like(x)
    anima.softmax(x, ref, N, D)
    big = _tile(x, reps)
    anima.softmax(big, big, N * reps, D)  # in place, rows beyond 2^31 / D
    torch.cuda.synchronize()
    assert _same_tiles(big, ref, reps), "softmax beyond 2^31 elements"


def test_head_transpose_beyond_2g_elements(anima, rng, free_memory):
    """[B*S, H*HD] -> [B, H, S, HD] with B*H*S*HD > 2^31: batch b of the result must be the
    transpose of batch b of the input (all batches equal here)."""
    S, H, HD = 64, 16, 128
    x = dev(O.randn_bf16(rng, (S, H * HD)))
    reps = -(-BIG // x.numel())
    ref = torch.empty((1, H, S, HD), dtype=x.dtype, device=x.device)
    anima.head_transpose_batched(x, ref, 1, H, S, HD)
    big = _tile(x, reps)
    out = torch.empty((reps, H, S, HD), dtype=x.dtype, device=x.device)
    anima.head_transpose_batched(big, out, reps, H, S, HD)
    torch.cuda.synchronize()
    assert _same_tiles(out, ref, reps), "head_transpose_batched beyond 2^31 elements"
