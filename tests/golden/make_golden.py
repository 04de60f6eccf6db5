"""Generates the golden fixtures in this directory by running the REFERENCE's own CUDA
kernels (src/kernels/*.cu compiled unchanged for sm_100a into oracle/_ref) on small
seeded inputs. Needs a GPU and oracle/_ref/libref_kernels.so; run on a B200 box:

    python tests/golden/make_golden.py --out tests/golden

Each fixture is an .npz of uint16 bf16 bit patterns (fp32 / int32 arrays where the
launcher takes them) holding the inputs and the reference outputs. The CPU test
tests/test_cpu_golden.py pins the CPU restatement in oracle/ against them.
"""
import argparse
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402  (inputs, tables and bf16 helpers only)
import refkernels  # noqa: E402


_KEEP = []  # every device tensor stays alive until exit: a temporary's block could be
            # handed to the next allocation before the kernel that reads it has run


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    t = torch.from_numpy(a).cuda()
    _KEEP.append(t)
    return t


def host(t, dtype=np.uint16):
    return t.cpu().numpy().view(dtype)


def craft_rope_standard_pin(rng):
    """Inputs on which the nine ways of contracting x1*c - x2*s and x2*c + x1*s into fmas
    give pairwise different bf16 outputs, so the reference's choice can be read off its
    result. Each pair's exact result is placed next to a bf16 rounding midpoint (solving
    for s), and only elements whose rounding depends on the contraction are kept: 400
    for each pair of choices of either product. Layout: 64 rows x 128 (64 pairs), T = 64,
    each row with its own table row."""
    import itertools

    def candidates(n, target):
        x1 = O.bf16_to_f32(O.f32_to_bf16(rng.uniform(0.5, 1.0, n).astype(np.float32)))
        x2 = O.bf16_to_f32(O.f32_to_bf16(rng.uniform(0.5, 1.0, n).astype(np.float32)))
        c = rng.uniform(0.5, 1.0, n).astype(np.float32)
        m = np.float64(0.5) + (rng.integers(0, 64, n) + 0.5) * 2.0 ** -8
        if target == 0:
            s = ((x1.astype(np.float64) * c - m) / x2).astype(np.float32)
        else:
            s = ((m - x2.astype(np.float64) * c) / x1).astype(np.float32)
        return x1, x2, c, s

    picked = []
    for target in (0, 1):
        x1, x2, c, s = candidates(1 << 20, target)
        n = x1.size
        x = np.stack([O.f32_to_bf16(x1), O.f32_to_bf16(x2)], 1)
        outs = [O.rope_standard(x, c.reshape(n, 1), s.reshape(n, 1), n, n, 2,
                                modes=(m, 0) if target == 0 else (0, m))[:, target] for m in range(3)]
        for p, q in itertools.combinations(range(3), 2):
            idx = np.nonzero(outs[p] != outs[q])[0][:400]
            picked.append(np.stack([x1[idx], x2[idx], c[idx], s[idx]], 1))
    P = np.concatenate(picked)
    fill = np.stack(candidates(64 * 64 - len(P), 0), 1)
    P = np.concatenate([P, fill])[rng.permutation(64 * 64)]
    x = np.zeros((64, 128), np.uint16)
    x[:, :64] = O.f32_to_bf16(P[:, 0]).reshape(64, 64)
    x[:, 64:] = O.f32_to_bf16(P[:, 1]).reshape(64, 64)
    return x, P[:, 2].reshape(64, 64).astype(np.float32), P[:, 3].reshape(64, 64).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    ap.add_argument("--only", nargs="*", default=None, help="write only these fixtures (names without .npz)")
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    R = refkernels.load_reference()
    s = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(20261201)
    fx = {}

    def put(name, **arrays):
        fx[name] = arrays

    # ---- row norms (layer_norm.cu, rms_norm.cu, adaln.cu, gemma_ops.cu)
    for N, D in [(8, 2048), (3, 96), (2, 4096), (16, 128)]:
        x = O.randn_bf16(rng, (N, D), mean=0.2)
        out = torch.empty((N, D), dtype=torch.int16, device="cuda")
        R.layer_norm_bf16(dev(x).data_ptr(), out.data_ptr(), N, D, 1e-6, s)
        torch.cuda.synchronize()
        put(f"layer_norm_{N}x{D}", x=x, out=host(out))
    for N, D in [(8, 2048), (4, 128), (2, 4096)]:
        x, sc, sh = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, D, std=0.1), O.randn_bf16(rng, D, std=0.1)
        out = torch.empty((N, D), dtype=torch.int16, device="cuda")
        R.adaln_layernorm_bf16(dev(x).data_ptr(), dev(sc).data_ptr(), dev(sh).data_ptr(), out.data_ptr(), N, D,
                               1e-6, s)
        torch.cuda.synchronize()
        put(f"adaln_layernorm_{N}x{D}", x=x, scale=sc, shift=sh, out=host(out))
    for N, D in [(8, 2048), (2, 4096), (4, 96)]:
        x, y = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D))
        g, sc, sh = (O.randn_bf16(rng, D, std=0.1) for _ in range(3))
        h = dev(x)
        out = torch.empty((N, D), dtype=torch.int16, device="cuda")
        R.residual_gate_adaln_bf16(h.data_ptr(), dev(y).data_ptr(), dev(g).data_ptr(), dev(sc).data_ptr(),
                                   dev(sh).data_ptr(), out.data_ptr(), N, D, 1e-6, s)
        torch.cuda.synchronize()
        put(f"residual_gate_adaln_{N}x{D}", x=x, y=y, gate=g, scale=sc, shift=sh, hidden=host(h), normed=host(out))
    for N, D, weighted in [(64, 128, True), (8, 1024, True), (4, 2048, False), (2, 4096, True), (3, 64, True)]:
        x, w = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, D, mean=1.0, std=0.02)
        out = torch.empty((N, D), dtype=torch.int16, device="cuda")
        dw = dev(w) if weighted else None
        R.rms_norm_bf16(dev(x).data_ptr(), dw.data_ptr() if weighted else None, out.data_ptr(), N, D, 1e-6, s)
        torch.cuda.synchronize()
        put(f"rms_norm_{N}x{D}_{'w' if weighted else 'nw'}", x=x, weight=w if weighted else np.zeros(0, np.uint16),
            out=host(out))
    N, D = 4, 2048
    x, sc, sh = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, (N, D), std=0.1), O.randn_bf16(rng, (N, D), std=0.1)
    out = torch.empty((N, D), dtype=torch.int16, device="cuda")
    R.adaln_rms_norm_bf16(dev(x).data_ptr(), dev(sc).data_ptr(), dev(sh).data_ptr(), out.data_ptr(), N, D, 1e-6, s)
    torch.cuda.synchronize()
    put("adaln_rms_norm_4x2048", x=x, scale=sc, shift=sh, out=host(out))
    N, D = 4, 1024
    x, w = O.randn_bf16(rng, (N, D)), O.randn_bf16(rng, D, std=0.1)
    out = torch.empty((N, D), dtype=torch.int16, device="cuda")
    R.gemma_rms_norm_bf16(dev(x).data_ptr(), dev(w).data_ptr(), out.data_ptr(), N, D, 1e-6, s)
    torch.cuda.synchronize()
    put("gemma_rms_norm_4x1024", x=x, weight=w, out=host(out))

    # ---- activations and elementwise (gelu.cu, silu.cu, elementwise.cu, gemma_ops.cu)
    ext = O.f32_to_bf16(np.array([0, -0.0, 1e-30, 3, -3, 8, -8, 20, -20, 88, -88, 3e38, -3e38], np.float32))
    for op in ("gelu_tanh", "silu"):
        x = np.concatenate([O.randn_bf16(rng, 8190, std=3.0), ext])
        out = torch.zeros(x.size, dtype=torch.int16, device="cuda")
        getattr(R, op + "_bf16")(dev(x).data_ptr(), out.data_ptr(), x.size, s)
        M, Db = 16, 96
        xb, b = O.randn_bf16(rng, (M, Db), std=2.0), O.randn_bf16(rng, Db, std=0.5)
        outb = torch.zeros(M * Db, dtype=torch.int16, device="cuda")
        getattr(R, op + "_bias_bf16")(dev(xb).data_ptr(), dev(b).data_ptr(), outb.data_ptr(), M * Db, Db, s)
        torch.cuda.synchronize()
        put(op, x=x, out=host(out))
        put(op + "_bias", x=xb, bias=b, out=host(outb))
    for op in ("add", "mul", "gated_gelu"):
        a, b = O.randn_bf16(rng, 4096, std=2.0), O.randn_bf16(rng, 4096)
        out = torch.zeros(4096, dtype=torch.int16, device="cuda")
        getattr(R, op + "_bf16")(dev(a).data_ptr(), dev(b).data_ptr(), out.data_ptr(), 4096, s)
        torch.cuda.synchronize()
        put(op, a=a, b=b, out=host(out))
    M, D = 8, 2048
    x, sc, sh, y = (O.randn_bf16(rng, (M, D)), O.randn_bf16(rng, D, std=0.1), O.randn_bf16(rng, D, std=0.1),
                    O.randn_bf16(rng, (M, D)))
    out = torch.empty((M, D), dtype=torch.int16, device="cuda")
    R.scale_shift_bcast_bf16(dev(x).data_ptr(), dev(sc).data_ptr(), dev(sh).data_ptr(), out.data_ptr(), M, D, s)
    out2 = torch.empty((M, D), dtype=torch.int16, device="cuda")
    R.residual_gate_bcast_bf16(dev(x).data_ptr(), dev(y).data_ptr(), dev(sc).data_ptr(), out2.data_ptr(), M, D, s)
    torch.cuda.synchronize()
    put("scale_shift_bcast", x=x, scale=sc, shift=sh, out=host(out))
    put("residual_gate_bcast", x=x, y=y, gate=sc, out=host(out2))

    # ---- RoPE (rope.cu, gemma_ops.cu); tables from the restated host builders
    B, pe, H, HD = 2, (1, 4, 4), 4, 128
    S = 16
    ct, st = O.cosmos_rope_tables(*pe, HD=HD)
    x = O.randn_bf16(rng, (B * S, H * HD))
    xd = dev(x)
    R.rope_cosmos_strided_bf16(xd.data_ptr(), dev(ct).data_ptr(), dev(st).data_ptr(), B, S, H, HD, s)
    torch.cuda.synchronize()
    put("rope_cosmos_strided", x=x, cos=ct, sin=st, out=host(xd), shape=np.array([B, S, H, HD], np.int32))
    for heads, T, HD, theta in [(4, 16, 128, 1e6), (2, 9, 64, 1e4)]:
        ct, st = O.standard_rope_tables(T, HD, theta)
        x = O.randn_bf16(rng, (heads * T, HD))
        xd = dev(x)
        R.rope_standard_bf16(xd.data_ptr(), dev(ct).data_ptr(),
                             dev(st).data_ptr(), heads * T, T, HD, s)
        torch.cuda.synchronize()
        put(f"rope_standard_{HD}", x=x, cos=ct, sin=st, out=host(xd), shape=np.array([heads * T, T, HD], np.int32))

    x, ct, st = craft_rope_standard_pin(rng)
    xd = dev(x)
    R.rope_standard_bf16(xd.data_ptr(), dev(ct).data_ptr(), dev(st).data_ptr(), 64, 64, 128, s)
    torch.cuda.synchronize()
    put("rope_standard_pin", x=x, cos=ct, sin=st, out=host(xd), shape=np.array([64, 64, 128], np.int32))

    # ---- gather and VAE channel norm (gemma_ops.cu, vae_kernels.cu)
    V, D, T = 1000, 64, 32
    table, ids = O.randn_bf16(rng, (V, D), std=0.02), rng.integers(0, V, T, dtype=np.int32)
    out = torch.empty((T, D), dtype=torch.int16, device="cuda")
    R.embedding_lookup_bf16(dev(table).data_ptr(), dev(ids).data_ptr(), out.data_ptr(), T, D, s)
    torch.cuda.synchronize()
    put("embedding_lookup", table=table, ids=ids, out=host(out))
    for B, C, sp in [(1, 96, 64), (2, 32, 40)]:
        x, g = O.randn_bf16(rng, (B, C, sp)), O.randn_bf16(rng, C, mean=1.0, std=0.02)
        out = torch.empty((B, C, sp), dtype=torch.int16, device="cuda")
        R.rms_norm_channel_bf16(dev(x).data_ptr(), dev(g).data_ptr(), out.data_ptr(), B, C, sp, 1e-6, s)
        torch.cuda.synchronize()
        put(f"rms_norm_channel_{B}x{C}x{sp}", x=x, gamma=g, out=host(out))

    # ---- broadcast bias add (elementwise.cu:184-213); its own seed, so earlier fixtures
    # do not change when it was added
    rng2 = np.random.default_rng(20261)
    M, D = 8, 2048
    x, b = O.randn_bf16(rng2, (M, D)), O.randn_bf16(rng2, D)
    out = torch.empty((M, D), dtype=torch.int16, device="cuda")
    R.bias_add_bf16(dev(x).data_ptr(), dev(b).data_ptr(), out.data_ptr(), M, D, s)
    torch.cuda.synchronize()
    put("bias_add", x=x, bias=b, out=host(out))

    # ---- sampler steps and latent I/O (transpose.cu, vae_kernels.cu); own seed as well
    rng3 = np.random.default_rng(20262)
    N = 4096
    smp, pos, neg, rn, od, odd = (O.randn_bf16(rng3, N) for _ in range(6))
    for name, sn in (("cfg_euler_step", 0.61), ("cfg_euler_step_last", 0.0)):
        out = torch.zeros(N, dtype=torch.int16, device="cuda")
        R.cfg_euler_step_bf16(dev(smp).data_ptr(), dev(pos).data_ptr(), dev(neg).data_ptr(), out.data_ptr(), 4.5,
                              0.73, sn, N, s)
        torch.cuda.synchronize()
        put(name, sample=smp, pos=pos, neg=neg, out=host(out), params=np.array([4.5, 0.73, sn], np.float32))
    out = torch.zeros(N, dtype=torch.int16, device="cuda")
    R.cfg_euler_a_rf_step_bf16(dev(smp).data_ptr(), dev(pos).data_ptr(), dev(neg).data_ptr(), dev(rn).data_ptr(),
                               out.data_ptr(), 3.5, 0.8, 0.55, 1.0, 1.0, N, s)
    torch.cuda.synchronize()
    put("cfg_euler_a_rf_step", sample=smp, pos=pos, neg=neg, rand=rn, out=host(out),
        params=np.array([3.5, 0.8, 0.55, 1.0, 1.0], np.float32))
    coeffs = [4.0, 0.7, 0.93, 0.051, 1.7, 0.02, 2.3, 0.004, 0.3]
    x, den, dd = dev(smp), torch.zeros(N, dtype=torch.int16, device="cuda"), torch.zeros(N, dtype=torch.int16,
                                                                                         device="cuda")
    R.cfg_er_sde_full_step_bf16(x.data_ptr(), dev(pos).data_ptr(), dev(neg).data_ptr(), den.data_ptr(),
                                dev(od).data_ptr(), dd.data_ptr(), dev(odd).data_ptr(), dev(rn).data_ptr(), *coeffs,
                                N, s)
    torch.cuda.synchronize()
    put("cfg_er_sde_full_step", x=smp, pos=pos, neg=neg, old_den=od, old_dd=odd, rand=rn, x_out=host(x),
        den_out=host(den), dd_out=host(dd), params=np.array(coeffs, np.float32))
    shape = (2, 4, 3, 8, 6, 1, 2, 2)
    B_, C_, T_, H_, W_, pT_, pH_, pW_ = shape
    vol = O.randn_bf16(rng3, (B_, C_, T_, H_, W_))
    S_, pd_ = (T_ // pT_) * (H_ // pH_) * (W_ // pW_), C_ * pT_ * pH_ * pW_
    pout = torch.zeros((B_, S_, pd_), dtype=torch.int16, device="cuda")
    R.patchify_3d_bf16(dev(vol).data_ptr(), pout.data_ptr(), *shape, s)
    pin = O.randn_bf16(rng3, (B_, S_, pd_))
    uout = torch.zeros((B_, C_, T_, H_, W_), dtype=torch.int16, device="cuda")
    R.unpatchify_3d_bf16(dev(pin).data_ptr(), uout.data_ptr(), *shape, s)
    torch.cuda.synchronize()
    put("patchify_3d", x=vol, out=host(pout), shape=np.array(shape, np.int32))
    put("unpatchify_3d", x=pin, out=host(uout), shape=np.array(shape, np.int32))
    cx = O.randn_bf16(rng3, (2, 16, 96))
    csc, csh = O.randn_bf16(rng3, 16, mean=1.0, std=0.3), O.randn_bf16(rng3, 16, std=0.5)
    cout = torch.zeros((2, 16, 96), dtype=torch.int16, device="cuda")
    R.channel_scale_shift_bf16(dev(cx).data_ptr(), dev(csc).data_ptr(), dev(csh).data_ptr(), cout.data_ptr(), 2, 16,
                               96, s)
    torch.cuda.synchronize()
    put("channel_scale_shift", x=cx, scale=csc, shift=csh, out=host(cout))

    # ---- VAE conv epilogue; own seed. The conv's bias kernel (causal_conv3d.cu:187-195) is
    # file-local to causal_conv3d_forward and computes bf16(x + bias[c]) per element, the same
    # fp32 add and RNE rounding as add_bf16 (elementwise.cu:37-53), so the fixtures come from
    # add_bf16 with the bias broadcast over each channel plane, then the reference's own chain
    # (vae.cpp:185-194): rms_norm_channel_bf16 + silu_bf16, or add_bf16 of the residual.
    rng4 = np.random.default_rng(20263)
    B, C, sp = 2, 24, 40
    x, b, res = O.randn_bf16(rng4, (B, C, sp)), O.randn_bf16(rng4, C, std=0.5), O.randn_bf16(rng4, (B, C, sp))
    g = O.randn_bf16(rng4, C, mean=1.0, std=0.02)
    n = B * C * sp
    bexp = np.ascontiguousarray(np.broadcast_to(b.reshape(1, C, 1), (B, C, sp)))
    hb = torch.zeros((B, C, sp), dtype=torch.int16, device="cuda")
    R.add_bf16(dev(x).data_ptr(), dev(bexp).data_ptr(), hb.data_ptr(), n, s)
    hr = torch.zeros((B, C, sp), dtype=torch.int16, device="cuda")
    R.add_bf16(hb.data_ptr(), dev(res).data_ptr(), hr.data_ptr(), n, s)
    hn = torch.zeros((B, C, sp), dtype=torch.int16, device="cuda")
    R.rms_norm_channel_bf16(hb.data_ptr(), dev(g).data_ptr(), hn.data_ptr(), B, C, sp, 1e-6, s)
    R.silu_bf16(hn.data_ptr(), hn.data_ptr(), n, s)
    torch.cuda.synchronize()
    put("conv_bias_add", x=x, bias=b, out=host(hb))
    put("conv_bias_residual_add", x=x, bias=b, residual=res, out=host(hr))
    put("conv_bias_rms_norm_channel_silu", x=x, bias=b, gamma=g, out=host(hn))

    # ---- pixel norm (vae_kernels.cu:15-52); own seed
    rng6 = np.random.default_rng(20265)
    px = O.randn_bf16(rng6, (2, 24, 40))
    po = torch.zeros((2, 24, 40), dtype=torch.int16, device="cuda")
    R.pixel_norm_bf16(dev(px).data_ptr(), po.data_ptr(), 2, 24, 40, 1e-6, s)
    torch.cuda.synchronize()
    put("pixel_norm", x=px, out=host(po))

    # ---- attention glue (transpose.cu, gemma_ops.cu, softmax.cu); own seed
    rng5 = np.random.default_rng(20264)
    H, T, HD = 4, 6, 16
    x = O.randn_bf16(rng5, (T, H * HD))
    th = torch.zeros((H, T, HD), dtype=torch.int16, device="cuda")
    R.head_transpose_bf16(dev(x).data_ptr(), th.data_ptr(), H, T, HD, s)
    kv = O.randn_bf16(rng5, (1, 2, T, HD))
    ek = torch.zeros((1, 6, T, HD), dtype=torch.int16, device="cuda")
    R.expand_kv_bf16(dev(kv).data_ptr(), ek.data_ptr(), 1, 2, 6, T, HD, s)
    sc = O.randn_bf16(rng5, (3, 40, 40), std=3.0)
    msk = dev(sc)
    R.causal_mask_bf16(msk.data_ptr(), 3, 40, s)
    sm = torch.zeros((3 * 40, 40), dtype=torch.int16, device="cuda")
    R.softmax_bf16(msk.data_ptr(), sm.data_ptr(), 3 * 40, 40, s)
    sx = O.randn_bf16(rng5, (4, 1500), std=3.0)
    sl = torch.zeros((4, 1500), dtype=torch.int16, device="cuda")
    R.softmax_bf16(dev(sx).data_ptr(), sl.data_ptr(), 4, 1500, s)
    fx32 = (rng5.standard_normal((8, 96)) * 4.0).astype(np.float32)
    sf = torch.zeros((8, 96), dtype=torch.int16, device="cuda")
    R.softmax_f32_to_bf16(torch.from_numpy(fx32).cuda().data_ptr(), sf.data_ptr(), 8, 96, s)
    torch.cuda.synchronize()
    put("head_transpose", x=x, out=host(th), shape=np.array([H, T, HD], np.int32))
    put("expand_kv", x=kv, out=host(ek), shape=np.array([1, 2, 6, T, HD], np.int32))
    put("causal_mask_softmax", x=sc, masked=host(msk), out=host(sm))
    put("softmax_1500", x=sx, out=host(sl))
    put("softmax_f32_to_bf16", x=fx32, out=host(sf))

    if args.only:
        fx = {k: v for k, v in fx.items() if k in args.only}
    for name, arrays in fx.items():
        np.savez_compressed(os.path.join(args.out, name + ".npz"), **arrays)
    print(f"wrote {len(fx)} fixtures to {args.out}")


if __name__ == "__main__":
    main()
