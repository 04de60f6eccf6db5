#!/usr/bin/env python
"""Benchmark of the anima.cu fused layer kernels on B200: one DiT denoising step's
elementwise/normalisation chain at BASELINE config 2 (1024x1024 image -> 4096 tokens,
CFG batch 2 -> 8192 rows x 2048 hidden, 16 heads x 128, MLP 8192, 512 text tokens,
28 blocks with fresh modulation vectors, timestep embedding).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl anima|reference]

One step = the timestep embedding + 28 x the block's chain as the reference wires it
(transformer.cpp:381-466), with the DiT FFN's GELU as a standalone op as BASELINE's chain
lists it:
    3x add (mod += temb)  adaLN-LN  QK-RMSNorm q,k  RoPE q,k  residual-gate+adaLN
    QK-RMSNorm q (cross) k (text)  residual-gate+adaLN  GELU [R,8192]  residual-gate
GEMMs and attention are not part of the chain (they stay cuBLAS/cuDNN); their outputs
(q, k, sub-layer outputs, FFN activations) are synthetic tensors resident in HBM.

--impl anima      this library through its C ABI (include/anima_b200.h)
--impl reference  the reference's own CUDA kernels (src/kernels/*.cu compiled unchanged
                  for sm_100a, oracle/_ref) through their kernels.h launchers, with the
                  reference's host-side timestep sinusoid + upload.

Prints one JSON line (rank 0). Multi-GPU runs (torchrun, one rank per GPU) replicate the
per-GPU workload (rows are independent; no collective on the data path) and report the
aggregate over ranks with the max-over-ranks device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "anima.cu_b200"))

METRIC = "fused-kernel HBM GB/s (% of B200 peak) at 4096×2048 bf16; DiT-step ms"

# ---------------------------------------------------------------- workload (cfg2)
CFG = dict(batch=2, pe=(1, 64, 64), hidden=2048, heads=16, head_dim=128, mlp=8192, text=512, blocks=28,
           ts_dim=2048, eps=1e-6)
NSETS = 4  # rotating activation buffer sets: ~1.4 GB touched per step, >> 126 MB L2
# 512x512 image -> 64x64 latent -> 32x32 patches = 1024 tokens, batch 1
CFG1 = dict(batch=1, pe=(1, 32, 32))


def chain_bytes(c=CFG):
    """Algorithmic HBM bytes of one step, per op type (each input read once, each output
    written once, broadcast vectors counted once)."""
    B, S = c["batch"], c["pe"][0] * c["pe"][1] * c["pe"][2]
    R, D, H, HD, M, T = B * S, c["hidden"], c["heads"], c["head_dim"], c["mlp"], c["text"]
    per_block = {
        "add": 3 * (3 * 2 * 3 * D),                      # mod[3D] += temb[3D], three times
        "adaln_layernorm": 4 * R * D + 4 * D,
        "rms_norm_qk128": 2 * (4 * R * H * HD + 2 * HD) + (4 * R * H * HD + 2 * HD) + (4 * B * T * H * HD + 2 * HD),
        "rope_cosmos_strided": 2 * (4 * R * H * HD + 2 * S * (HD // 2) * 2),
        "residual_gate_adaln": 2 * (8 * R * D + 6 * D),
        "gelu_tanh": 4 * R * M,
        "residual_gate_bcast": 6 * R * D + 2 * D,
    }
    launches_per_block = {"add": 3, "adaln_layernorm": 1, "rms_norm_qk128": 4, "rope_cosmos_strided": 2,
                          "residual_gate_adaln": 2, "gelu_tanh": 1, "residual_gate_bcast": 1}
    ts = 2 * c["ts_dim"] + 4 * 2 * c["ts_dim"]            # sinusoid write; RMSNorm read+weight+write
    total = c["blocks"] * sum(per_block.values()) + ts
    return total, per_block, launches_per_block


# ---------------------------------------------------------------- launchers
class AnimaOps:
    """The B200 library's C ABI, raw pointers, status checked on every call."""

    kind = "anima"

    def __init__(self):
        import anima_b200

        self.m = anima_b200
        self.L = anima_b200.lib

    def _ck(self, name, st):
        if st != 0:
            raise self.m.AnimaError(name, st, self.m.status_string(st))

    def add(self, a, b, o, n, s):
        self._ck("add", self.L.anima_add_bf16(a, b, o, n, s))

    def adaln_layernorm(self, x, sc, sh, o, N, D, eps, s):
        self._ck("adaln", self.L.anima_adaln_layernorm_bf16(x, sc, sh, o, N, D, eps, s))

    def rms_norm(self, x, w, o, N, D, eps, s):
        self._ck("rms", self.L.anima_rms_norm_bf16(x, w, o, N, D, eps, s))

    def rope_cosmos_strided(self, x, c, sn, B, S, H, HD, s):
        self._ck("rope", self.L.anima_rope_cosmos_strided_bf16(x, c, sn, B, S, H, HD, s))

    def residual_gate_adaln(self, h, y, g, sc, sh, o, N, D, eps, s):
        self._ck("resgate", self.L.anima_residual_gate_adaln_bf16(h, y, g, sc, sh, o, N, D, eps, s))

    def gelu_tanh(self, x, o, n, s):
        self._ck("gelu", self.L.anima_gelu_tanh_bf16(x, o, n, s))

    def residual_gate_bcast(self, x, y, g, o, M, D, s):
        self._ck("bcast", self.L.anima_residual_gate_bcast_bf16(x, y, g, o, M, D, s))

    def timestep(self, t, w, sin_out, normed, dim, eps, s, host_buf=None, sin_tensor=None):
        self._ck("timestep", self.L.anima_timestep_embedding_bf16(t, w, sin_out, normed, dim, eps, s))

    def call(self, name, *args):
        """Any entry point that keeps the reference launcher's argument list."""
        self._ck(name, getattr(self.L, "anima_" + name + "_bf16")(*args))

    def embedding_lookup(self, table, ids, out, T, D, vocab, s):
        self._ck("embedding", self.L.anima_embedding_lookup_bf16(table, ids, out, T, D, vocab, None, s))

    # opt-in fused entry points (no reference counterpart; the reference arm runs its chain)
    def swiglu(self, g, u, o, n, s):
        self._ck("swiglu", self.L.anima_swiglu_bf16(g, u, o, n, s))

    def rms_norm_channel_silu(self, x, gamma, o, B, C, sp, eps, s):
        self._ck("cn_silu", self.L.anima_rms_norm_channel_silu_bf16(x, gamma, o, B, C, sp, eps, s))

    def layer_norm_modulate(self, x, sc, sh, o, N, D, eps, s):
        self._ck("ln_mod", self.L.anima_layer_norm_modulate_bf16(x, sc, sh, o, N, D, eps, s))

    def causal_softmax(self, sc, o, H, T, s):
        self._ck("causal_softmax", self.L.anima_causal_softmax_bf16(sc, o, H, T, s))

    def head_qk_norm_rope(self, src, w, c, sn, dst, H, T, HD, eps, s):
        self._ck("head_qk_norm_rope", self.L.anima_head_transpose_qk_norm_rope_bf16(src, w, c, sn, dst, H, T, HD, eps, s))

    def softmax_f32_to_bf16(self, x, o, N, D, s):
        self._ck("softmax_f32", self.L.anima_softmax_f32_to_bf16(x, o, N, D, s))

    def qk_norm_rope(self, x, w, c, sn, B, S, H, HD, eps, s):
        self._ck("qk_norm_rope", self.L.anima_qk_norm_rope_bf16(x, w, c, sn, B, S, H, HD, eps, s))

    def adaln_layernorm_temb(self, x, mod, temb, gate_out, o, N, D, eps, s):
        self._ck("adaln_temb", self.L.anima_adaln_layernorm_temb_bf16(x, mod, temb, gate_out, o, N, D, eps, s))

    def residual_gate_adaln_temb(self, h, y, g_in, mod, temb, g_out, o, N, D, eps, s):
        self._ck("resgate_temb", self.L.anima_residual_gate_adaln_temb_bf16(h, y, g_in, mod, temb, g_out, o, N, D,
                                                                            eps, s))


class RefOps:
    """The reference's kernels.h launchers from oracle/_ref (C++ linkage, void)."""

    kind = "reference"

    def __init__(self):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O  # the reference's host sinusoid loop, restated in C
        import refkernels

        self.R = refkernels.load_reference()
        self.O = O

    def add(self, a, b, o, n, s):
        self.R.add_bf16(a, b, o, n, s)

    def adaln_layernorm(self, x, sc, sh, o, N, D, eps, s):
        self.R.adaln_layernorm_bf16(x, sc, sh, o, N, D, eps, s)

    def rms_norm(self, x, w, o, N, D, eps, s):
        self.R.rms_norm_bf16(x, w, o, N, D, eps, s)

    def rope_cosmos_strided(self, x, c, sn, B, S, H, HD, s):
        self.R.rope_cosmos_strided_bf16(x, c, sn, B, S, H, HD, s)

    def residual_gate_adaln(self, h, y, g, sc, sh, o, N, D, eps, s):
        self.R.residual_gate_adaln_bf16(h, y, g, sc, sh, o, N, D, eps, s)

    def gelu_tanh(self, x, o, n, s):
        self.R.gelu_tanh_bf16(x, o, n, s)

    def residual_gate_bcast(self, x, y, g, o, M, D, s):
        self.R.residual_gate_bcast_bf16(x, y, g, o, M, D, s)

    def timestep(self, t, w, sin_out, normed, dim, eps, s, host_buf=None, sin_tensor=None):
        # transformer.cpp:182-200: host sinusoid, bf16 upload, then rms_norm_bf16 on one row
        host_buf.numpy()[:] = self.O.timestep_sinusoid(t, dim).view(np.int16)
        sin_tensor.copy_(host_buf, non_blocking=False)  # synchronous, like the reference's cudaMemcpy
        self.R.rms_norm_bf16(sin_out, w, normed, 1, dim, eps, s)

    def call(self, name, *args):
        getattr(self.R, name + "_bf16")(*args)

    def embedding_lookup(self, table, ids, out, T, D, vocab, s):
        self.R.embedding_lookup_bf16(table, ids, out, T, D, s)

    # the reference's call chains that the fused entry points replace
    def swiglu(self, g, u, o, n, s):  # qwen3.cpp:248-250
        self.R.silu_bf16(g, o, n, s)
        self.R.mul_bf16(o, u, o, n, s)

    def rms_norm_channel_silu(self, x, gamma, o, B, C, sp, eps, s):  # vae.cpp:148,184
        self.R.rms_norm_channel_bf16(x, gamma, o, B, C, sp, eps, s)
        self.R.silu_bf16(o, o, B * C * sp, s)

    def head_qk_norm_rope(self, src, w, c, sn, dst, H, T, HD, eps, s):  # qwen3.cpp:164-178
        self.R.head_transpose_bf16(src, dst, H, T, HD, s)
        self.R.rms_norm_bf16(dst, w, dst, H * T, HD, eps, s)
        self.R.rope_standard_bf16(dst, c, sn, H * T, T, HD, s)

    def causal_softmax(self, sc, o, H, T, s):  # qwen3.cpp:205-208
        self.R.causal_mask_bf16(sc, H, T, s)
        self.R.softmax_bf16(sc, o, H * T, T, s)

    def softmax_f32_to_bf16(self, x, o, N, D, s):
        self.R.softmax_f32_to_bf16(x, o, N, D, s)

    def layer_norm_modulate(self, x, sc, sh, o, N, D, eps, s):  # transformer.cpp:563-564
        self.R.layer_norm_bf16(x, o, N, D, eps, s)
        self.R.scale_shift_bcast_bf16(o, sc, sh, o, N, D, s)

    def qk_norm_rope(self, x, w, c, sn, B, S, H, HD, eps, s):  # transformer.cpp:350-358
        self.R.rms_norm_bf16(x, w, x, B * S * H, HD, eps, s)
        self.R.rope_cosmos_strided_bf16(x, c, sn, B, S, H, HD, s)


# ---------------------------------------------------------------- device state
class Chain:
    def __init__(self, ops, device, seed=1234, cfg=None):
        import torch

        import tables

        self.ops, self.dev = ops, device
        c = self.cfg = dict(cfg if cfg is not None else CFG)
        self.B, self.S = c["batch"], c["pe"][0] * c["pe"][1] * c["pe"][2]
        self.R, self.D, self.H, self.HD = self.B * self.S, c["hidden"], c["heads"], c["head_dim"]
        self.M, self.T, self.NB, self.eps = c["mlp"], c["text"], c["blocks"], c["eps"]
        g = torch.Generator(device=device).manual_seed(seed)

        def randn(shape, mean=0.0, std=1.0):
            return (torch.randn(shape, generator=g, device=device) * std + mean).to(torch.bfloat16)

        R, D, H, HD = self.R, self.D, self.H, self.HD
        self.sets = []
        for _ in range(NSETS):
            self.sets.append(dict(
                hidden=randn((R, D)), normed=torch.empty((R, D), dtype=torch.bfloat16, device=device),
                sub=randn((R, D)), q=randn((R, H * HD)), k=randn((R, H * HD)), qc=randn((R, H * HD)),
                kc=randn((self.B * self.T, H * HD)), ff=randn((R, self.M)),
                ff_out=torch.empty((R, self.M), dtype=torch.bfloat16, device=device)))
        # fresh modulation per block (3 adaLN-Zero sets of shift|scale|gate) + temb
        self.mod_raw = randn((self.NB, 3, 3 * D), std=0.1)
        self.mod = torch.empty_like(self.mod_raw)
        self.temb = randn((3 * D,), std=0.1)
        self.qk_w = randn((self.NB, 4, HD), mean=1.0, std=0.02)
        cos_t, sin_t = tables.cosmos_rope_tables(*c["pe"], HD)
        self.cos = torch.from_numpy(cos_t.view(np.int16)).to(device)
        self.sin = torch.from_numpy(sin_t.view(np.int16)).to(device)
        self.ts_w = randn((c["ts_dim"],), mean=1.0, std=0.02)
        self.ts_sin = torch.empty((c["ts_dim"],), dtype=torch.bfloat16, device=device)
        self.ts_out = torch.empty((c["ts_dim"],), dtype=torch.bfloat16, device=device)
        self.ts_host = torch.empty((c["ts_dim"],), dtype=torch.int16).pin_memory()
        self.ts_rng = np.random.default_rng(seed)
        self.launches_per_block = 14
        self.gates = [torch.empty((D,), dtype=torch.bfloat16, device=device) for _ in range(2)]
        self.launches_fused = 7 * self.NB + (self.NB - 1) + 2  # + the first adaLN and the last residual gate

    def timestep(self, stream):
        import torch

        t = float(np.float32(self.ts_rng.uniform()) * np.float32(1000.0))
        self.ops.timestep(t, self.ts_w.data_ptr(), self.ts_sin.data_ptr(), self.ts_out.data_ptr(), self.cfg["ts_dim"],
                          self.eps, stream, host_buf=self.ts_host, sin_tensor=self.ts_sin.view(torch.int16))

    def block(self, i, stream, only=None):
        """One DiT block's chain; `only` restricts it to one op type (for per-op timing)."""
        o, st = self.ops, stream
        bs = self.sets[i % NSETS]
        R, D, H, HD, B, S = self.R, self.D, self.H, self.HD, self.B, self.S
        mod = [self.mod[i, j] for j in range(3)]
        w = self.qk_w[i]
        P = lambda t: t.data_ptr()  # noqa: E731

        def run(name, fn, *args):
            if only is None or only == name:
                fn(*args)

        for j in range(3):  # compute_adaln_zero's mod += temb (transformer.cpp:408)
            run("add", o.add, P(self.mod_raw[i, j]), P(self.temb), P(mod[j]), 3 * D, st)
        shift, scale, gate = (lambda m: (P(m), P(m) + 2 * D, P(m) + 4 * D))(mod[0])
        run("adaln_layernorm", o.adaln_layernorm, P(bs["hidden"]), scale, shift, P(bs["normed"]), R, D, self.eps, st)
        run("rms_norm_qk128", o.rms_norm, P(bs["q"]), P(w[0]), P(bs["q"]), R * H, HD, self.eps, st)
        run("rms_norm_qk128", o.rms_norm, P(bs["k"]), P(w[1]), P(bs["k"]), R * H, HD, self.eps, st)
        run("rope_cosmos_strided", o.rope_cosmos_strided, P(bs["q"]), P(self.cos), P(self.sin), B, S, H, HD, st)
        run("rope_cosmos_strided", o.rope_cosmos_strided, P(bs["k"]), P(self.cos), P(self.sin), B, S, H, HD, st)
        shift, scale, gate2 = (P(mod[1]), P(mod[1]) + 2 * D, P(mod[1]) + 4 * D)
        run("residual_gate_adaln", o.residual_gate_adaln, P(bs["hidden"]), P(bs["sub"]), gate, scale, shift,
            P(bs["normed"]), R, D, self.eps, st)
        run("rms_norm_qk128", o.rms_norm, P(bs["qc"]), P(w[2]), P(bs["qc"]), R * H, HD, self.eps, st)
        run("rms_norm_qk128", o.rms_norm, P(bs["kc"]), P(w[3]), P(bs["kc"]), B * self.T * H, HD, self.eps, st)
        shift, scale, gate3 = (P(mod[2]), P(mod[2]) + 2 * D, P(mod[2]) + 4 * D)
        run("residual_gate_adaln", o.residual_gate_adaln, P(bs["hidden"]), P(bs["sub"]), gate2, scale, shift,
            P(bs["normed"]), R, D, self.eps, st)
        # the FFN activation is fresh every step (a GEMM output), so GELU reads ff and
        # writes ff_out rather than re-applying itself to its own output
        run("gelu_tanh", o.gelu_tanh, P(bs["ff"]), P(bs["ff_out"]), R * self.M, st)
        run("residual_gate_bcast", o.residual_gate_bcast, P(bs["hidden"]), P(bs["sub"]), gate3, P(bs["hidden"]), R,
            D, st)

    def block_fused(self, i, stream, g0, g1, first, last):
        """The same block through the opt-in fused entry points (one-line caller changes):
        mod += temb and the gate copy folded into the adaLN / residual-gate norms (two gate
        buffers alternate: g0 holds this block's adaLN gate), QK RMSNorm + RoPE in one pass. The
        residual gate that ends the block and the adaLN-Zero that starts the next are one
        residual_gate_adaln_temb (the next block's modulation GEMM depends only on temb, so a
        caller can run it first). Returns the next block's (g0, g1)."""
        o, st = self.ops, stream
        bs = self.sets[i % NSETS]
        R, D, H, HD, B, S = self.R, self.D, self.H, self.HD, self.B, self.S
        w = self.qk_w[i]
        P = lambda t: t.data_ptr()  # noqa: E731
        temb = P(self.temb)
        if first:
            o.adaln_layernorm_temb(P(bs["hidden"]), P(self.mod_raw[i, 0]), temb, g0, P(bs["normed"]), R, D, self.eps,
                                   st)
        o.qk_norm_rope(P(bs["q"]), P(w[0]), P(self.cos), P(self.sin), B, S, H, HD, self.eps, st)
        o.qk_norm_rope(P(bs["k"]), P(w[1]), P(self.cos), P(self.sin), B, S, H, HD, self.eps, st)
        o.residual_gate_adaln_temb(P(bs["hidden"]), P(bs["sub"]), g0, P(self.mod_raw[i, 1]), temb, g1,
                                   P(bs["normed"]), R, D, self.eps, st)
        o.rms_norm(P(bs["qc"]), P(w[2]), P(bs["qc"]), R * H, HD, self.eps, st)
        o.rms_norm(P(bs["kc"]), P(w[3]), P(bs["kc"]), B * self.T * H, HD, self.eps, st)
        o.residual_gate_adaln_temb(P(bs["hidden"]), P(bs["sub"]), g1, P(self.mod_raw[i, 2]), temb, g0,
                                   P(bs["normed"]), R, D, self.eps, st)
        o.gelu_tanh(P(bs["ff"]), P(bs["ff_out"]), R * self.M, st)
        if last:
            o.residual_gate_bcast(P(bs["hidden"]), P(bs["sub"]), g0, P(bs["hidden"]), R, D, st)
            return g0, g1
        nxt = self.sets[(i + 1) % NSETS]
        o.residual_gate_adaln_temb(P(bs["hidden"]), P(bs["sub"]), g0, P(self.mod_raw[i + 1, 0]), temb, g1,
                                   P(nxt["normed"]), R, D, self.eps, st)
        return g1, g0

    def blocks(self, stream, only=None):
        for i in range(self.NB):
            self.block(i, stream, only)

    def blocks_fused(self, stream):
        g0, g1 = self.gates[0].data_ptr(), self.gates[1].data_ptr()
        for i in range(self.NB):
            g0, g1 = self.block_fused(i, stream, g0, g1, i == 0, i == self.NB - 1)


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.reader = None

    def start(self, ready_timeout=10.0):
        """Start sampling and wait (bounded) for the first sample, so that a slow nvidia-smi
        start-up on a fresh box cannot leave a short timed region without samples."""
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.lines = []

        def read(stream, sink):
            for line in stream:
                sink.append(line)

        self.reader = threading.Thread(target=read, args=(self.proc.stdout, self.lines), daemon=True)
        self.reader.start()
        deadline = time.time() + ready_timeout
        while not self.lines and self.proc.poll() is None and time.time() < deadline:
            time.sleep(0.02)

    def mark(self):
        """Wall-clock bounds of the timed region (samples outside it are dropped)."""
        import datetime

        return datetime.datetime.now()

    def stop(self, t0=None, t1=None):
        import datetime

        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        if self.reader is not None:
            self.reader.join(timeout=5)
        out = "".join(self.lines)
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                ts = None
            if t0 is not None and ts is not None and not (t0 <= ts <= t1):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- multi-rank plumbing
def reduce_max(value: float, dist, device) -> float:
    """Max of a per-rank scalar over all ranks (the slowest rank's device time)."""
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_gbs(n_ranks: int, bytes_per_step: int, steps: int, max_ms: float) -> float:
    """Whole-job throughput: every rank processed `steps` steps of `bytes_per_step`
    (weak scaling); the job took as long as its slowest rank."""
    return n_ranks * bytes_per_step * steps / (max_ms * 1e-3) / 1e9


# ---------------------------------------------------------------- measurements
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def dram_traffic(op):
    """DRAM bytes per launch of `op` from the ncu capture summarised in profiles/ (None
    if that kernel has not been captured)."""
    try:
        with open(os.path.join(ROOT, "profiles", "dram_traffic.txt")) as f:
            for line in f:
                parts = line.split()
                if parts and not parts[0].startswith("#") and parts[0] == op:
                    return int(parts[1])
    except OSError:
        pass
    return None


def time_steps(chain, steps, stream_obj, graph, ts=True):
    """Device time (ms) of `steps` steps on the current stream, events on both sides."""
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        if ts:
            chain.timestep(stream_obj.cuda_stream)
        if graph is not None:
            graph.replay()
        else:
            chain.blocks(stream_obj.cuda_stream)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def e2e_pipelined(chain, graph, steps, h_in, m_in, h_out):
    """End to end with host buffers, double-buffered as a serving loop would run it: step k+1's
    hidden-state upload and step k's download run on a copy stream while step k computes.
    Device staging buffers decouple them from the chain's own buffers (two device-to-device
    copies per step on the compute stream, inside the timed region). Every step still moves
    its full input host->device and its result device->host. Returns ms per step."""
    import torch

    R, D = chain.R, chain.D
    last = chain.sets[(chain.NB - 1) % NSETS]["hidden"]
    compute, copy = torch.cuda.Stream(), torch.cuda.Stream()
    in_stage = [torch.empty((R, D), dtype=torch.bfloat16, device=chain.dev) for _ in range(2)]
    out_stage = [torch.empty((R, D), dtype=torch.bfloat16, device=chain.dev) for _ in range(2)]
    ev_in, ev_in_free, ev_out, ev_out_free = ([torch.cuda.Event() for _ in range(2)] for _ in range(4))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(compute):
        a.record()
    copy.wait_event(a)
    with torch.cuda.stream(copy):
        in_stage[0].copy_(h_in, non_blocking=True)
        ev_in[0].record()
    for k in range(steps):
        j, n = k % 2, (k + 1) % 2
        if k + 1 < steps:  # the next step's upload, once step k-1 has consumed that stage
            with torch.cuda.stream(copy):
                if k >= 1:
                    copy.wait_event(ev_in_free[n])
                in_stage[n].copy_(h_in, non_blocking=True)
                ev_in[n].record()
        with torch.cuda.stream(compute):
            compute.wait_event(ev_in[j])
            chain.sets[0]["hidden"].copy_(in_stage[j], non_blocking=True)
            ev_in_free[j].record()
            chain.mod_raw.copy_(m_in, non_blocking=True)
            chain.timestep(compute.cuda_stream)
            if graph is not None:
                graph.replay()
            else:
                chain.blocks(compute.cuda_stream)
            if k >= 2:
                compute.wait_event(ev_out_free[j])
            out_stage[j].copy_(last, non_blocking=True)
            ev_out[j].record()
        with torch.cuda.stream(copy):
            copy.wait_event(ev_out[j])
            h_out.copy_(out_stage[j], non_blocking=True)
            ev_out_free[j].record()
    compute.wait_stream(copy)
    with torch.cuda.stream(compute):
        b.record()
    torch.cuda.synchronize()
    del in_stage, out_stage
    return a.elapsed_time(b) / steps


def capture(fn):
    """CUDA graph of the launches `fn(stream_handle)` makes (on a side stream)."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            fn(side.cuda_stream)
    torch.cuda.current_stream().wait_stream(side)
    return g


def per_op_times(chain, ops, reps):
    """Device time per launch of each op type: a CUDA graph holding only that op's launches
    of one step (its real arguments, so it cycles the same >L2 buffer sets), replayed
    `reps` times between CUDA events. Returns op -> mean ms per launch."""
    import torch

    out = {}
    for name, per_step in ops.items():
        g = capture(lambda s: chain.blocks(s, only=name))
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        out[name] = a.elapsed_time(b) / (reps * per_step)
        del g
    return out


def headline_kernels(ops, device, peak, reps=384, only=None, steps=3, warmup=3):
    """Every in-scope row / elementwise kernel at the headline shape, 4096 tokens x 2048
    (GELU and SiLU at the FFN width, [4096, 8192]; QK RMSNorm on the same tensor as
    [4096*16, 128] head rows; Cosmos RoPE on [4096, 16*128] with the (1, 64, 64) grid's
    tables), each launch cycling 8 buffer sets (> 2x L2) so every launch reads from HBM.
    Each case is a CUDA graph of 48 back-to-back launches of that kernel alone, replayed;
    us = graph time / launches. Returns name -> {us, gbs, frac}.

    only: the name of one case (profiling aid, for ncu captures): run `warmup` then `steps`
    eager launches of it, print their timing and return None."""
    import torch

    import tables

    N, D, M, H, HD = 4096, 2048, 8192, 16, 128
    sets = 8
    x = [torch.randn((N, D), device=device).to(torch.bfloat16) for _ in range(sets)]
    y = [torch.randn((N, D), device=device).to(torch.bfloat16) for _ in range(sets)]
    o = [torch.empty((N, D), dtype=torch.bfloat16, device=device) for _ in range(sets)]
    f = [torch.randn((N, M), device=device).to(torch.bfloat16) for _ in range(4)]
    v = (torch.randn((3 * D,), device=device) * 0.1).to(torch.bfloat16)
    w = (torch.randn((D,), device=device) * 0.02 + 1.0).to(torch.bfloat16)
    sc, sh, g = v.data_ptr(), v.data_ptr() + 2 * D, v.data_ptr() + 4 * D
    ct, st = tables.cosmos_rope_tables(1, 64, 64, HD)
    ct_d = torch.from_numpy(ct.view(np.int16)).to(device)
    st_d = torch.from_numpy(st.view(np.int16)).to(device)
    eps = 1e-6
    P = lambda t: t.data_ptr()  # noqa: E731

    def S():
        return torch.cuda.current_stream().cuda_stream  # the capture stream inside capture()

    # (§8 row, algorithmic bytes per launch, launch(i)); bytes as in SURVEY §8(a)
    cases = {
        "a1_adaln_layernorm": (4 * N * D + 4 * D,
                               lambda i: ops.adaln_layernorm(P(x[i]), sc, sh, P(o[i]), N, D, eps, S())),
        "a2_residual_gate_adaln": (8 * N * D + 6 * D, lambda i: ops.residual_gate_adaln(
            P(x[i]), P(y[i]), g, sc, sh, P(o[i]), N, D, eps, S())),
        "a3_residual_gate_bcast": (6 * N * D + 2 * D, lambda i: ops.residual_gate_bcast(
            P(x[i]), P(y[i]), g, P(x[i]), N, D, S())),
        "a4_layer_norm": (4 * N * D, lambda i: ops.call("layer_norm", P(x[i]), P(o[i]), N, D, eps, S())),
        "a5_scale_shift_bcast": (4 * N * D + 4 * D, lambda i: ops.call(
            "scale_shift_bcast", P(x[i]), sc, sh, P(o[i]), N, D, S())),
        "a6_rms_norm_2048": (4 * N * D + 2 * D, lambda i: ops.rms_norm(P(x[i]), P(w), P(o[i]), N, D, eps, S())),
        "a6_rms_norm_qk128": (4 * N * D + 2 * HD, lambda i: ops.rms_norm(P(x[i]), P(w), P(o[i]), N * H, HD, eps,
                                                                         S())),
        "a7_rope_cosmos_strided": (4 * N * D + 2 * N * (HD // 2) * 2, lambda i: ops.rope_cosmos_strided(
            P(x[i]), P(ct_d), P(st_d), 1, N, H, HD, S())),
        "a8_gelu_tanh_4096x8192": (4 * N * M, lambda i: ops.gelu_tanh(P(f[i % 2]), P(f[2 + i % 2]), N * M, S())),
        "a9_silu_4096x8192": (4 * N * M, lambda i: ops.call("silu", P(f[i % 2]), P(f[2 + i % 2]), N * M, S())),
        "a10_add": (6 * N * D, lambda i: ops.add(P(x[i]), P(y[i]), P(o[i]), N * D, S())),
        "a10_mul": (6 * N * D, lambda i: ops.call("mul", P(x[i]), P(y[i]), P(o[i]), N * D, S())),
    }
    if only is not None:
        if only not in cases:
            raise SystemExit(f"--only {only}: no such case (cases: {', '.join(cases)})")
        nbytes, fn = cases[only]
        for i in range(warmup):
            fn(i % sets)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(steps):
            fn(i % sets)
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / steps
        print(json.dumps({"op": only, "impl": ops.kind, "calls": steps, "us_per_call": round(us, 2),
                          "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}))
        return None
    res = {}
    per_graph = 6 * sets  # launches per captured graph, cycling the buffer sets
    for name, (nbytes, fn) in cases.items():
        for i in range(4):
            fn(i % sets)
        torch.cuda.synchronize()
        graph = capture(lambda st: [fn(i % sets) for i in range(per_graph)])
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_rep = max(1, reps // per_graph)
        a.record()
        for _ in range(n_rep):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        del graph
        us = a.elapsed_time(b) * 1e3 / (n_rep * per_graph)
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)}
    del x, y, o, f
    torch.cuda.empty_cache()
    return res


def other_ops(ops, device, peak, reps=96, only=None, steps=3, warmup=3):
    """The in-scope ops outside the cfg2 chain, at BASELINE's other configs, each through
    the arm's own entry points: cfg3 (Qwen3-0.6B layer ops at seq 512), cfg4 (the VAE
    decoder's channel RMSNorm + SiLU at its four shapes), and the final LayerNorm +
    modulate and QK-norm + RoPE chains at cfg2. Where this library has a fused entry point
    (SwiGLU, channel norm + SiLU, LayerNorm + modulate, QK-norm + RoPE) the anima arm
    times the fused call and the reference arm the reference's call chain it replaces;
    the anima arm also times its own drop-in chain. Each case cycles enough buffer sets
    to exceed L2 where its tensors are large (small cfg3 tensors stay L2-resident, as in
    the model) and is timed as a CUDA graph replay. Returns name -> us per call, GB/s.

    only: the name of one case (profiling aid, for ncu captures): allocate only what that
    case needs where the tensors are large (the cfg4 shapes), run `warmup` then `steps`
    eager calls of it, print their timing and return None."""
    import torch

    import tables

    eps = 1e-6
    P = lambda t: t.data_ptr()  # noqa: E731
    g = torch.Generator(device=device).manual_seed(99)

    def bf(shape, mean=0.0, std=1.0):
        return (torch.randn(shape, generator=g, device=device) * std + mean).to(torch.bfloat16)

    def S():
        return torch.cuda.current_stream().cuda_stream

    cases = []  # (name, algorithmic bytes per call, launches per call, sets, make(i) -> fn)

    # ---- cfg3: Qwen3-0.6B, seq 512
    T, Dq, V, F = 512, 1024, 151936, 3072
    table = bf((V, Dq), std=0.02)
    ids = torch.randint(0, V, (8, T), generator=g, device=device, dtype=torch.int32)
    emb = [torch.empty((T, Dq), dtype=torch.bfloat16, device=device) for _ in range(8)]
    cases.append(("cfg3_embedding_lookup_512x1024", 4 * T * Dq + 4 * T, 1, 8,
                  lambda i: ops.embedding_lookup(P(table), P(ids[i]), P(emb[i]), T, Dq, V, S())))
    xq = [bf((T, Dq)) for _ in range(8)]
    wq = bf((Dq,), mean=1.0, std=0.02)
    oq = [torch.empty_like(x) for x in xq]
    cases.append(("cfg3_rms_norm_512x1024", 4 * T * Dq + 2 * Dq, 1, 8,
                  lambda i: ops.call("rms_norm", P(xq[i]), P(wq), P(oq[i]), T, Dq, eps, S())))
    qh = [bf((16 * T, 128)) for _ in range(8)]
    wh = bf((128,), mean=1.0, std=0.02)
    cases.append(("cfg3_qk_rms_norm_16x512x128", 4 * 16 * T * 128 + 256, 1, 8,
                  lambda i: ops.call("rms_norm", P(qh[i]), P(wh), P(qh[i]), 16 * T, 128, eps, S())))
    cs, sn = tables.standard_rope_tables(T, 128, 1e6)
    cs_d, sn_d = torch.from_numpy(cs).to(device), torch.from_numpy(sn).to(device)
    cases.append(("cfg3_rope_standard_16x512x128", 4 * 16 * T * 128 + 4 * T * 128, 1, 8,
                  lambda i: ops.call("rope_standard", P(qh[i]), P(cs_d), P(sn_d), 16 * T, T, 128, S())))
    gt = [bf((T, F)) for _ in range(8)]
    ut = [bf((T, F)) for _ in range(8)]
    st_ = [torch.empty_like(x) for x in gt]
    cases.append(("cfg3_swiglu_512x3072", 6 * T * F, 1 if ops.kind == "anima" else 2, 8,
                  lambda i: ops.swiglu(P(gt[i]), P(ut[i]), P(st_[i]), T * F, S())))
    if ops.kind == "anima":
        cases.append(("cfg3_swiglu_512x3072_as_silu_mul", 6 * T * F, 2, 8,
                      lambda i: (ops.call("silu", P(gt[i]), P(st_[i]), T * F, S()),
                                 ops.call("mul", P(st_[i]), P(ut[i]), P(st_[i]), T * F, S()))))

    # cfg3 attention glue (qwen3.cpp:164-226): head layout, GQA expansion, causal softmax
    QH, KVH, HDq = 16, 8, 128
    qb = [bf((T, QH * HDq)) for _ in range(8)]
    qhd = [torch.empty((QH, T, HDq), dtype=torch.bfloat16, device=device) for _ in range(8)]
    cases.append(("cfg3_head_transpose_512x16x128", 4 * T * QH * HDq, 1, 8,
                  lambda i: ops.call("head_transpose", P(qb[i]), P(qhd[i]), QH, T, HDq, S())))
    cases.append(("cfg3_head_untranspose_16x512x128", 4 * T * QH * HDq, 1, 8,
                  lambda i: ops.call("head_untranspose", P(qhd[i]), P(qb[i]), QH, T, HDq, S())))
    cases.append(("cfg3_head_transpose_qk_norm_rope_512x16x128", 4 * T * QH * HDq + 2 * HDq + 4 * T * HDq,
                  1 if ops.kind == "anima" else 3, 8,
                  lambda i: ops.head_qk_norm_rope(P(qb[i]), P(wh), P(cs_d), P(sn_d), P(qhd[i]), QH, T, HDq, eps, S())))
    if ops.kind == "anima":
        cases.append(("cfg3_head_transpose_qk_norm_rope_512x16x128_as_three_calls",
                      4 * T * QH * HDq + 2 * HDq + 4 * T * HDq, 3, 8,
                      lambda i: (ops.call("head_transpose", P(qb[i]), P(qhd[i]), QH, T, HDq, S()),
                                 ops.call("rms_norm", P(qhd[i]), P(wh), P(qhd[i]), QH * T, HDq, eps, S()),
                                 ops.call("rope_standard", P(qhd[i]), P(cs_d), P(sn_d), QH * T, T, HDq, S()))))
    kvh = [bf((KVH, T, HDq)) for _ in range(8)]
    cases.append(("cfg3_expand_kv_8to16x512x128", 2 * (KVH + QH) * T * HDq, 1, 8,
                  lambda i: ops.call("expand_kv", P(kvh[i]), P(qhd[i]), 1, KVH, QH, T, HDq, S())))
    scs = [bf((QH, T, T), std=3.0) for _ in range(8)]
    cases.append(("cfg3_softmax_16x512x512", 4 * QH * T * T, 1, 8,
                  lambda i: ops.call("softmax", P(scs[i]), P(scs[i]), QH * T, T, S())))
    cases.append(("cfg3_causal_mask_softmax_16x512x512", 4 * QH * T * T, 1 if ops.kind == "anima" else 2, 8,
                  lambda i: ops.causal_softmax(P(scs[i]), P(scs[i]), QH, T, S())))
    if ops.kind == "anima":
        cases.append(("cfg3_causal_mask_softmax_16x512x512_as_two_calls", 4 * QH * T * T, 2, 8,
                      lambda i: (ops.call("causal_mask", P(scs[i]), QH, T, S()),
                                 ops.call("softmax", P(scs[i]), P(scs[i]), QH * T, T, S()))))
    # cfg4 VAE attention softmax (vae.cpp:262): fp32 scores [512, 512] -> bf16
    vsc = [torch.randn((512, 512), generator=g, device=device) * 4.0 for _ in range(8)]
    vsb = [torch.empty((512, 512), dtype=torch.bfloat16, device=device) for _ in range(8)]
    cases.append(("cfg4_softmax_f32_to_bf16_512x512", 6 * 512 * 512, 1, 8,
                  lambda i: ops.softmax_f32_to_bf16(P(vsc[i]), P(vsb[i]), 512, 512, S())))

    # ---- cfg2 denoising-loop I/O: CFG + Euler step, patchify / unpatchify, latent denorm
    Cl, Hl = 16, 128
    nl = Cl * Hl * Hl
    lat = [bf((nl,)) for _ in range(8)]
    npos, nneg = [bf((nl,)) for _ in range(8)], [bf((nl,)) for _ in range(8)]
    cases.append(("cfg2_cfg_euler_step_16x128x128", 8 * nl, 1, 8,
                  lambda i: ops.call("cfg_euler_step", P(lat[i]), P(npos[i]), P(nneg[i]), P(lat[i]), 4.5, 0.73, 0.61,
                                     nl, S())))
    ptok = [torch.empty((4096, 64), dtype=torch.bfloat16, device=device) for _ in range(8)]
    cases.append(("cfg2_patchify_3d_16x128x128", 4 * nl, 1, 8,
                  lambda i: ops.call("patchify_3d", P(lat[i]), P(ptok[i]), 1, Cl, 1, Hl, Hl, 1, 2, 2, S())))
    cases.append(("cfg2_unpatchify_3d_16x128x128", 4 * nl, 1, 8,
                  lambda i: ops.call("unpatchify_3d", P(ptok[i]), P(npos[i]), 1, Cl, 1, Hl, Hl, 1, 2, 2, S())))
    lsc, lsh = bf((Cl,), mean=1.0, std=0.3), bf((Cl,), std=0.5)
    cases.append(("cfg2_channel_scale_shift_16x128x128", 4 * nl + 4 * Cl, 1, 8,
                  lambda i: ops.call("channel_scale_shift", P(nneg[i]), P(lsc), P(lsh), P(nneg[i]), 1, Cl, Hl * Hl,
                                     S())))

    # ---- cfg4: VAE channel RMSNorm + SiLU, NCHW
    for (C, Hs) in ((512, 128), (512, 256), (256, 512), (128, 1024)):
        if only is not None and not (only.startswith("cfg4_") and only.endswith(f"_{C}x{Hs}x{Hs}")):
            continue
        sp = Hs * Hs
        sets = max(2, min(8, -(-512 * 2**20 // (4 * C * sp))))
        xs = [bf((C, sp)) for _ in range(sets)]
        ys = [torch.empty_like(x) for x in xs]
        gm = bf((C,), mean=1.0, std=0.02)
        cases.append((f"cfg4_rms_norm_channel_silu_{C}x{Hs}x{Hs}", 4 * C * sp + 2 * C,
                      1 if ops.kind == "anima" else 2, sets,
                      (lambda xs, ys, gm, C, sp: lambda i: ops.rms_norm_channel_silu(
                          P(xs[i]), P(gm), P(ys[i]), 1, C, sp, eps, S()))(xs, ys, gm, C, sp)))
        if ops.kind == "anima":
            cases.append((f"cfg4_rms_norm_channel_silu_{C}x{Hs}x{Hs}_as_two_calls", 4 * C * sp + 2 * C, 2, sets,
                          (lambda xs, ys, gm, C, sp: lambda i: (
                              ops.call("rms_norm_channel", P(xs[i]), P(gm), P(ys[i]), 1, C, sp, eps, S()),
                              ops.call("silu", P(ys[i]), P(ys[i]), C * sp, S())))(xs, ys, gm, C, sp)))
            # The conv epilogue (causal_conv3d.cu:187-195 and the chains after it, vae.cpp:185-194).
            # The reference's bias kernel is file-local to causal_conv3d_forward, so there is
            # no reference-arm timing of it.
            cb = bf((C,), std=0.5)
            cases.append((f"cfg4_conv_bias_add_{C}x{Hs}x{Hs}", 4 * C * sp + 2 * C, 1, sets,
                          (lambda xs, ys, cb, C, sp: lambda i: ops.call(
                              "conv_bias_add", P(xs[i]), P(cb), P(ys[i]), 1, C, sp, S()))(xs, ys, cb, C, sp)))
            cases.append((f"cfg4_conv_bias_residual_add_{C}x{Hs}x{Hs}", 6 * C * sp + 2 * C, 1, sets,
                          (lambda xs, ys, cb, C, sp: lambda i: ops.call(
                              "conv_bias_residual_add", P(xs[i]), P(cb), P(ys[i]), P(ys[i]), 1, C, sp,
                              S()))(xs, ys, cb, C, sp)))
            cases.append((f"cfg4_conv_bias_rms_norm_channel_silu_{C}x{Hs}x{Hs}", 4 * C * sp + 4 * C, 1, sets,
                          (lambda xs, ys, cb, gm, C, sp: lambda i: ops.call(
                              "conv_bias_rms_norm_channel_silu", P(xs[i]), P(cb), P(gm), P(ys[i]), 1, C, sp, eps,
                              S()))(xs, ys, cb, gm, C, sp)))

    # ---- cfg2: bias add after a Linear, final LayerNorm + modulate, QK RMSNorm + RoPE on q
    R, D, H, HD = 8192, 2048, 16, 128
    xl = [bf((R, D)) for _ in range(4)]
    ol = [torch.empty_like(x) for x in xl]
    mv = bf((2 * D,), std=0.1)
    cases.append(("cfg2_bias_add_8192x2048", 4 * R * D + 2 * D, 1, 4,
                  lambda i: ops.call("bias_add", P(xl[i]), P(mv), P(ol[i]), R, D, S())))
    cases.append(("cfg2_layer_norm_modulate_8192x2048", 4 * R * D + 4 * D, 1 if ops.kind == "anima" else 2, 4,
                  lambda i: ops.layer_norm_modulate(P(xl[i]), P(mv), P(mv) + 2 * D, P(ol[i]), R, D, eps, S())))
    if ops.kind == "anima":
        cases.append(("cfg2_layer_norm_modulate_8192x2048_as_two_calls", 4 * R * D + 4 * D, 2, 4,
                      lambda i: (ops.call("layer_norm", P(xl[i]), P(ol[i]), R, D, eps, S()),
                                 ops.call("scale_shift_bcast", P(ol[i]), P(mv), P(mv) + 2 * D, P(ol[i]), R, D,
                                          S()))))
    ct, st2 = tables.cosmos_rope_tables(1, 64, 64, HD)
    ct_d = torch.from_numpy(ct.view(np.int16)).to(device)
    st_d = torch.from_numpy(st2.view(np.int16)).to(device)
    qk_bytes = 4 * R * D + 2 * HD + 2 * 4096 * HD * 2
    cases.append(("cfg2_qk_norm_rope_8192x16x128", qk_bytes, 1 if ops.kind == "anima" else 2, 4,
                  lambda i: ops.qk_norm_rope(P(xl[i]), P(wh), P(ct_d), P(st_d), 2, 4096, H, HD, eps, S())))
    if ops.kind == "anima":
        cases.append(("cfg2_qk_norm_rope_8192x16x128_as_two_calls", qk_bytes, 2, 4,
                      lambda i: (ops.call("rms_norm", P(xl[i]), P(wh), P(xl[i]), R * H, HD, eps, S()),
                                 ops.call("rope_cosmos_strided", P(xl[i]), P(ct_d), P(st_d), 2, 4096, H, HD,
                                          S()))))
    # the adaLN-Zero temb folds (one launch each for add + norm + gate copy) and the GPU
    # timestep embedding; the reference arm times its own chains for these in the DiT step
    if ops.kind == "anima":
        yl = [bf((R, D)) for _ in range(4)]
        mods = bf((3 * D,), std=0.1)
        tembv = bf((3 * D,), std=0.1)
        gts = [torch.empty((D,), dtype=torch.bfloat16, device=device) for _ in range(2)]
        cases.append(("cfg2_adaln_layernorm_temb_8192x2048", 4 * R * D + 12 * D, 1, 4,
                      lambda i: ops.adaln_layernorm_temb(P(xl[i]), P(mods), P(tembv), P(gts[i % 2]), P(ol[i]), R, D,
                                                         eps, S())))
        cases.append(("cfg2_residual_gate_adaln_temb_8192x2048", 8 * R * D + 14 * D, 1, 4,
                      lambda i: ops.residual_gate_adaln_temb(P(xl[i]), P(yl[i]), P(gts[i % 2]), P(mods), P(tembv),
                                                             P(gts[(i + 1) % 2]), P(ol[i]), R, D, eps, S())))
        tsw = bf((2048,), mean=1.0, std=0.02)
        tss = [torch.empty((2048,), dtype=torch.bfloat16, device=device) for _ in range(2)]
        cases.append(("cfg2_timestep_embedding_2048", 2 * 2048 + 6 * 2048, 1, 2,
                      lambda i: ops.timestep(617.25 + i, P(tsw), P(tss[0]), P(tss[1]), 2048, eps, S())))

    if only is not None:
        match = [c for c in cases if c[0] == only]
        if not match:
            raise SystemExit(f"--only {only}: no such case (cases: {', '.join(c[0] for c in cases)})")
        name, nbytes, launches, sets, fn = match[0]
        for i in range(warmup):
            fn(i % sets)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(steps):
            fn(i % sets)
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / steps
        print(json.dumps({"op": name, "impl": ops.kind, "calls": steps, "launches_per_call": launches,
                          "us_per_call": round(us, 2), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}))
        return None

    res = {}
    for name, nbytes, launches, sets, fn in cases:
        for i in range(sets):
            fn(i)
        torch.cuda.synchronize()
        per_graph = sets * max(1, 16 // sets)
        graph = capture(lambda st: [fn(i % sets) for i in range(per_graph)])
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_rep = max(2, reps // per_graph)
        a.record()
        for _ in range(n_rep):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        del graph
        us = a.elapsed_time(b) * 1e3 / (n_rep * per_graph)
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us": round(us, 2), "launches": launches, "bytes": nbytes, "gbs": round(gbs, 1),
                     "frac": round(gbs / peak, 3), "l2_resident": nbytes * sets < 126 * 2**20}
    torch.cuda.empty_cache()
    return res


def cpu_baseline_sample(blocks=2, rows=8192, threads=1):
    """The plain C host loop of the chain's ops (oracle/hostloop.c: fp32 math on bf16
    storage, gcc -O3 -march=native -fopenmp, built on this host) over `blocks` blocks of the
    cfg2 chain at full size on `threads` OpenMP threads. Returns (GB/s, description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hostloop
    import oracle as O

    L = hostloop.load()
    L.hostloop_set_threads(threads)
    rng = np.random.default_rng(5)
    c = CFG
    B, S = c["batch"], c["pe"][0] * c["pe"][1] * c["pe"][2]
    R = rows
    D, H, HD, M, T = c["hidden"], c["heads"], c["head_dim"], c["mlp"], c["text"]
    hidden, sub, normed = O.randn_bf16(rng, (R, D)), O.randn_bf16(rng, (R, D)), np.empty((R, D), np.uint16)
    q, k, qc = (O.randn_bf16(rng, (R * H, HD)) for _ in range(3))
    kc = O.randn_bf16(rng, (B * T * H, HD))
    ff, ff_out = O.randn_bf16(rng, R * M), np.empty(R * M, np.uint16)
    mod_raw = O.randn_bf16(rng, (3, 3 * D), std=0.1)
    mod = np.empty_like(mod_raw)
    temb = O.randn_bf16(rng, 3 * D, std=0.1)
    w = O.randn_bf16(rng, HD, mean=1.0, std=0.02)
    ct, st = O.cosmos_rope_tables(*c["pe"], HD)
    A = lambda a: a.ctypes.data  # noqa: E731
    eps = np.float32(1e-6)
    t0 = time.perf_counter()
    for _ in range(blocks):
        for j in range(3):
            L.hostloop_add(A(mod_raw[j]), A(temb), A(mod[j]), 3 * D)
        sh = [A(mod[j]) for j in range(3)]
        sc = [A(mod[j]) + 2 * D for j in range(3)]
        gt = [A(mod[j]) + 4 * D for j in range(3)]
        L.hostloop_adaln_layernorm(A(hidden), sc[0], sh[0], A(normed), R, D, eps)
        L.hostloop_rms_norm(A(q), A(w), A(q), R * H, HD, eps)
        L.hostloop_rms_norm(A(k), A(w), A(k), R * H, HD, eps)
        L.hostloop_rope_cosmos(A(q), A(ct), A(st), B, S, H, HD)
        L.hostloop_rope_cosmos(A(k), A(ct), A(st), B, S, H, HD)
        L.hostloop_residual_gate_adaln(A(hidden), A(sub), gt[0], sc[1], sh[1], A(normed), R, D, eps)
        L.hostloop_rms_norm(A(qc), A(w), A(qc), R * H, HD, eps)
        L.hostloop_rms_norm(A(kc), A(w), A(kc), B * T * H, HD, eps)
        L.hostloop_residual_gate_adaln(A(hidden), A(sub), gt[1], sc[2], sh[2], A(normed), R, D, eps)
        L.hostloop_gelu_tanh(A(ff), A(ff_out), R * M)
        L.hostloop_residual_gate_bcast(A(hidden), A(sub), gt[2], A(hidden), R, D)
    dt = time.perf_counter() - t0
    _, per_block, _ = chain_bytes()
    nbytes = blocks * sum(per_block.values()) * R / (B * S)
    return nbytes / dt / 1e9, (f"{blocks} of the 28 blocks of the cfg2 chain at {R} rows on {threads} OpenMP "
                               f"thread{'s' if threads > 1 else ''} ({dt:.1f} s)")


def cfg1_step(ops, device, steps, peak):
    """BASELINE config 1 (512x512 image, 1024 tokens, batch 1): the same 28-block chain at 1024
    rows, timed as CUDA graph replays and as eager launches. The per-block figure is the
    single-block chain BASELINE names. Its activations (~58 MB per buffer set) sit near the L2
    size, so the 4 rotating sets keep most reads in HBM; launches dominate at this size."""
    import torch

    c = dict(CFG, **CFG1)
    chain = Chain(ops, device, cfg=c)
    total, per_block, lpb = chain_bytes(c)
    s = torch.cuda.current_stream()
    for _ in range(3):
        chain.timestep(s.cuda_stream)
        chain.blocks(s.cuda_stream)
    torch.cuda.synchronize()
    graph = capture(lambda st: chain.blocks(st))
    graph.replay()
    torch.cuda.synchronize()
    k = max(3, min(steps, 50))
    g_ms = time_steps(chain, k, s, graph) / k
    del graph
    e_ms = time_steps(chain, max(3, min(steps, 20)), s, None) / max(3, min(steps, 20))
    f_ms = None
    if ops.kind == "anima":  # the same step through the opt-in fused entry points
        fgraph = capture(lambda st: chain.blocks_fused(st))
        fgraph.replay()
        torch.cuda.synchronize()
        f_ms = time_steps(chain, k, s, fgraph) / k
        del fgraph
    gbs = total / (g_ms * 1e-3) / 1e9
    out = {"workload": "cfg1: 512x512 image -> 1024 tokens, batch 1, 28-block DiT elementwise chain",
           "rows": chain.R, "bytes_per_step": total, "launches_per_step": c["blocks"] * chain.launches_per_block + 1,
           "ms_per_step": round(g_ms, 4), "ms_per_block": round(g_ms / c["blocks"], 4), "gbs": round(gbs, 1),
           "frac": round(gbs / peak, 3), "eager_ms_per_step": round(e_ms, 4),
           "fused_ms_per_step": round(f_ms, 4) if f_ms is not None else None,
           "fused_launches_per_step": chain.launches_fused + 1 if f_ms is not None else None}
    del chain
    torch.cuda.empty_cache()
    return out


def profile_one_op(args, chain, launches_per_step, bytes_per_launch):
    """--only: W eager warm-up steps then K timed eager steps of one op type (its real
    arguments across the 28 blocks). Small and self-contained, for ncu captures."""
    import torch

    s = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        chain.blocks(s, only=args.only)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        chain.blocks(s, only=args.only)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (args.steps * launches_per_step)
    print(json.dumps({"op": args.only, "impl": args.impl, "launches": args.steps * launches_per_step,
                      "us_per_launch": round(us, 2), "gbs": round(bytes_per_launch / (us * 1e-6) / 1e9, 1)}))


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["anima", "reference"], default="anima")
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of CUDA graph replay")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-headline", action="store_true")
    ap.add_argument("--no-other-ops", action="store_true", help="skip the cfg3/cfg4/fused-entry measurements")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg5"], default="cfg2",
                    help="cfg2 (default): 8192 rows per GPU, weak scaling. cfg1: BASELINE's 512x512 image, "
                         "1024 tokens, batch 1 (weak scaling). cfg5: BASELINE's throughput sweep, "
                         "8 image pairs at 1536x1536 (18432 rows each) split 8/N pairs per GPU, strong scaling")
    ap.add_argument("--only", default=None,
                    help="profiling aid: run only this op type of the chain, or this case of the other "
                         "configs (e.g. cfg4_rms_norm_channel_silu_512x256x256), eagerly; print its timing, exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    # Both arms run one replica per rank: the reference's launchers are stateless and act on the
    # calling rank's own device, so at N GPUs its line reports the same N-replica aggregate.
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    n_gpus = world if dist is not None else 1
    if n_gpus > 1:
        # the headline sweep, the other configs and the CPU baseline are single-GPU figures
        # (the N=1 line carries them); at N > 1 the other ranks would only wait at the final
        # barrier while rank 0 ran them
        args.no_headline = args.no_other_ops = args.no_cpu_baseline = True
    if args.workload == "cfg5":
        # 8 images at 1536x1536 -> 192x192 latent -> 96x96 patches = 9216 tokens, x CFG 2; the
        # image pairs are shared out over the GPUs as extra batch rows (rows are independent)
        if 8 % n_gpus:
            raise SystemExit("cfg5 shares 8 image pairs over the GPUs: use 1, 2, 4 or 8")
        CFG.update(pe=(1, 96, 96), batch=2 * (8 // n_gpus))
        args.no_headline = args.no_other_ops = args.no_cpu_baseline = True
    elif args.workload == "cfg1":
        CFG.update(CFG1)
        args.no_headline = args.no_other_ops = True

    ops = AnimaOps() if args.impl == "anima" else RefOps()
    peak, peak_kind = peaks()
    total_bytes, per_block, lpb = chain_bytes()
    if args.only is not None and args.only not in lpb:  # one case of the other measurements
        if args.only.startswith("a") and args.only[1:2].isdigit():
            return headline_kernels(ops, device, peak, only=args.only, steps=args.steps, warmup=args.warmup)
        return other_ops(ops, device, peak, only=args.only, steps=args.steps, warmup=args.warmup)
    chain = Chain(ops, device)
    stream = torch.cuda.current_stream()

    if args.only is not None:
        return profile_one_op(args, chain, lpb[args.only] * CFG["blocks"], per_block[args.only] / lpb[args.only])

    # warm-up (also initialises every kernel and the library's device caches)
    for _ in range(args.warmup):
        chain.timestep(stream.cuda_stream)
        chain.blocks(stream.cuda_stream)
    torch.cuda.synchronize()

    graph = None
    if not args.eager:
        graph = capture(lambda s: chain.blocks(s))
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()

    # timed region: barrier + synchronize on both sides, device events, max over ranks
    try:
        smi_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        smi_id = str(local_rank)
    clocks = ClockSampler(smi_id)
    clocks.start()  # returns once nvidia-smi has produced its first sample
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = clocks.mark()
    ms = time_steps(chain, args.steps, stream, graph)
    t_end = clocks.mark()
    ms = reduce_max(ms, dist, device)
    if dist is not None:
        dist.barrier()
    clk = clocks.stop(t_begin, t_end)
    ms_per_step = ms / args.steps
    value = aggregate_gbs(n_gpus, total_bytes, args.steps, ms)

    # the same steps launched eagerly (no graph): the reference launches this way on stream 0
    # (transformer.cpp:476); here both arms go through the same Python launcher loop
    eager = None
    if graph is not None:
        e_steps = max(3, min(args.steps, 20))
        eager_ms = reduce_max(time_steps(chain, e_steps, stream, None), dist, device) / e_steps
        eager = {"ms_per_step": round(eager_ms, 4),
                 "value": round(aggregate_gbs(n_gpus, total_bytes, 1, eager_ms), 1), "unit": "GB/s",
                 "steps": e_steps,
                 "note": "eager launches from the Python harness, one ctypes call per launch (host-bound)"}

    # BASELINE config 1 beside the default workload: the 28-block chain at 1024 tokens, batch 1
    cfg1 = None
    if args.workload == "cfg2" and rank == 0 and not args.no_other_ops:
        cfg1 = cfg1_step(ops, device, args.steps, peak)

    # per-op device times (graph replay of each op type alone) -> roofline
    ops_t = per_op_times(chain, {k: v * CFG["blocks"] for k, v in lpb.items()}, 50)
    kernels = {}
    for name, mean_ms in ops_t.items():
        per_launch = per_block[name] / lpb[name]
        gbs = per_launch / (mean_ms * 1e-3) / 1e9
        kernels[name] = {"launches_per_step": lpb[name] * CFG["blocks"], "us": round(mean_ms * 1e3, 2),
                         "bytes_per_launch": int(per_launch), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3),
                         "share": None}
    tot = sum(v["us"] * v["launches_per_step"] for v in kernels.values())
    for v in kernels.values():
        v["share"] = round(v["us"] * v["launches_per_step"] / tot, 3)
    dom = max(kernels, key=lambda k: kernels[k]["share"])
    dk = kernels[dom]

    # end to end through the C ABI with host buffers: pinned hidden + modulation in, hidden out
    h_in = torch.empty((chain.R, chain.D), dtype=torch.bfloat16).pin_memory()
    m_in = torch.empty_like(chain.mod_raw, device="cpu").pin_memory()
    h_out = torch.empty((chain.R, chain.D), dtype=torch.bfloat16).pin_memory()
    h_in.copy_(chain.sets[0]["hidden"].cpu())
    m_in.copy_(chain.mod_raw.cpu())
    e2e_steps = max(3, min(args.steps, 50))
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e2e_steps):
        chain.sets[0]["hidden"].copy_(h_in, non_blocking=True)
        chain.mod_raw.copy_(m_in, non_blocking=True)
        chain.timestep(stream.cuda_stream)
        if graph is not None:
            graph.replay()
        else:
            chain.blocks(stream.cuda_stream)
        h_out.copy_(chain.sets[(CFG["blocks"] - 1) % NSETS]["hidden"], non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    e2e_serial_ms = reduce_max(a.elapsed_time(b) / e2e_steps, dist, device)
    e2e_ms = reduce_max(e2e_pipelined(chain, graph, e2e_steps, h_in, m_in, h_out), dist, device)
    h2d = h_in.numel() * 2 + m_in.numel() * 2 + (0 if args.impl == "anima" else CFG["ts_dim"] * 2)
    d2h = h_out.numel() * 2

    # the same step through the opt-in fused entry points (anima only)
    fused = None
    if args.impl == "anima" and not args.eager:
        fgraph = capture(lambda s: chain.blocks_fused(s))
        for _ in range(2):
            fgraph.replay()
        torch.cuda.synchronize()
        fsteps = max(3, min(args.steps, 50))
        fms = reduce_max(time_steps(chain, fsteps, stream, fgraph), dist, device) / fsteps
        del fgraph
        fused = {"ms_per_step": round(fms, 4), "launches_per_step": chain.launches_fused + 1,
                 "speedup_vs_drop_in": round(ms_per_step / fms, 3),
                 "note": "same step with mod+=temb and the gate copy folded into the adaLN/residual-gate norms, "
                         "QK RMSNorm+RoPE fused, and each block's closing residual gate fused with the next "
                         "block's adaLN (opt-in entry points); fewer bytes cross HBM"}

    headline = None
    if not args.no_headline and rank == 0:
        headline = headline_kernels(ops, device, peak)
    other = None
    if not args.no_other_ops and rank == 0:
        other = other_ops(ops, device, peak)

    cpu = None
    if not args.no_cpu_baseline and rank == 0:
        n_cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        v1, sample1 = cpu_baseline_sample(blocks=2, threads=1)
        vn, samplen = cpu_baseline_sample(blocks=8 if n_cores >= 8 else 2, threads=n_cores)
        cpu_model = None
        try:
            with open("/proc/cpuinfo") as f:
                cpu_model = next((l.split(":", 1)[1].strip() for l in f if l.startswith("model name")), None)
        except OSError:
            pass
        cpu = {"value": round(vn, 3), "unit": "GB/s", "cores": n_cores, "kind": "port", "sample": samplen,
               "cpu_model": cpu_model, "host_threads": os.cpu_count(),
               "single_thread": {"value": round(v1, 3), "cores": 1, "sample": sample1},
               "note": "plain C host loop of the chain's ops (oracle/hostloop.c, gcc -O3 -march=native -fopenmp, "
                       "built on this host); the reference itself has no CPU implementation of these ops"}

    used_graph = graph is not None
    del graph  # release the captured graph before the process group goes away
    launches_per_step = CFG["blocks"] * chain.launches_per_block + 1
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": n_gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak" if args.workload == "cfg2" else "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) activations, N(0,0.1) modulation and temb, 1+N(0,0.02) norm weights, "
                "t~U(0,1)*1000; GEMM/attention outputs are resident synthetic tensors",
        "config": {"workload": ("cfg2: 1024x1024 image -> 4096 tokens x CFG 2, 28-block DiT elementwise chain"
                                if args.workload == "cfg2" else
                                f"cfg5: 8 images at 1536x1536 -> 9216 tokens x CFG 2, 28-block DiT elementwise "
                                f"chain, {8 // n_gpus} image pair(s) per GPU"),
                   "rows": chain.R, "hidden": chain.D, "heads": chain.H, "head_dim": chain.HD, "mlp": chain.M,
                   "text_tokens": chain.T, "blocks": chain.NB, "timestep_dim": CFG["ts_dim"],
                   "algorithmic_bytes_per_step": total_bytes,
                   "l2": f"{NSETS} rotating activation sets, each >> 126 MB L2 (no flush)",
                   "timing": ("CUDA graph replay of the 28 blocks + eager timestep launch per step"
                              if used_graph else "eager launches"),
                   "parallelism": (f"replicas x{n_gpus} (rows independent; no collective on the data path)"
                                   if args.workload == "cfg2" else
                                   f"{8 // n_gpus} of 8 image pairs per GPU x{n_gpus} (no collective on the data path)")},
        "e2e": {"value": round(aggregate_gbs(n_gpus, total_bytes, 1, e2e_ms), 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "method": "pinned host buffers; step k+1's upload and step k's download overlap step k's "
                          "compute on a copy stream through device staging buffers",
                "serial": {"value": round(aggregate_gbs(n_gpus, total_bytes, 1, e2e_serial_ms), 1),
                           "ms_per_step": round(e2e_serial_ms, 4),
                           "method": "upload, step, download back to back on one stream"}},
        "gpu_launches": launches_per_step * args.steps if args.impl == "anima" else 0,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": dk["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": dk["frac"], "peak_kind": peak_kind,
                     "traffic": dram_traffic(dom) if args.impl == "anima" else None,
                     "bytes_per_launch": dk["bytes_per_launch"], "us_per_launch": dk["us"]},
        "chain_frac_of_peak": round(value / n_gpus / peak, 3),
        "cpu_baseline": cpu,
        "clocks": clk,
        # compact per-case figures ({us, frac}); the full record is in the DESIGN tables
        "other_ops": ({k: {"us": v["us"], "frac": v["frac"]} for k, v in other.items()} if other else None),
        "kernels": {k: {"us": v["us"], "frac": v["frac"], "share": v["share"], "launches": v["launches_per_step"]}
                    for k, v in kernels.items()},
        "fused_step": fused,
        "eager_step": eager,
        "cfg1": cfg1,
    }
    if args.impl == "reference":
        line["impl"] = "reference"
        line["reference_kind"] = ("the reference's own CUDA kernels (src/kernels/*.cu compiled unchanged for sm_100a, "
                                  "oracle/_ref) through their kernels.h launchers; host-side timestep sinusoid + "
                                  "synchronous upload as transformer.cpp:182-200")
        line["gpu_launches"] = 0
        # this run is the reference's own implementation of the path (its CUDA kernels: it has
        # no CPU implementation of these ops); the CPU restatement's figure moves beside it
        line["cpu_restatement"] = line["cpu_baseline"]
        line["cpu_baseline"] = {"value": line["value"], "unit": "GB/s", "kind": "reference", "cores": 1,
                                "sample": f"{args.steps} full {args.workload} steps: the reference's kernels.h launchers driven "
                                          "from one host thread, kernels on the B200",
                                "note": "the reference implements this path only as CUDA kernels"}
    # last, so that it survives in any tail of the output: every in-scope kernel at the
    # headline [4096, 2048] shape, the metric BASELINE.json names
    line["headline_4096x2048"] = headline
    if rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
