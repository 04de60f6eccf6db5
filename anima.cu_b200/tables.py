"""Host-side RoPE table builders: the inputs of the RoPE kernels.

The reference builds these on the host once per resolution / sequence length and uploads
them; the kernels consume them unchanged. These numpy versions follow the same formulas:

- cosmos_rope_tables: transformer.cpp:213-318. Head dim split t/h/w = HD-2*(HD//6*2),
  HD//6*2, HD//6*2 (44/42/42 at HD = 128), NTK-scaled thetas (h, w: 1e4 * 4^(d/(d-2));
  t: 1e4), per-axis frequencies 1/theta^(2i/d), row = [t, h, w] halves repeated twice,
  rounded to bf16.
- standard_rope_tables: qwen3.cpp:12-23 (theta 1e6) and llm_adapter.cpp:11-22 (theta 1e4),
  fp32 [T, HD/2].

Every fp32 step of the reference is reproduced in fp32; cos/sin/pow are evaluated in
double and rounded once, which gives the correctly rounded fp32 value (the reference's
glibc cosf/sinf/powf differ from that by at most one fp32 ulp in rare cases, which bf16
rounding almost never exposes).
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def _bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _powf(base: float, e: np.ndarray) -> np.ndarray:
    return np.power(np.float64(base), np.asarray(e, np.float32).astype(np.float64)).astype(np.float32)


def _axis_freqs(dim: int, theta: np.float32) -> np.ndarray:
    i = np.arange(dim // 2)
    expo = (2 * i).astype(np.float32) / f32(dim)
    return (f32(1.0) / _powf(float(theta), expo)).astype(np.float32)


def cosmos_rope_tables(pe_t: int, pe_h: int, pe_w: int, HD: int = 128):
    """bf16 bit patterns cos, sin of shape [pe_t*pe_h*pe_w, HD]."""
    dim_h = (HD // 6) * 2
    dim_w = dim_h
    dim_t = HD - dim_h - dim_w
    h_ntk = _powf(4.0, np.float32(f32(dim_h) / f32(dim_h - 2)))
    w_ntk = _powf(4.0, np.float32(f32(dim_w) / f32(dim_w - 2)))
    t_ntk = _powf(1.0, np.float32(f32(dim_t) / f32(dim_t - 2)))
    ft = _axis_freqs(dim_t, f32(10000.0) * t_ntk)
    fh = _axis_freqs(dim_h, f32(10000.0) * h_ntk)
    fw = _axis_freqs(dim_w, f32(10000.0) * w_ntk)
    t, h, w = np.meshgrid(np.arange(pe_t), np.arange(pe_h), np.arange(pe_w), indexing="ij")
    t, h, w = (a.reshape(-1, 1).astype(np.float32) for a in (t, h, w))
    ang = np.concatenate([t * ft, h * fh, w * fw], axis=1).astype(np.float32)
    ang = np.concatenate([ang, ang], axis=1)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    return _bf16(c), _bf16(s)


def standard_rope_tables(T: int, HD: int, theta: float):
    """fp32 cos, sin of shape [T, HD/2]."""
    d = np.arange(HD // 2)
    freq = (f32(1.0) / _powf(float(f32(theta)), (2 * d).astype(np.float32) / f32(HD))).astype(np.float32)
    ang = (np.arange(T, dtype=np.float32).reshape(-1, 1) * freq).astype(np.float32)
    return (np.cos(ang.astype(np.float64)).astype(np.float32),
            np.sin(ang.astype(np.float64)).astype(np.float32))
