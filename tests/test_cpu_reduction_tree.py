"""The B200 row kernels reproduce the reference's CTA reduction order with a different
thread organisation (anima.cu_b200/csrc/common.cuh, rownorm.cu). This CPU test emulates
both lane schedules in fp32 and requires them to equal, bit for bit, the oracle's literal
replay of the reference tree (warp shfl_down tree, then warp 0 over the per-warp sums,
src/cuda_utils.cuh:46-50, src/kernels/layer_norm.cu:7-19) on random rows of every
supported width:

* segment kernels: one 64-element segment (one reference warp) per lane, the warp tree as
  in-register adds, the cross-warp level as lane XORs (row_seg / seg_tree / seg_cross);
* transposed butterfly: a team of LPR lanes holding chunks l + LPR*k, lane XORs 4/2/1 with
  halving of the live values, then the cross-warp level (ref_pair_tree_sum; used by the
  small-row RMSNorm and the fused QK-norm + RoPE).
"""
import ctypes

import numpy as np
import pytest

import oracle as O

f32 = np.float32
_ref = O.lib.oracle_ref_block_sum
_ref.restype = ctypes.c_float
_ref.argtypes = [ctypes.c_void_p, ctypes.c_int]


def reference_sum(pairs):
    d2 = pairs.size
    T = O.lib.oracle_ref_row_threads(2 * d2)
    per = np.zeros(T, f32)
    per[:d2] = pairs
    return f32(_ref(per.ctypes.data_as(ctypes.c_void_p), T))


def segment_schedule(pairs):
    nw = pairs.size // 32

    def lane_tree(p):  # offsets 16, 8, 4, 2, 1 inside one reference warp
        a = [f32(p[r] + p[r + 16]) for r in range(16)]
        b = [f32(a[r] + a[r + 8]) for r in range(8)]
        c = [f32(b[r] + b[r + 4]) for r in range(4)]
        d = [f32(c[0] + c[2]), f32(c[1] + c[3])]
        return f32(d[0] + d[1])

    s = [lane_tree(pairs[32 * w:32 * w + 32]) for w in range(nw)]
    for off in (16, 8, 4, 2, 1):
        if off < nw:
            s = [f32(s[w] + s[w ^ off]) for w in range(nw)]
    assert len({float(v) for v in s}) == 1  # every lane of the team holds the total
    return s[0]


def butterfly_schedule(pairs, LPR, K):
    lanes = range(LPR)
    cur = {l: [[pairs[4 * (l + LPR * k) + j] for j in range(4)] for k in range(K)] for l in lanes}
    m = K
    for bit in (2, 1, 0):
        nxt = {}
        for l in lanes:
            p = l ^ (1 << bit)
            if m > 1:
                up, pup = (l >> bit) & 1, (p >> bit) & 1
                nxt[l] = [[f32((cur[l][i + m // 2][j] if up else cur[l][i][j]) +
                               (cur[p][i][j] if pup else cur[p][i + m // 2][j])) for j in range(4)]
                          for i in range(m // 2)]
            else:
                nxt[l] = [[f32(cur[l][0][j] + cur[p][0][j]) for j in range(4)]]
        cur, m = nxt, max(m // 2, 1)
    s = {l: f32(f32(cur[l][0][0] + cur[l][0][2]) + f32(cur[l][0][1] + cur[l][0][3])) for l in lanes}
    lg_g, lg_k, nw = {1: 0, 2: 1, 4: 2}[LPR // 8], {1: 0, 2: 1, 4: 2, 8: 3}[K], (LPR // 8) * K
    for i in range(4, -1, -1):
        if (1 << i) >= nw:
            continue
        lb = 3 + i if i < lg_g else (i - lg_g) + 3 - lg_k
        s = {l: f32(s[l] + s[l ^ (1 << lb)]) for l in lanes}
    assert len({float(v) for v in s.values()}) == 1
    return s[0]


def _rows(rng, d2, n=40):
    for _ in range(n):
        yield (rng.standard_normal(d2) * 10.0 ** rng.integers(-3, 4)).astype(f32)


@pytest.mark.parametrize("D", [64, 128, 256, 512, 1024, 2048])
def test_segment_schedule_matches_reference_tree(D):
    rng = np.random.default_rng(D)
    for p in _rows(rng, D // 2):
        assert segment_schedule(p).tobytes() == reference_sum(p).tobytes()


@pytest.mark.parametrize("LPR,K", [(8, 1), (8, 2), (8, 4), (8, 8), (16, 8), (32, 8)])
def test_butterfly_schedule_matches_reference_tree(LPR, K):
    rng = np.random.default_rng(LPR * 10 + K)
    for p in _rows(rng, 4 * LPR * K, n=15):
        assert butterfly_schedule(p, LPR, K).tobytes() == reference_sum(p).tobytes()


def test_a_different_order_is_detected():
    """Sanity: a plain left-to-right sum does differ from the reference tree."""
    rng = np.random.default_rng(1)
    diffs = 0
    for p in _rows(rng, 1024, n=20):
        seq = f32(0)
        for v in p:
            seq = f32(seq + v)
        diffs += seq.tobytes() != reference_sum(p).tobytes()
    assert diffs > 0
