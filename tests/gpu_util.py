"""Helpers for the GPU parity tests: numpy <-> device copies of bf16 bit patterns and a
comparison report. bf16 tensors live on the device as int16 storage (the kernels take raw
pointers, so the storage dtype only has to have the right width)."""
import numpy as np
import torch

import oracle as O


def dev(a: np.ndarray, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(device)


def host(t: torch.Tensor, dtype=np.uint16) -> np.ndarray:
    a = t.detach().cpu().numpy()
    return a.view(dtype) if a.dtype.itemsize == np.dtype(dtype).itemsize else a.astype(dtype)


def empty_bf16(shape, device="cuda") -> torch.Tensor:
    return torch.empty(shape, dtype=torch.int16, device=device)


def stream_ptr():
    return torch.cuda.current_stream().cuda_stream


def compare(got: np.ndarray, want: np.ndarray):
    """(exact fraction, max ulp distance, fraction within one ulp of max(|want|, 2^-12))."""
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    assert got.shape == want.shape
    if got.size == 0:
        return 1.0, 0, 1.0
    d = O.ulp_distance(got, want)
    within = O.within_one_ulp(got, want)
    return float(np.mean(d == 0)), int(d.max()), float(np.mean(within))


def assert_bit_exact(got, want, what=""):
    ex, mx, _ = compare(got, want)
    assert mx == 0, f"{what}: not bit-exact ({ex:.6f} exact, max {mx} ulp)"


def assert_one_ulp(got, want, what=""):
    ex, mx, w1 = compare(got, want)
    assert w1 == 1.0, f"{what}: {1 - w1:.3e} of elements beyond 1 bf16 ulp (exact {ex:.6f}, max {mx} ulp)"
