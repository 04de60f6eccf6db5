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


def assert_bit_exact_or_reference_race(got, ref_out, oracle_fn, what="", rerun=None):
    """Bit-exact against a kernel of the reference's layer_norm.cu, allowing for that file's
    one race. Its CTA reduction helper (layer_norm.cu:7-19) returns shared[0] with no barrier
    after the read, and its kernels call it twice in a row (the sum, then the sum of squares):
    warp 0 can write its next partial into shared[0] before a slower warp has read the first
    total, and that warp then normalises its elements with a wrong mean (rarely; errors on a
    few dozen elements). A mismatch is accepted only where it is that: on few elements, with
    our value within one ulp of the race-free CPU restatement (oracle_fn()), and then either
    a fresh run of the reference kernel on the same inputs (rerun(), when given: it returns
    that run's output) is bit-exact with ours, or the racing run's values mostly miss the
    restatement (a wrong mean can leave an element near zero within one ulp by chance: one
    of a warp's 128 elements did so in one run; a wrong mean close to the true one leaves
    more, hence the fresh run)."""
    got = np.asarray(got).reshape(-1)
    ref_out = np.asarray(ref_out).reshape(-1)
    diff = np.nonzero(got != ref_out)[0]
    if diff.size == 0:
        return
    assert diff.size <= max(512, got.size // 1000), f"{what}: {diff.size} elements differ from the reference"
    want = np.asarray(oracle_fn()).reshape(-1)
    ours_ok = O.within_one_ulp(got[diff], want[diff])
    if rerun is not None and ours_ok.all():
        for _ in range(2):
            if np.array_equal(got, np.asarray(rerun()).reshape(-1)):
                return
    theirs_ok = O.within_one_ulp(ref_out[diff], want[diff])
    assert ours_ok.all() and theirs_ok.mean() < 0.5, (
        f"{what}: {diff.size} elements differ from the reference, and not as its reduction race would make them "
        f"({int(ours_ok.sum())} of ours and {int(theirs_ok.sum())} of the reference's follow the CPU restatement)")


def fresh_run(launch, shape):
    """A `rerun` for assert_bit_exact_or_reference_race: launch(out) runs the reference kernel
    once more on the same inputs into a new buffer `out` of `shape`; returns its host copy."""
    def run():
        out = empty_bf16(shape)
        launch(out)
        torch.cuda.synchronize()
        return host(out)
    return run
