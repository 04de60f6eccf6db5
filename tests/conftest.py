"""Shared test setup: import paths, the `gpu` marker, and fixtures for the three
implementations a parity test compares -- the B200 library (through its C ABI), the
reference's own CUDA kernels (oracle/_ref, GPU) and the CPU restatement (oracle/).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("anima.cu_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    return O


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def anima(cuda):
    import anima_b200

    return anima_b200


@pytest.fixture(scope="session")
def ref(cuda):
    import refkernels

    if not refkernels.reference_available():
        pytest.fail("oracle/_ref/libref_kernels.so is missing (build it with `make -C oracle ref`)")
    return refkernels.load_reference()


@pytest.fixture
def rng(request):
    # A stable per-test seed, so a failure reproduces with the same inputs.
    import zlib

    seed = zlib.crc32(request.node.nodeid.encode())
    return np.random.default_rng(seed)
