"""TEST INFRASTRUCTURE ONLY: ctypes bindings of hostloop.c, the plain C host loop that
bench.py times as its CPU baseline.

`load()` compiles hostloop.c with `gcc -O3 -march=native -fopenmp` for the machine it
runs on (the GPU box's host CPU may differ from the build container's, so the library is
built where it is used, keyed by CPU model and compiler flags) and returns the bound
library. Nothing in the product imports this module.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import platform
import subprocess
from ctypes import c_float, c_int, c_int64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(_HERE, "hostloop.c")
CFLAGS = ["-O3", "-march=native", "-fopenmp", "-fPIC", "-shared", "-std=c11"]

P, I32, I64, F32 = c_void_p, c_int, c_int64, c_float
_SIGS = {
    "hostloop_set_threads": (I32,),
    "hostloop_add": (P, P, P, I64),
    "hostloop_adaln_layernorm": (P, P, P, P, I64, I32, F32),
    "hostloop_residual_gate_adaln": (P, P, P, P, P, P, I64, I32, F32),
    "hostloop_rms_norm": (P, P, P, I64, I32, F32),
    "hostloop_rope_cosmos": (P, P, P, I32, I32, I32, I32),
    "hostloop_gelu_tanh": (P, P, I64),
    "hostloop_residual_gate_bcast": (P, P, P, P, I64, I32),
}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def _lib_path() -> str:
    with open(SRC, "rb") as f:
        key = hashlib.sha1(f.read() + " ".join(CFLAGS).encode() + cpu_model().encode()).hexdigest()[:12]
    return os.path.join(_HERE, "_cpu", f"libhostloop-{key}.so")


def load():
    """Build (once per source, flags and CPU model) and bind the host-loop library."""
    path = _lib_path()
    if not os.path.exists(path):
        os.makedirs(os.path.dirname(path), exist_ok=True)
        tmp = f"{path}.{os.getpid()}.tmp"
        subprocess.run(["gcc", *CFLAGS, "-o", tmp, SRC, "-lm"], check=True)
        os.replace(tmp, path)
    lib = ctypes.CDLL(path)
    for name, argtypes in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = None
    lib.hostloop_max_threads.restype = c_int
    lib.hostloop_max_threads.argtypes = []
    return lib


def flags() -> str:
    return "gcc " + " ".join(CFLAGS[:3])
