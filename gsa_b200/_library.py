# SPDX-License-Identifier: Apache-2.0
"""Load the in-tree native libraries (mirror of GSA ``gsa/_library.py``).

``load(name)`` opens ``gsa_b200/_native/<name>.so``.  There is no CPU
fallback: a missing library raises immediately.
"""

import ctypes
from pathlib import Path

import torch

NATIVE_DIR = Path(__file__).resolve().parent / "_native"
_loaded = {}


def path(name):
    return NATIVE_DIR / (name + ".so")


def load(name):
    """Return the ``ctypes.CDLL`` of ``_native/<name>.so`` (cached)."""
    if name in _loaded:
        return _loaded[name]
    p = path(name)
    if not p.is_file():
        raise RuntimeError(
            "Compile gsa_b200 first: python -m gsa_b200._build "
            "(needs nvcc; builds sm_100a libraries in gsa_b200/_native)"
        )
    lib = ctypes.CDLL(str(p))
    _loaded[name] = lib
    return lib


_cuda_ready = False


def current_stream():
    """``(device index, raw cudaStream_t)`` of the current CUDA stream: what
    ``torch.cuda.current_device()`` and ``torch.cuda.current_stream()
    .cuda_stream`` return, read through torch's C accessors once CUDA is
    initialised (the public calls re-check the CUDA state on every call, which
    dominates the host cost of a small query)."""
    global _cuda_ready
    if not _cuda_ready:
        torch.cuda.init()
        _cuda_ready = True
    device = torch._C._cuda_getDevice()
    return device, torch._C._cuda_getCurrentRawStream(device)


def stream():
    """Raw handle of the current CUDA stream."""
    return current_stream()[1]


def launch_counter():
    """Kernel launches the native libraries have enqueued in this process
    (both libraries' counters added; a replayed CUDA graph adds nothing)."""
    total = 0
    for name in ("gsa_bvh", "reference_queries"):
        lib = load(name)
        v = ctypes.c_ulonglong()
        lib.launch_counter.argtypes = [ctypes.POINTER(ctypes.c_ulonglong)]
        lib.launch_counter.restype = ctypes.c_int
        lib.launch_counter(ctypes.byref(v))
        total += v.value
    return total
