# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of the prefix-BVH library (drop-in for GSA ``gsa/runtime.py``).

``Tree(x, prefix=False, leaf=16)`` indexes a borrowed CUDA FP32 ``(N, 3)``
tensor; ``Tree.query`` is the exact 3NN query and ``Tree.ball`` the exact
ordered radius query, both on the current CUDA stream.  Contract violations
raise ``ValueError`` and native error codes raise ``RuntimeError``, under the
same conditions as ``gsa/runtime.py:44-178``; ``pool_memory`` reports the
native pool's high-water marks (``gsa/runtime.py:34-41``).
"""

import ctypes
import math

import torch

# _stream: the current raw stream, also used as runtime._stream by the
# forest and hierarchy modules
from ._library import current_stream, load, stream as _stream

lib = load("gsa_bvh")
_ptr, _int = ctypes.c_void_p, ctypes.c_int
_u64p, _intp = ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int)
for _name, _args in {
    "build_bvh": [_ptr, _int, _int, _int, ctypes.POINTER(_ptr), _ptr],
    "query_bvh": [_ptr, _ptr, _int, _int, _int, _ptr, _ptr, _ptr, _ptr],
    "query_ball_bvh": [_ptr, _ptr, _int, _int, _int, ctypes.c_float, _int, _ptr, _ptr, _ptr],
    "query_bvh_unordered": [_ptr, _ptr, _int, _int, _int, _ptr, _ptr, _ptr, _ptr],
    "query_ball_bvh_unordered": [_ptr, _ptr, _int, _int, _int, ctypes.c_float, _int, _ptr, _ptr, _ptr],
    "free_bvh": [_ptr, _int, _ptr],
    "pool_memory": [_u64p, _u64p],
    "pool_reset_peak": [],
    "set_pool_mode": [_int],
    "bvh_info": [_ptr, _intp, _intp, _intp, _intp],
}.items():
    getattr(lib, _name).argtypes = _args
    getattr(lib, _name).restype = _int

_FLT_MAX = torch.finfo(torch.float32).max
_pool_device = None


def check(code):
    if code:
        raise RuntimeError(f"BVH error {code}")


def pool_memory():
    used, reserved = ctypes.c_uint64(), ctypes.c_uint64()
    check(lib.pool_memory(ctypes.byref(used), ctypes.byref(reserved)))
    return {
        "native_pool_used_peak_bytes": used.value,
        "native_pool_reserved_peak_bytes": reserved.value,
    }


def pool_reset_peak():
    check(lib.pool_reset_peak())


def set_pool_mode(enabled):
    check(lib.set_pool_mode(int(bool(enabled))))


def prefix_sizes(n):
    """Supports a prefix index over ``n`` points serves: ``n, n//4, n//16,
    n//64`` (``docs/api.md`` "Index reuse")."""
    return [n >> (2 * level) for level in range(4)]


def support_rows(q, x):
    """Whether the query tensor starts at the support tensor's first row
    (its rows are then the support's points, which the query kernels walk
    in the tree's leaf order); other query sets take the ``_unordered``
    entries, which walk them in their own Morton order.  Either way the
    results are the same; only the speed differs."""
    return q.data_ptr() == x.data_ptr()


def _is_points(x):
    return (
        isinstance(x, torch.Tensor)
        and x.is_cuda
        and x.is_contiguous()
        and x.dtype == torch.float32
        and x.ndim == 2
        and x.shape[1] == 3
    )


def _is_rows(t, like, rows, width, dtype):
    return (
        t.is_cuda
        and t.get_device() == like.get_device()
        and t.is_contiguous()
        and t.dtype == dtype
        and t.shape == (rows, width)
    )


class Tree:
    """Exact query index over a borrowed support tensor."""

    def __init__(self, x, prefix=False, leaf=16):
        global _pool_device
        if not (
            _is_points(x)
            and x.shape[0] > 0
            and x.get_device() == current_stream()[0]
            and isinstance(leaf, int)
            and leaf >= 1
        ):
            raise ValueError(
                "Tree requires nonempty contiguous CUDA FP32 (N,3) on the current device and a positive leaf size"
            )
        if _pool_device not in (None, x.device.index):
            raise ValueError("The native allocator supports one CUDA device per process")
        _pool_device = x.device.index
        self.x = x
        self.prefix = prefix
        self.device, self.stream = current_stream()
        self.sizes = prefix_sizes(x.shape[0]) if prefix else None
        self.ptr = _ptr()
        self.fallback = torch.zeros(1, device=x.device, dtype=torch.int32)
        check(lib.build_bvh(x.data_ptr(), len(x), int(prefix), leaf, ctypes.byref(self.ptr), self.stream))

    def level(self, m):
        """Bounds level for support prefix ``m`` (-1 for a plain tree)."""
        return self.sizes.index(m) if self.prefix else -1

    def _usable_here(self):
        return bool(self.ptr) and current_stream() == (self.device, self.stream)

    def _check_query(self, q, m, idx, width):
        if not (
            self._usable_here()
            and _is_points(q)
            and q.get_device() == self.device
            and _is_rows(idx, q, q.shape[0], width, torch.int32)
            and 1 <= m <= self.x.shape[0]
        ):
            raise ValueError("Invalid query buffers, support length, or tree lifetime/device/stream")

    def query(self, q, m, d, idx):
        """Exact 3NN of ``q`` against support IDs ``< m``; ``d``/``idx`` (Q, 3)."""
        self._check_query(q, m, idx, 3)
        nq = q.shape[0]
        if m < 3 or not _is_rows(d, q, nq, 3, torch.float32):
            raise ValueError("3NN requires at least 3 supports and FP32 (Q,3) distances")
        if nq:
            fn = lib.query_bvh if support_rows(q, self.x) else lib.query_bvh_unordered
            check(
                fn(
                    self.ptr, q.data_ptr(), nq, m, self.level(m), d.data_ptr(),
                    idx.data_ptr(), self.fallback.data_ptr(), self.stream,
                )
            )
        return d, idx

    def ball(self, q, m, r, ns, idx):
        """First ``ns`` support IDs ``< m`` within radius ``r`` per query."""
        self._check_query(q, m, idx, ns)
        if not (isinstance(ns, int) and 1 <= ns <= 32 and math.isfinite(r) and 0 <= r <= _FLT_MAX):
            raise ValueError("Radius query requires K in [1,32] and finite nonnegative FP32 radius")
        nq = q.shape[0]
        if nq:
            fn = lib.query_ball_bvh if support_rows(q, self.x) else lib.query_ball_bvh_unordered
            check(
                fn(
                    self.ptr, q.data_ptr(), nq, m, self.level(m), r, ns,
                    idx.data_ptr(), self.fallback.data_ptr(), self.stream,
                )
            )
        return idx

    def close(self):
        if not self.ptr:
            return
        if current_stream() != (self.device, self.stream):
            raise ValueError("Close the tree on its original device and stream")
        check(lib.free_bvh(self.ptr, 1, self.stream))
        self.ptr = _ptr()
