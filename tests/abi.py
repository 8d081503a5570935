# SPDX-License-Identifier: Apache-2.0
"""Thin ctypes calls of the C ABI for the GPU parity tests (torch tensors in,
raw device pointers through ``include/gsa_bvh.h`` / ``reference_queries.h``)."""

import ctypes

import torch

from gsa_b200 import _library

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def bvh_lib(name="gsa_bvh"):
    lib = _library.load(name)
    lib.build_bvh.argtypes = [P, I, I, I, ctypes.POINTER(P), P]
    lib.query_bvh.argtypes = [P, P, I, I, I, P, P, P, P]
    lib.query_ball_bvh.argtypes = [P, P, I, I, I, F, I, P, P, P]
    lib.free_bvh.argtypes = [P, I, P]
    lib.build_bvh_batch.argtypes = [P, P, I, I, I, ctypes.POINTER(P), P]
    lib.query_ball_bvh_batch.argtypes = [P, P, P, P, P, I, I, F, I, P, P, P]
    lib.query_bvh_batch.argtypes = [P, P, P, P, P, I, I, P, P, P, P]
    lib.coords_mismatch_strided.argtypes = [I, P, ctypes.c_longlong, P, ctypes.c_longlong, ctypes.c_longlong, P, I, P]
    lib.reuse_rows_batch.argtypes = [I, P, ctypes.c_longlong, I, P, I, I, P, ctypes.c_longlong, P, P]
    LL = ctypes.c_longlong
    lib.reuse_prefix_batch.argtypes = [I, P, LL, P, LL, LL, LL, P, LL, I, I, I, P, LL, P, P, P]
    lib.reuse_prefix_stages.argtypes = [I, I, P, LL, P, LL, P, P, P, P, I, P, I, P, P, P, P, P]
    lib.coords_mismatch.argtypes = [I, P, P, P, P, P]
    lib.reuse_rows.argtypes = [I, P, P, I, I, I, P, P, P]
    lib.gather_rows.argtypes = [P, I, I, I, P, P]
    lib.session_lookup.argtypes = [I, P, P, P, I, P, I, I, I, P, P, P, P]
    lib.query_bvh_unordered.argtypes = [P, P, I, I, I, P, P, P, P]
    lib.query_ball_bvh_unordered.argtypes = [P, P, I, I, I, F, I, P, P, P]
    lib.fps_order.argtypes = [I, I, P, P, P, P]
    lib.furthest_point_sample.argtypes = [I, I, I, P, P, P, P]
    lib.bvh_info.argtypes = [P] + [ctypes.POINTER(I)] * 4
    lib.pool_memory.argtypes = [ctypes.POINTER(ctypes.c_uint64)] * 2
    return lib


def ref_lib():
    lib = _library.load("reference_queries")
    lib.ball.argtypes = [I, I, I, F, I, P, P, P, P]
    lib.nn3.argtypes = [I, I, I, P, P, P, P, P]
    return lib


def stream():
    return torch.cuda.current_stream().cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


class Handle:
    def __init__(self, lib, x, prefix=1, leaf=16):
        self.lib, self.x = lib, x
        self.h = P()
        self.code = lib.build_bvh(ptr(x), len(x), prefix, leaf, ctypes.byref(self.h), stream())

    def ball(self, q, m, level, r, ns, out=None, fallback=None, unordered=False):
        out = torch.full((len(q), ns), -7, dtype=torch.int32, device="cuda") if out is None else out
        fb = torch.zeros(1, dtype=torch.int32, device="cuda") if fallback is None else fallback
        fn = self.lib.query_ball_bvh_unordered if unordered else self.lib.query_ball_bvh
        code = fn(self.h, ptr(q), len(q), m, level, r, ns, ptr(out), ptr(fb), stream())
        return code, out, fb

    def knn(self, q, m, level, fallback=None, unordered=False):
        d = torch.full((len(q), 3), -1.0, device="cuda")
        ix = torch.full((len(q), 3), -7, dtype=torch.int32, device="cuda")
        fb = torch.zeros(1, dtype=torch.int32, device="cuda") if fallback is None else fallback
        fn = self.lib.query_bvh_unordered if unordered else self.lib.query_bvh
        code = fn(self.h, ptr(q), len(q), m, level, ptr(d), ptr(ix), ptr(fb), stream())
        return code, d, ix, fb

    def free(self, async_free=1):
        code = self.lib.free_bvh(self.h, async_free, stream())
        self.h = P()
        return code


def scan_ball(q, x, r, ns, init=None, b=1):
    lib = ref_lib()
    m = q.shape[-2]
    n = x.shape[-2]
    out = (torch.full((b, m, ns), -5, dtype=torch.int32, device="cuda") if init is None else init.clone())
    code = lib.ball(b, n, m, r, ns, ptr(q), ptr(x), ptr(out), stream())
    return code, out


def scan_nn3(q, x, b=1):
    lib = ref_lib()
    n = q.shape[-2]
    m = x.shape[-2]
    d = torch.full((b, n, 3), -1.0, device="cuda")
    ix = torch.full((b, n, 3), -7, dtype=torch.int32, device="cuda")
    code = lib.nn3(b, n, m, ptr(q), ptr(x), ptr(d), ptr(ix), stream())
    return code, d, ix
