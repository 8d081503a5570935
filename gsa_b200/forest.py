# SPDX-License-Identifier: Apache-2.0
"""Batched multi-scene index: B independent prefix trees in one object.

The reference API serves one scene per call.  Batched inference over many
small scenes (e.g. 64 room scenes of 24,000 points) would leave most of a
B200's 148 SMs idle per call; ``Forest`` builds all trees with one launch per
build step and answers a query stage of every scene with one launch.
Results per scene are identical to ``Tree`` on that scene.

Layout: the supports of all scenes are concatenated into one contiguous
``(N_total, 3)`` float32 CUDA tensor with host offsets ``seg`` (B+1 values);
the queries of a stage are concatenated the same way with offsets ``qseg``.
Tree ``i`` answers its queries against its own prefix of size
``n_i >> (2 * level)`` (``n_i`` for ``level = -1``).
"""

import ctypes

import torch

from . import runtime as er

lib = er.lib
_ptr, _int = ctypes.c_void_p, ctypes.c_int
lib.build_bvh_batch.argtypes = [_ptr, _ptr, _int, _int, _int, ctypes.POINTER(_ptr), _ptr]
lib.build_bvh_batch.restype = _int
lib.query_ball_bvh_batch.argtypes = [_ptr, _ptr, _ptr, _ptr, _int, ctypes.c_float, _int, _ptr, _ptr, _ptr]
lib.query_ball_bvh_batch.restype = _int
lib.query_bvh_batch.argtypes = [_ptr, _ptr, _ptr, _ptr, _int, _ptr, _ptr, _ptr, _ptr]
lib.query_bvh_batch.restype = _int


def _host_offsets(seg):
    seg = [int(v) for v in seg]
    return seg, (ctypes.c_int * len(seg))(*seg)


class Forest:
    def __init__(self, x, seg, prefix=True, leaf=16):
        seg, self._seg_c = _host_offsets(seg)
        if not (
            er._is_points(x)
            and x.device.index == torch.cuda.current_device()
            and len(seg) >= 2
            and seg[0] == 0
            and seg[-1] == len(x)
            and all(b > a for a, b in zip(seg, seg[1:]))
            and isinstance(leaf, int)
            and leaf >= 1
        ):
            raise ValueError("Forest requires contiguous CUDA FP32 (N,3) points and ascending non-empty scene offsets")
        self.x = x
        self.seg = seg
        self.prefix = prefix
        self.stream = er._stream()
        self.sizes = [b - a for a, b in zip(seg, seg[1:])]
        self.ptr = _ptr()
        self.fallback = torch.zeros(1, device=x.device, dtype=torch.int32)
        self._qseg = {}
        er.check(
            lib.build_bvh_batch(
                x.data_ptr(), self._seg_c, len(self.sizes), int(prefix), leaf,
                ctypes.byref(self.ptr), self.stream,
            )
        )

    def __len__(self):
        return len(self.sizes)

    def level_sizes(self, level):
        return [n if level < 0 else n >> (2 * level) for n in self.sizes]

    def _offsets(self, qseg, device):
        key = tuple(int(v) for v in qseg)
        hit = self._qseg.get(key)
        if hit is None:
            host = (ctypes.c_int * len(key))(*key)
            dev = torch.tensor(key, dtype=torch.int32).to(device, non_blocking=False)
            hit = self._qseg[key] = (host, dev)
        return key, hit

    def _check(self, q, qseg, level):
        key, (host, dev) = self._offsets(qseg, q.device)
        if not (
            self.ptr
            and er._stream() == self.stream
            and er._is_points(q)
            and q.device == self.x.device
            and len(key) == len(self.sizes) + 1
            and key[0] == 0
            and key[-1] == len(q)
            and -1 <= level < (4 if self.prefix else 1)
        ):
            raise ValueError("Invalid forest query: points, offsets, level, or stream")
        return host, dev

    def ball(self, q, qseg, level, r, ns, out):
        """Ordered radius query of every scene; ``out`` int32 (Q_total, ns)."""
        host, dev = self._check(q, qseg, level)
        if not (er._is_rows(out, q, len(q), ns, torch.int32) and 1 <= ns <= 32 and r >= 0):
            raise ValueError("Invalid radius query output, K or radius")
        if len(q):
            er.check(
                lib.query_ball_bvh_batch(
                    self.ptr, q.data_ptr(), dev.data_ptr(), host, level, r, ns,
                    out.data_ptr(), self.fallback.data_ptr(), er._stream(),
                )
            )
        return out

    def query(self, q, qseg, level, d, idx):
        """Exact 3NN of every scene; ``d`` float32 / ``idx`` int32 (Q_total, 3)."""
        host, dev = self._check(q, qseg, level)
        if not (er._is_rows(d, q, len(q), 3, torch.float32) and er._is_rows(idx, q, len(q), 3, torch.int32)):
            raise ValueError("Invalid 3NN outputs")
        if len(q):
            er.check(
                lib.query_bvh_batch(
                    self.ptr, q.data_ptr(), dev.data_ptr(), host, level, d.data_ptr(),
                    idx.data_ptr(), self.fallback.data_ptr(), er._stream(),
                )
            )
        return d, idx

    def close(self):
        if self.ptr:
            er.check(lib.free_bvh(self.ptr, 1, er._stream()))
            self.ptr = _ptr()
