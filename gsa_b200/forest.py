# SPDX-License-Identifier: Apache-2.0
"""Batched multi-scene index: B independent prefix trees in one object.

The reference API serves one scene per call.  Batched inference over many
small scenes (e.g. 64 room scenes of 24,000 points) would leave most of a
B200's 148 SMs idle per call; ``Forest`` builds all trees with one launch per
build step and answers a query stage of every scene with one launch.
Results per scene are identical to ``Tree`` on that scene.

Layout: the supports of all scenes are concatenated into one contiguous
``(N_total, 3)`` float32 CUDA tensor with host offsets ``seg`` (B+1 values).
A query stage passes per-scene query counts; queries are either a separate
concatenated tensor or, with ``ball_prefix``/``query_prefix``, each scene's
own first points (no copy).  Scene ``i`` searches its support prefix of
``m`` points, by default its level size ``n_i >> (2 * level)``.
"""

import ctypes
import itertools

import torch

from . import runtime as er

lib = er.lib
_ptr, _int = ctypes.c_void_p, ctypes.c_int
lib.build_bvh_batch.argtypes = [_ptr, _ptr, _int, _int, _int, ctypes.POINTER(_ptr), _ptr]
lib.build_bvh_batch.restype = _int
lib.query_ball_bvh_batch.argtypes = [_ptr, _ptr, _ptr, _ptr, _ptr, _int, _int, ctypes.c_float, _int, _ptr, _ptr, _ptr]
lib.query_ball_bvh_batch.restype = _int
lib.query_bvh_batch.argtypes = [_ptr, _ptr, _ptr, _ptr, _ptr, _int, _int, _ptr, _ptr, _ptr, _ptr]
lib.query_bvh_batch.restype = _int
lib.rebuild_bvh_batch.argtypes = [_ptr, _ptr, _ptr]
lib.rebuild_bvh_batch.restype = _int

_INT_CACHE = {}


def _device_ints(values, device):
    """Cached device copy of a small int32 offset list (one upload per
    distinct list, so repeated batches issue no host-to-device copies)."""
    key = (tuple(values), str(device))
    t = _INT_CACHE.get(key)
    if t is None:
        if len(_INT_CACHE) > 256:
            _INT_CACHE.clear()
        t = _INT_CACHE[key] = torch.tensor(key[0], dtype=torch.int32).to(device)
    return t


class Forest:
    def __init__(self, x, seg, prefix=True, leaf=16):
        seg = [int(v) for v in seg]
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
        self._dev = {}
        self._starts = _device_ints(seg[:-1], x.device)
        seg_c = (ctypes.c_int * len(seg))(*seg)
        er.check(lib.build_bvh_batch(x.data_ptr(), seg_c, len(self.sizes), int(prefix), leaf, ctypes.byref(self.ptr), self.stream))

    def __len__(self):
        return len(self.sizes)

    def level_sizes(self, level):
        return [n if level < 0 else n >> (2 * level) for n in self.sizes]

    def _offsets(self, counts, device):
        key = tuple(int(c) for c in counts)
        hit = self._dev.get(key)
        if hit is None:
            qseg = [0] + list(itertools.accumulate(key))
            host = (ctypes.c_int * len(qseg))(*qseg)
            dev = _device_ints(qseg, device)
            hit = self._dev[key] = (qseg, host, dev)
        return hit

    def _prepare(self, q, counts, level, m, min_m):
        if isinstance(counts, int):
            counts = [counts] * len(self.sizes)
        qseg, host, dev = self._offsets(counts, q.device)
        # queries may run on any stream ordered after the build (several
        # stages can run concurrently); close() must be ordered after them
        if not (
            self.ptr
            and er._is_points(q)
            and q.device == self.x.device
            and len(qseg) == len(self.sizes) + 1
            and -1 <= level < (4 if self.prefix else 1)
            and m >= 0
        ):
            raise ValueError("Invalid forest query: points, counts, level, or stream")
        for c, size in zip(counts, self.level_sizes(level)):
            if c and not (min_m <= (m or size) <= size):
                raise ValueError("Support prefix outside the level's bounds")
        return qseg, host, dev

    def _ball(self, q, qstart, counts, level, r, ns, out, m):
        qseg, host, dev = self._prepare(q, counts, level, m, 1)
        if not (er._is_rows(out, q, qseg[-1], ns, torch.int32) and 1 <= ns <= 32 and r >= 0):
            raise ValueError("Invalid radius query output, K or radius")
        if qseg[-1]:
            er.check(
                lib.query_ball_bvh_batch(
                    self.ptr, q.data_ptr(), qstart, dev.data_ptr(), host, m, level, r, ns,
                    out.data_ptr(), self.fallback.data_ptr(), er._stream(),
                )
            )
        return out

    def _query(self, q, qstart, counts, level, d, idx, m):
        qseg, host, dev = self._prepare(q, counts, level, m, 3)
        rows = qseg[-1]
        if not (er._is_rows(d, q, rows, 3, torch.float32) and er._is_rows(idx, q, rows, 3, torch.int32)):
            raise ValueError("Invalid 3NN outputs")
        if rows:
            er.check(
                lib.query_bvh_batch(
                    self.ptr, q.data_ptr(), qstart, dev.data_ptr(), host, m, level,
                    d.data_ptr(), idx.data_ptr(), self.fallback.data_ptr(), er._stream(),
                )
            )
        return d, idx

    def ball(self, q, counts, level, r, ns, out, m=0):
        """Radius query; scene i's queries are the next counts[i] rows of q."""
        if len(q) != sum(counts):
            raise ValueError("query rows must equal the sum of counts")
        return self._ball(q, None, counts, level, r, ns, out, m)

    def query(self, q, counts, level, d, idx, m=0):
        """3NN; scene i's queries are the next counts[i] rows of q."""
        if len(q) != sum(counts):
            raise ValueError("query rows must equal the sum of counts")
        return self._query(q, None, counts, level, d, idx, m)

    def ball_prefix(self, count, level, r, ns, out, m=0):
        """Radius query of each scene's own first ``count`` support points."""
        if any(count > n for n in self.sizes):
            raise ValueError("prefix longer than a scene")
        return self._ball(self.x, self._starts.data_ptr(), count, level, r, ns, out, m)

    def query_prefix(self, count, level, d, idx, m=0):
        """3NN of each scene's own first ``count`` support points."""
        if any(count > n for n in self.sizes):
            raise ValueError("prefix longer than a scene")
        return self._query(self.x, self._starts.data_ptr(), count, level, d, idx, m)

    def rebuild(self, x):
        """Rebuild every tree in place from ``x``, new coordinates with the
        shape the forest was created with (``x`` is borrowed from then on).
        The first call keeps the build temporaries with the forest; later
        calls allocate nothing, so a rebuild and the queries after it can be
        captured in a CUDA graph."""
        if not (
            self.ptr
            and er._is_points(x)
            and len(x) == len(self.x)
            and x.device == self.x.device
        ):
            raise ValueError("rebuild requires contiguous CUDA FP32 points shaped like the forest's")
        self.x = x
        er.check(lib.rebuild_bvh_batch(self.ptr, x.data_ptr(), er._stream()))

    def close(self):
        if self.ptr:
            er.check(lib.free_bvh(self.ptr, 1, er._stream()))
            self.ptr = _ptr()
