# SPDX-License-Identifier: Apache-2.0
"""The PointNeXt-shaped query hierarchy, per scene and for scene batches.

A scene's support ``P`` is farthest-point ordered; its sampled levels are the
prefixes ``P_s = P[:sizes[s]]`` (ratio 4).  Per encoder stage ``s`` the
hierarchy runs, with K = 32 (``data/summaries`` call structure of GSA):

* ``ball(P_s -> P_s, r_s)``      computed self-query rows;
* ``ball(P_{s+1} -> P_s, r_s)``  down-sampling rows, answered from the
  self-query rows after the support / query-prefix value checks (reuse hit);

and per decoder stage ``nn(P_s -> P_{s+1})`` for s = 3..0.

``run_session`` issues exactly these calls through the drop-in
``QuerySession``.  ``Batch`` runs the same hierarchy for B equally sized
scenes with one launch per build step / query stage (forest build, radius
and 3NN traversal of every scene, one launch per stage for the value checks
and the row gather); its outputs equal ``run_session``'s for every scene.
"""

import contextlib
import ctypes

import torch

from . import runtime as er
from .forest import Forest

ROOM_SIZES = (24000, 6000, 1500, 375, 94)
ROOM_RADII = (0.1, 0.2, 0.4, 0.8)
LARGE_SIZES = (1_000_000, 250_000, 62_500, 15_625, 3_906)
LARGE_RADII = (0.05, 0.1, 0.2, 0.4)
K = 32

_P, _I, _LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
er.lib.coords_mismatch_strided.argtypes = [_I, _P, _LL, _P, _LL, _LL, _P, _I, _P]
er.lib.coords_mismatch_strided.restype = _I
er.lib.reuse_rows_batch.argtypes = [_I, _P, _LL, _I, _P, _I, _I, _P, _LL, _P, _P]
er.lib.reuse_rows_batch.restype = _I
er.lib.reuse_prefix_batch.argtypes = [_I, _P, _LL, _P, _LL, _LL, _LL, _P, _LL, _I, _I, _I, _P, _LL, _P, _P, _P]
er.lib.reuse_prefix_batch.restype = _I
er.lib.reuse_prefix_stages.argtypes = [_I, _I, _P, _LL, _P, _LL, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P, _P, _P]
er.lib.reuse_prefix_stages.restype = _I


def unit_counts(sizes):
    """Rows answered per scene: (computed radius, reuse hits, 3NN)."""
    return sum(sizes[:4]), sum(sizes[1:5]), sum(sizes[:4])


def session_outputs(sizes=ROOM_SIZES, device="cuda", flat=None):
    """Output tensors of one ``run_session`` call as views of one flat int32
    buffer (distances viewed as FP32), so a scene's results leave the device
    in a single copy.  Returns ``(flat, outputs)``; pass ``flat`` to reuse a
    buffer of ``session_words(sizes)`` elements."""
    if flat is None:
        flat = torch.empty(session_words(sizes), dtype=torch.int32, device=device)
    out, at = {}, 0

    def take(key, rows, width, dtype):
        nonlocal at
        v = flat[at : at + rows * width].view(rows, width)
        out[key] = v if dtype == torch.int32 else v.view(dtype)
        at += rows * width

    for s in range(4):
        take(f"ball{s}", sizes[s], K, torch.int32)
        take(f"hit{s}", sizes[s + 1], K, torch.int32)
    for s in range(3, -1, -1):
        take(f"nnd{s}", sizes[s], 3, torch.float32)
        take(f"nni{s}", sizes[s], 3, torch.int32)
    return flat, out


def session_words(sizes=ROOM_SIZES):
    """32-bit words of one scene's outputs."""
    return sum(sizes[s] * K + sizes[s + 1] * K + 6 * sizes[s] for s in range(4))


def run_session(session, P, sizes=ROOM_SIZES, radii=ROOM_RADII, out=None):
    """Run the hierarchy on one scene through ``QuerySession``; returns the
    outputs as a dict of device tensors (``out``: preallocated tensors with
    the same keys, e.g. from ``session_outputs``)."""
    if out is None:
        out = {}
        for s in range(4):
            out[f"ball{s}"] = torch.empty((sizes[s], K), dtype=torch.int32, device=P.device)
            out[f"hit{s}"] = torch.empty((sizes[s + 1], K), dtype=torch.int32, device=P.device)
            out[f"nnd{s}"] = torch.empty((sizes[s], 3), device=P.device)
            out[f"nni{s}"] = torch.empty((sizes[s], 3), dtype=torch.int32, device=P.device)
    for s in range(4):
        ps, pn = P[: sizes[s]], P[: sizes[s + 1]]
        session.ball_into(ps, ps, radii[s], K, out[f"ball{s}"])
        session.ball_into(pn, ps, radii[s], K, out[f"hit{s}"])
    for s in range(3, -1, -1):
        session.nn_into(P[: sizes[s]], P[: sizes[s + 1]], out[f"nnd{s}"], out[f"nni{s}"])
    return out


def graph_model(ops, sizes=ROOM_SIZES, radii=ROOM_RADII, out=None):
    """The hierarchy as a fixed PointNet++-style network for
    ``fixed_graph_forward``: ``model(data)`` takes ``data["pos"]`` of shape
    (1, N, 3) and issues, through ``ops.ball_query_wrapper`` /
    ``ops.three_nn_wrapper`` (looked up at call time, so the adapter's
    patched wrappers run), the same calls in the same order as
    ``run_session``: per stage s the self query of P_s and the down-sampling
    query of P_{s+1} against P_s, then 3NN for s = 3..0.  Rows go to ``out``
    (tensors keyed and shaped like ``run_session``'s, e.g. the views of
    ``session_outputs``)."""

    def model(data):
        root = data["pos"]
        for s in range(4):
            ps, pn = root[:, : sizes[s]], root[:, : sizes[s + 1]]
            ops.ball_query_wrapper(1, sizes[s], sizes[s], radii[s], K, ps, ps, out[f"ball{s}"][None])
            ops.ball_query_wrapper(1, sizes[s], sizes[s + 1], radii[s], K, pn, ps, out[f"hit{s}"][None])
        for s in range(3, -1, -1):
            ops.three_nn_wrapper(1, sizes[s], sizes[s + 1], root[:, : sizes[s]], root[:, : sizes[s + 1]],
                                 out[f"nnd{s}"][None], out[f"nni{s}"][None])
        return out

    return model


# Batches from this many scenes take the four stages' reuse checks in one
# launch after the radius stages (64 rooms: 63 -> 41 us of reuse, step
# unchanged); smaller ones check each stage right after its radius stage,
# where the single launch would lengthen the step's tail (8 / 16 rooms:
# 0.414 -> 0.430 and 0.540 -> 0.575 ms per step with it).
FUSED_REUSE_MIN_SCENES = 48


class Batch:
    """Hierarchy over B scenes of N points each, all on the device."""

    def __init__(self, sizes=ROOM_SIZES, radii=ROOM_RADII, leaf=16):
        self.sizes = tuple(sizes)
        self.radii = tuple(radii)
        self.leaf = leaf
        self._streams = {}

    def _level(self, size, n):
        for level in range(4):
            if size <= n >> (2 * level):
                best = level
        return best

    def allocate(self, B, device):
        """Output buffers of one run (reusable across runs)."""
        z = {}
        for s in range(4):
            z[f"ball{s}"] = torch.empty((B * self.sizes[s], K), dtype=torch.int32, device=device)
            z[f"hit{s}"] = torch.empty((B * self.sizes[s + 1], K), dtype=torch.int32, device=device)
            z[f"nnd{s}"] = torch.empty((B * self.sizes[s], 3), device=device)
            z[f"nni{s}"] = torch.empty((B * self.sizes[s], 3), dtype=torch.int32, device=device)
        z["flags"] = torch.zeros((4, 2 * B), dtype=torch.int32, device=device)
        z["hits"] = torch.zeros((4, B), dtype=torch.int32, device=device)
        z["snapshot"] = torch.empty((B, self.sizes[0], 3), device=device)
        return z

    def _side_streams(self, device):
        streams = self._streams.get(device)
        if streams is None:
            streams = self._streams[device] = [torch.cuda.Stream(device) for _ in range(8)]
        return streams

    def _check_input(self, X):
        if not (X.is_cuda and X.is_contiguous() and X.dtype == torch.float32 and X.ndim == 3
                and X.shape[2] == 3 and X.shape[1] == self.sizes[0]):
            raise ValueError("Batch needs contiguous CUDA FP32 (B, sizes[0], 3)")

    def run(self, X, out=None, timer=None, concurrent=True):
        """X: CUDA float32 (B, N, 3), N == sizes[0], each scene FPS-ordered.

        After the forest build, the eight query stages (radius and 3NN for
        s = 0..3) depend only on the build, so with ``concurrent`` they run
        on eight streams and the small, latency-bound stages overlap the
        large ones; the four stages' reuse checks follow the radius stages
        (in one launch for large batches); the caller's stream waits for all
        of them.  ``timer.span(name)``, if given, brackets each stage on the
        stream it runs on (build, ball<s>, reuse or reuse<s>, nn<s>)."""
        self._check_input(X)
        B, N = X.shape[0], X.shape[1]
        out = out if out is not None else self.allocate(B, X.device)
        timer = timer or _NoTimer()
        with timer.span("build"):
            out["snapshot"].copy_(X)  # retained snapshot of every support, as the session keeps
            forest = Forest(X.view(-1, 3), [i * N for i in range(B + 1)], prefix=True, leaf=self.leaf)
        self._stages(X, out, forest, timer, concurrent)
        forest.close()
        return out

    def capture(self, X, out=None):
        """The whole step over fixed buffers ``X`` and ``out`` as one CUDA
        graph (``CapturedStep``): snapshot copy, in-place forest rebuild and
        all eight query stages on their streams.  Replaying it answers the
        hierarchy for whatever coordinates ``X`` holds at replay time, with
        one host call per step instead of ~40 library calls."""
        self._check_input(X)
        out = out if out is not None else self.allocate(X.shape[0], X.device)
        return CapturedStep(self, X, out)

    def _stages(self, X, out, forest, timer=None, concurrent=True):
        """Enqueue the eight query stages on ``forest`` (built over X) and
        the reuse checks of the four radius stages: for batches of at least
        FUSED_REUSE_MIN_SCENES scenes in one launch after them, else each
        right after its radius stage."""
        B, N = X.shape[0], X.shape[1]
        timer = timer or _NoTimer()
        main = torch.cuda.current_stream()
        snap = out["snapshot"]

        fused = B >= FUSED_REUSE_MIN_SCENES

        def radius_stage(s):
            n_s, n_q = self.sizes[s], self.sizes[s + 1]
            with timer.span(f"ball{s}"):
                forest.ball_prefix(n_s, s, self.radii[s], K, out[f"ball{s}"])
            if fused:
                return
            # this stage's reuse admission right after it: support P_s and
            # query prefix P_{s+1} equal the retained snapshot, then the
            # first n_q rows of each scene are copied (a cluster per scene)
            with timer.span(f"reuse{s}"):
                er.check(
                    er.lib.reuse_prefix_batch(
                        B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, n_s * 3, n_q * 3,
                        out[f"ball{s}"].data_ptr(), n_s * K, K, n_q, K, out[f"hit{s}"].data_ptr(),
                        n_q * K, out["flags"][s].data_ptr(), out["hits"][s].data_ptr(), er._stream(),
                    )
                )

        def reuse_stages():
            # reuse admission of every stage in one launch (a thread-block
            # cluster per stage and scene): support P_s and query prefix
            # P_{s+1} equal the retained snapshot, then the first n_{s+1}
            # rows of each scene's radius rows are copied
            st = range(4)
            ns = (ctypes.c_longlong * 4)(*[self.sizes[s] * 3 for s in st])
            nq = (ctypes.c_longlong * 4)(*[self.sizes[s + 1] * 3 for s in st])
            src = (ctypes.c_void_p * 4)(*[out[f"ball{s}"].data_ptr() for s in st])
            src_stride = (ctypes.c_longlong * 4)(*[self.sizes[s] * K for s in st])
            rows = (ctypes.c_int * 4)(*[self.sizes[s + 1] for s in st])
            dst = (ctypes.c_void_p * 4)(*[out[f"hit{s}"].data_ptr() for s in st])
            dst_stride = (ctypes.c_longlong * 4)(*[self.sizes[s + 1] * K for s in st])
            flags = (ctypes.c_void_p * 4)(*[out["flags"][s].data_ptr() for s in st])
            hits = (ctypes.c_void_p * 4)(*[out["hits"][s].data_ptr() for s in st])
            with timer.span("reuse"):
                er.check(
                    er.lib.reuse_prefix_stages(
                        4, B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, ns, nq, src,
                        src_stride, K, rows, K, dst, dst_stride, flags, hits, er._stream(),
                    )
                )

        def nn_stage(s):
            m = self.sizes[s + 1]
            level = self._level(m, N)
            with timer.span(f"nn{s}"):
                forest.query_prefix(self.sizes[s], level, out[f"nnd{s}"], out[f"nni{s}"], m=m if m != N >> (2 * level) else 0)

        stages = []
        for s in range(4):  # largest stages first, so small ones fill gaps
            stages += [lambda s=s: radius_stage(s), lambda s=s: nn_stage(s)]
        if concurrent:
            built = torch.cuda.Event()
            built.record(main)
            done = []
            streams = self._side_streams(X.device)
            for job, stream in zip(stages, streams):
                stream.wait_event(built)
                with torch.cuda.stream(stream):
                    job()
                    ev = torch.cuda.Event()
                    ev.record(stream)
                done.append(ev)
            if fused:
                # the reuse checks read the four radius stages' rows (jobs 0,
                # 2, 4, 6); they run on radius stage 0's stream, the longest
                for ev in done[2::2]:
                    streams[0].wait_event(ev)
                with torch.cuda.stream(streams[0]):
                    reuse_stages()
                    ev = torch.cuda.Event()
                    ev.record(streams[0])
                done[0] = ev
            for ev in done:
                main.wait_event(ev)
        else:
            for job in stages:
                job()
            if fused:
                reuse_stages()


class CapturedStep:
    """One hierarchy step over fixed input and output buffers, captured as a
    CUDA graph.

    The forest is created once and rebuilt in place inside the graph (its
    build temporaries stay allocated with it), so a replay allocates nothing
    and enqueues the snapshot copy, every build kernel, the eight query
    stages on their side streams and the reuse checks with one
    ``cudaGraphLaunch``.  ``launches`` is the number of library kernel
    launches one replay runs (counted while capturing).  Outputs equal
    ``Batch.run`` on the same coordinates."""

    def __init__(self, batch, X, out):
        from ._library import launch_counter

        B, N = X.shape[0], X.shape[1]
        self.X, self.out = X, out
        flat = X.view(-1, 3)
        self.forest = Forest(flat, [i * N for i in range(B + 1)], prefix=True, leaf=batch.leaf)
        # eager pass: keeps the build temporaries, fills the host-side caches
        out["snapshot"].copy_(X)
        self.forest.rebuild(flat)
        batch._stages(X, out, self.forest)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        before = launch_counter()
        with torch.cuda.graph(self.graph):
            out["snapshot"].copy_(X)
            self.forest.rebuild(flat)
            batch._stages(X, out, self.forest)
        self.launches = launch_counter() - before
        torch.cuda.synchronize()

    def replay(self):
        """Enqueue one step on the current stream; returns the outputs."""
        self.graph.replay()
        return self.out

    def close(self):
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None
            self.forest.close()


class _NoTimer:
    @contextlib.contextmanager
    def span(self, name):
        yield


class StageTimer:
    """CUDA events around each stage, recorded on the stream it runs on."""

    def __init__(self):
        self.records = []

    @contextlib.contextmanager
    def span(self, name):
        start = torch.cuda.Event(enable_timing=True)
        start.record()
        yield
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        self.records.append((name, start, end))

    def totals(self):
        """Milliseconds per stage name (call after synchronising)."""
        t = {}
        for name, start, end in self.records:
            t[name] = t.get(name, 0.0) + start.elapsed_time(end)
        return t
