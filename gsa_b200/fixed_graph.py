# SPDX-License-Identifier: Apache-2.0
"""Fixed hierarchical graph adapter (drop-in for GSA ``gsa/fixed_graph.py``).

``forward(model, data, ops=..., policy=...)`` swaps the two PointNet++
operator wrappers of ``ops`` (``ball_query_wrapper``, ``three_nn_wrapper``)
for the duration of one model forward and restores them, freeing every
index, when the forward returns or raises.

Admission is structural (``docs/integration.md``): the first radius call
fixes the ordered first sampled level; every later support shorter than the
root is an ordered prefix of it.  ``policy="prefix"`` serves all such
supports from one shared prefix index, ``"scale"`` builds one index per
support size, ``"flash"`` leaves the wrappers alone.  A self-query radius
call on a non-root support stores 32 IDs per row; a later call with the same
support length and radius slices those rows.  ``verify=True`` asserts the
coordinate conditions (here with one device comparison launch per check)
and collects traversal fallbacks.  Counters match ``gsa/fixed_graph.py``.
"""

import torch

from . import runtime as er
from .session import _CudaOps


class _Adapter:
    def __init__(self, ops, policy, cache, threshold, leaf, verify, n_root):
        self.ops = ops
        self.shared_prefix = policy == "prefix"
        self.cache = cache
        self.threshold = threshold
        self.leaf = leaf
        self.verify = verify
        self.n_root = n_root
        self.level0 = None  # queries of the first radius call, (1, S, 3)
        self.indices = {}  # "prefix" or support length -> Tree
        self.rows = {}  # (support length, radius) -> (rows, queries, support)
        self.dev = _CudaOps()
        self.counters = {
            "builds": 0,
            "ball_calls": 0,
            "ball_hits": 0,
            "nn_calls": 0,
            "cache_bytes": 0,
            "fallbacks": 0,
        }
        self.saved = (ops.ball_query_wrapper, ops.three_nn_wrapper)

    def _all_equal(self, pairs):
        """torch.equal over every pair, evaluated in one device launch."""
        for a, b in pairs:
            if a.shape != b.shape or a.dtype != b.dtype or a.device != b.device:
                return False
            if not (a.is_contiguous() and b.is_contiguous()):
                return all(torch.equal(u, v) for u, v in pairs)
        flags = self.dev.fetch(self.dev.mismatch(pairs, pairs[0][0].device))
        return not any(flags)

    def _index_for(self, x):
        size = x.shape[1]
        nested = self.shared_prefix and size != self.n_root
        if nested and self.verify:
            assert self._all_equal([(x, self.level0[:, :size])])
        key = "prefix" if nested else size
        tree = self.indices.get(key)
        if tree is None:
            tree = er.Tree(self.level0[0] if nested else x[0], nested, self.leaf)
            self.indices[key] = tree
            self.counters["builds"] += 1
        return tree

    def _release(self, key):
        tree = self.indices.pop(key)
        if self.verify:
            self.counters["fallbacks"] += int(tree.fallback.item())
        tree.close()

    def ball(self, b, n, m, r, ns, q, x, idx):
        assert b == 1 and ns <= 32
        self.counters["ball_calls"] += 1
        if self.level0 is None:
            assert n == self.n_root
            self.level0 = q
        key = (n, r)
        keep = self.cache and n != self.n_root
        hit = self.rows.get(key) if keep else None
        if hit is not None:
            rows, queries, support = hit
            if self.verify:
                assert self._all_equal([(q, queries[:, :m]), (x, support)])
            self.dev.copy_cols(idx[0], rows[0], ns)
            self.counters["ball_hits"] += 1
            return
        width = 32 if keep else ns
        result = torch.zeros((b, m, width), device=q.device, dtype=torch.int32)
        if n <= self.threshold:
            self.saved[0](b, n, m, r, width, q, x, result)
        else:
            self._index_for(x).ball(q[0], n, r, width, result[0])
        if width == ns:
            idx.copy_(result)
        else:
            self.dev.copy_cols(idx[0], result[0], ns)
        if keep and m == n:
            self.rows[key] = (result, q, x)
            self.counters["cache_bytes"] += result.numel() * result.element_size()
        if n == self.n_root and n in self.indices:
            self._release(n)  # the root-resolution index serves one call

    def nn(self, b, n, m, q, x, d, idx):
        assert b == 1
        self.counters["nn_calls"] += 1
        if m <= self.threshold:
            self.saved[1](b, n, m, q, x, d, idx)
        else:
            self._index_for(x).query(q[0], m, d[0], idx[0])

    def install(self):
        self.ops.ball_query_wrapper = self.ball
        self.ops.three_nn_wrapper = self.nn

    def restore(self, stats):
        self.ops.ball_query_wrapper, self.ops.three_nn_wrapper = self.saved
        for key in list(self.indices):
            self._release(key)
        if stats is not None:
            stats.update(self.counters)


def forward(
    model,
    data,
    *,
    ops,
    model_forward=None,
    policy="prefix",
    cache=True,
    threshold=1024,
    leaf=16,
    verify=True,
    stats=None
):
    """Run ``model_forward(model, data)`` (default ``model(data)``) with the
    query wrappers of ``ops`` routed through GSA indices and row reuse."""
    assert policy in ("flash", "prefix", "scale")
    run = model_forward if model_forward is not None else (lambda m, d: m(d))
    if policy == "flash":
        return run(model, data)
    adapter = _Adapter(ops, policy, cache, threshold, leaf, verify, data["pos"].shape[1])
    adapter.install()
    try:
        return run(model, data)
    finally:
        adapter.restore(stats)
