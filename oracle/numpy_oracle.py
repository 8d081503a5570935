# SPDX-License-Identifier: Apache-2.0
"""CPU oracle for GSA's exact radius and three-nearest-neighbour queries.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or as the timed CPU baseline.  The product
(``gsa_b200``) never imports it and has no CPU fallback.

It restates, in NumPy, the independent FP32 oracle of the reference test
``tests/check_queries.py`` (GSA, qmkkk/GSA):

* ``distance``      follows ``tests/check_queries.py:23-27``
* ``ball_oracle``   follows ``tests/check_queries.py:30-40``
* ``nn_oracle``     follows ``tests/check_queries.py:64-78``

Arithmetic contract (``docs/api.md`` "Coordinate and execution contract"):
squared distance is ``((dx*dx + dy*dy) + dz*dz)`` in float32 with
round-to-nearest and no fused multiply-add; radius qualification is strict,
``d2 < f32(r) * f32(r)``; 3NN keeps the three smallest finite squared
distances in ``(d2, id)`` order and fills missing entries with ``(inf, 0)``.

Pinning: ``tests/test_oracle_golden.py`` reproduces every one of the 69
``ids_sha256`` values the reference committed in
``data/query_session/correctness.json`` from this module (fixture
``tests/golden/query_session_correctness.json``).

The ``*_fast`` variants compute the same results in O(N) memory per query
chunk (no per-row sort) so that the oracle finishes at the larger synthetic
workloads; ``tests/test_oracle_golden.py`` checks them against the literal
restatements.
"""

import numpy as np

__all__ = [
    "distance",
    "radius_squared",
    "ball_oracle",
    "ball_oracle_fast",
    "nn_oracle",
    "nn_oracle_fast",
    "ball_scan_untouched",
]


def distance(q, x):
    """Squared distances ``(len(q), len(x))`` in float32, reference order of
    operations ``(sq0 + sq1) + sq2`` (``tests/check_queries.py:23-27``)."""
    q = np.asarray(q, np.float32)
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        delta = q[:, None, :] - x[None, :, :]
        sq = delta * delta
        return (sq[:, :, 0] + sq[:, :, 1]) + sq[:, :, 2]


def radius_squared(r):
    """``f32(r) * f32(r)`` with overflow to +inf allowed
    (``tests/check_queries.py:33-34``)."""
    with np.errstate(over="ignore", under="ignore"):
        return np.float32(r) * np.float32(r)


def ball_oracle(q, x, r, k):
    """Literal restatement of ``tests/check_queries.py:30-40``.

    First ``k`` qualifying support IDs in ascending ID order, padded with the
    first qualifying ID; an all-zero row when nothing qualifies.
    """
    q = np.asarray(q, np.float32)
    x = np.asarray(x, np.float32)
    result = np.zeros((len(q), k), np.int32)
    if len(q) == 0:
        return result
    d = distance(q, x)
    r2 = radius_squared(r)
    for i, mask in enumerate(d < r2):
        ids = np.flatnonzero(mask)[:k]
        if len(ids):
            result[i, :] = ids[0]
            result[i, : len(ids)] = ids
    return result


def _chunks(nq, nx, budget=1 << 23):
    step = max(1, budget // max(1, nx))
    for s in range(0, nq, step):
        yield s, min(nq, s + step)


def _distance_lean(q, x):
    """Same values as :func:`distance` (same float32 operations in the same
    order) without the (Q, N, 3) temporary."""
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        d = q[:, None, 0] - x[None, :, 0]
        acc = d * d
        d = q[:, None, 1] - x[None, :, 1]
        acc += d * d
        d = q[:, None, 2] - x[None, :, 2]
        acc += d * d
        return acc


def ball_oracle_fast(q, x, r, k):
    """Same result as :func:`ball_oracle`, vectorised over query chunks.

    Uses a running count of qualifying points per row instead of
    ``flatnonzero`` per row; no sorting, so it is O(len(x)) per query.
    """
    q = np.asarray(q, np.float32)
    x = np.asarray(x, np.float32)
    result = np.zeros((len(q), k), np.int32)
    r2 = radius_squared(r)
    for s, e in _chunks(len(q), len(x)):
        mask = _distance_lean(q[s:e], x) < r2
        rank = np.cumsum(mask, axis=1, dtype=np.int32)
        keep = mask & (rank <= k)
        rows, cols = np.nonzero(keep)
        block = np.zeros((e - s, k), np.int32)
        block[rows, rank[rows, cols] - 1] = cols
        count = np.minimum(rank[:, -1] if len(x) else np.zeros(e - s, np.int32), k)
        # pad with the first qualifying ID (column 0 of the block)
        pad = np.arange(k)[None, :] >= count[:, None]
        block = np.where(pad, block[:, :1], block)
        block[count == 0] = 0
        result[s:e] = block
    return result


def ball_scan_untouched(q, x, r, k, initial):
    """The original-order scan kernel's contract
    (``csrc/reference_queries.cu:6-48``): like :func:`ball_oracle` except that
    a row with no qualifying point is left as it was in ``initial``."""
    out = np.array(initial, np.int32, copy=True)
    res = ball_oracle_fast(q, x, r, k)
    hit = (distance(q, x) < radius_squared(r)).any(axis=1) if len(x) else np.zeros(len(q), bool)
    out[hit] = res[hit]
    return out


def nn_oracle(q, x):
    """Literal restatement of ``tests/check_queries.py:64-78``.

    Finite distances only, stable argsort, first three; missing entries are
    ``inf`` with ID ``0``.
    """
    q = np.asarray(q, np.float32)
    x = np.asarray(x, np.float32)
    ed = np.full((len(q), 3), np.inf, np.float32)
    ei = np.zeros((len(q), 3), np.int32)
    if len(q) == 0:
        return ed, ei
    distances = distance(q, x)
    for i, row in enumerate(distances):
        valid = np.flatnonzero(np.isfinite(row))
        order = valid[np.argsort(row[valid], kind="stable")[:3]]
        ed[i, : len(order)] = row[order]
        ei[i, : len(order)] = order
    return ed, ei


def nn_oracle_fast(q, x):
    """Same result as :func:`nn_oracle` by three rounds of (min, first
    arg-min) per query chunk, i.e. lexicographic ``(d2, id)`` selection."""
    q = np.asarray(q, np.float32)
    x = np.asarray(x, np.float32)
    ed = np.full((len(q), 3), np.inf, np.float32)
    ei = np.zeros((len(q), 3), np.int32)
    if len(q) == 0 or len(x) == 0:
        return ed, ei
    for s, e in _chunks(len(q), len(x)):
        d = _distance_lean(q[s:e], x)
        d[~np.isfinite(d)] = np.inf
        rows = np.arange(e - s)
        for j in range(min(3, len(x))):
            col = np.argmin(d, axis=1)  # first occurrence = lowest ID on ties
            val = d[rows, col]
            ok = np.isfinite(val)
            ed[s:e, j] = np.where(ok, val, np.inf)
            ei[s:e, j] = np.where(ok, col, 0)
            d[rows, col] = np.inf
    return ed, ei


def hierarchy_oracle(P, sizes, radii, k=32, fraction=1.0):
    """Oracle outputs of the PointNeXt-shaped query hierarchy on one scene:
    per stage s the self rows ``ball(P_s -> P_s, r_s)``, the down-sampling
    rows (the first ``sizes[s+1]`` self rows, which the reuse cache serves)
    and ``nn(P_s -> P_{s+1})``.  With ``fraction < 1`` only the first
    ``ceil(fraction * len)`` queries of each call are answered (a bounded
    sample for timing).  Returns (outputs dict, rows answered)."""
    P = np.asarray(P, np.float32)
    out, rows = {}, 0
    for s in range(4):
        ps = P[: sizes[s]]
        nq = int(np.ceil(fraction * sizes[s]))
        res = ball_oracle_fast(ps[:nq], ps, radii[s], k)
        out[f"ball{s}"] = res
        nh = int(np.ceil(fraction * sizes[s + 1]))
        out[f"hit{s}"] = res[:nh].copy()
        d, i = nn_oracle_fast(ps[:nq], P[: sizes[s + 1]])
        out[f"nnd{s}"], out[f"nni{s}"] = d, i
        rows += 2 * nq + nh
    return out, rows
