# SPDX-License-Identifier: Apache-2.0
"""Sequential farthest-point order on the CPU (test infrastructure).

Rule shared with the GPU generator ``fps_order`` of ``include/gsa_bvh.h``:
running minimum of the exact float32 squared distance
``((dx*dx + dy*dy) + dz*dz)`` to the chosen points, chosen points marked -1,
next point = first index of the maximum.  Used to check the GPU generator
and the ``furthest_point_sample`` op (their first m entries) and to build
the CPU baseline's scenes without the GPU.
"""

import numpy as np


def fps_order(p, start, m=None):
    """The first ``m`` (default all) indices of the order from ``start``."""
    p = np.asarray(p, np.float32)
    n = len(p)
    m = n if m is None else m
    mind = np.full(n, np.inf, np.float32)
    order = np.empty(m, np.int64)
    cur = int(start)
    with np.errstate(over="ignore", invalid="ignore"):
        for it in range(m):
            order[it] = cur
            d = p[:, 0] - p[cur, 0]
            acc = d * d
            d = p[:, 1] - p[cur, 1]
            acc += d * d
            d = p[:, 2] - p[cur, 2]
            acc += d * d
            # fmin: a NaN distance never lowers a running minimum
            np.fmin(mind, acc, out=mind, where=mind >= 0)
            mind[cur] = -1.0
            cur = int(np.argmax(mind))
    return order
