# SPDX-License-Identifier: Apache-2.0
"""Seeded synthetic scenes standing in for the reference's S3DIS/ScanNet data.

The reference measured on real scans that are not available here; these
generators produce point clouds with the same sizes, hierarchy shapes and
value distributions as its workloads:

* ``unit_case``      4096 N(0,1) points (torch seed 0), queries = first 128.
* ``room``           a room of uniform floor/ceiling/wall points with N(0, 1 cm)
                     normal jitter (70 % of points, area-weighted over the six
                     planes) plus 30 Gaussian object clusters (sigma 0.15 m,
                     30 %); 24,000 points in 3x3x3 m, or 1,000,000 points in a
                     20x20x3 m box.
* ``clustered``      50 Gaussian clusters of sigma 1e-3 in [0,3]^3 with 20 %
                     exact duplicate coordinates and 5 % points at FP32 squared
                     distance exactly f32(r)^2 from a query point.

Supports of the hierarchical workloads are farthest-point ordered
(``fps_order``, exact and deterministic, lowest index on ties), so the
prefixes n, n/4, n/16, ... are the sampled levels.
"""

import ctypes

import numpy as np
import torch

PLANE_FRACTION = 0.7
ROOM_CLUSTERS = 30
ROOM_SIGMA = 0.15
ROOM_JITTER = 0.01


def unit_case():
    """Support ``torch.randn(4096, 3)`` from seed 0 (CPU generator)."""
    g = torch.Generator().manual_seed(0)
    return torch.randn(4096, 3, generator=g).numpy()


def room(seed, n=24000, box=(3.0, 3.0, 3.0)):
    """Unordered room scene (float32 ``(n, 3)``) and a seeded FPS start index."""
    rng = np.random.default_rng(seed)
    w, d, h = box
    n_plane = int(round(PLANE_FRACTION * n))
    n_clu = n - n_plane
    areas = np.array([w * d, w * d, d * h, d * h, w * h, w * h])
    plane = rng.choice(6, size=n_plane, p=areas / areas.sum())
    u, v = rng.random(n_plane), rng.random(n_plane)
    jit = rng.normal(0.0, ROOM_JITTER, n_plane)
    p = np.empty((n_plane, 3))
    # floor z=0, ceiling z=h, walls x=0, x=w, y=0, y=d; jitter along the normal
    table = [
        (u * w, v * d, 0.0 + jit),
        (u * w, v * d, h + jit),
        (0.0 + jit, u * d, v * h),
        (w + jit, u * d, v * h),
        (u * w, 0.0 + jit, v * h),
        (u * w, d + jit, v * h),
    ]
    for k, (a, b, c) in enumerate(table):
        sel = plane == k
        p[sel, 0] = a[sel] if np.ndim(a) else a
        p[sel, 1] = b[sel] if np.ndim(b) else b
        p[sel, 2] = c[sel] if np.ndim(c) else c
    centres = rng.random((ROOM_CLUSTERS, 3)) * np.array(box)
    which = rng.integers(ROOM_CLUSTERS, size=n_clu)
    c = centres[which] + rng.normal(0.0, ROOM_SIGMA, (n_clu, 3))
    pts = np.concatenate([p, c]).astype(np.float32)
    pts = pts[rng.permutation(n)]
    start = int(rng.integers(n))
    return np.ascontiguousarray(pts), start


def clustered(seed=0, n=200_000, clusters=50, sigma=1e-3, dup=0.2, exact=0.05,
              r=0.25, n_queries=50_000):
    """Exactness-stress scene; returns (points float32 (n,3), info dict)."""
    rng = np.random.default_rng(seed)
    centres = rng.random((clusters, 3)) * 3.0
    pts = (centres[rng.integers(clusters, size=n)] + rng.normal(0.0, sigma, (n, 3))).astype(np.float32)
    ids = rng.permutation(n)
    n_dup, n_exact = int(dup * n), int(exact * n)
    dup_ids = ids[:n_dup]
    exact_ids = ids[n_dup:n_dup + n_exact]
    rest = ids[n_dup + n_exact:]
    pts[dup_ids] = pts[rng.choice(rest, size=n_dup)]
    r2 = np.float32(r) * np.float32(r)
    qsel = rest[rest < n_queries]
    placed = 0
    anchors = []
    for pid in exact_ids:
        for _ in range(16):
            qi = int(rng.choice(qsel))
            axis = int(rng.integers(3))
            sign = 1.0 if rng.random() < 0.5 else -1.0
            cand = pts[qi].copy()
            cand[axis] = np.float32(cand[axis] + np.float32(sign * r))
            delta = pts[qi] - cand
            sq = delta * delta
            if (sq[0] + sq[1]) + sq[2] == r2:
                pts[pid] = cand
                anchors.append((int(pid), qi))
                placed += 1
                break
    return np.ascontiguousarray(pts), {
        "exact_points": placed,
        "anchors": anchors,
        "duplicates": n_dup,
        "queries": n_queries,
        "r": r,
    }


def _fps_lib():
    from ._library import load

    lib = load("gsa_bvh")
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.fps_order.argtypes = [I, I, P, P, P, P]
    lib.fps_order.restype = I
    lib.fps_order_large.argtypes = [I, P, I, P, P, P, P]
    lib.fps_order_large.restype = I
    return lib


SMALL_FPS_MAX = 51200


def fps_order(points, starts, large=None):
    """Farthest-point order of ``b`` scenes of equal size on the GPU.

    points: CUDA float32 (b, n, 3) or (n, 3); starts: ints.  Returns an int64
    CPU tensor (b, n) (or (n,)) of point indices.  Scenes of more than
    51,200 points (or ``large=True``) use the cooperative-grid kernel, one
    scene at a time.
    """
    squeeze = points.ndim == 2
    x = points[None] if squeeze else points
    x = x.contiguous()
    b, n = x.shape[0], x.shape[1]
    starts = list(starts) if not np.isscalar(starts) else [starts]
    order = torch.empty((b, n), dtype=torch.int32, device=x.device)
    lib = _fps_lib()
    stream = torch.cuda.current_stream().cuda_stream
    if large or (large is None and n > SMALL_FPS_MAX):
        scratch = torch.empty(8, dtype=torch.int64, device=x.device)
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        for i in range(b):
            code = lib.fps_order_large(
                n, x[i].data_ptr(), int(starts[i]), order[i].data_ptr(), scratch.data_ptr(), err.data_ptr(), stream
            )
            if code or err.item():
                raise RuntimeError(f"fps_order_large error {code} / barrier {err.item()}")
    else:
        st = torch.as_tensor(starts, dtype=torch.int32).to(x.device)
        code = lib.fps_order(b, n, x.data_ptr(), st.data_ptr(), order.data_ptr(), stream)
        if code:
            raise RuntimeError(f"fps_order error {code}")
    order = order.long().cpu()
    return order[0] if squeeze else order


def room_batch(seeds, n=24000, box=(3.0, 3.0, 3.0), device="cuda"):
    """FPS-ordered room scenes, float32 CUDA tensor (len(seeds), n, 3)."""
    raw, starts = [], []
    for s in seeds:
        p, st = room(s, n, box)
        raw.append(p)
        starts.append(st)
    x = torch.from_numpy(np.stack(raw)).to(device)
    order = fps_order(x, starts).to(device)
    return torch.gather(x, 1, order[:, :, None].expand(-1, -1, 3)).contiguous()


def hierarchy(n, levels=5):
    """Support sizes of a ratio-4 hierarchy: n, n/4, n/16, ..."""
    return [n >> (2 * i) for i in range(levels)]
