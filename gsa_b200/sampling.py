# SPDX-License-Identifier: Apache-2.0
"""Furthest point sampling, the op that produces the query levels.

GSA's networks search FPS-ordered prefixes: the sampled level of a stage is
the first m points of a farthest-point order of the level above (the
reference takes it from FlashFPS upstream and ships no FPS of its own).
``furthest_point_sampling_wrapper`` has the PointNet++ operator's arguments,
so a network's ``ops`` module can route its FPS calls here next to
``ball_query_wrapper`` / ``three_nn_wrapper``; ``furthest_point_sample`` is
the tensor form.  Rule (``include/gsa_bvh.h`` ``furthest_point_sample``):
start at index 0, next = largest running minimum of the exact FP32 squared
distance to the chosen points, ties to the lowest index.
"""

import ctypes

import torch

from . import runtime as er

_P, _I = ctypes.c_void_p, ctypes.c_int
er.lib.furthest_point_sample.argtypes = [_I, _I, _I, _P, _P, _P, _P]
er.lib.furthest_point_sample.restype = _I

SMALL_MAX = 51200  # points per scene whose running minima fit in shared memory


def furthest_point_sampling_wrapper(b, n, m, points, temp, idx):
    """PointNet++ signature: points (b, n, 3) float32, temp (b, n) float32
    scratch (used for scenes of more than 51,200 points), idx (b, m) int32
    output; all contiguous CUDA tensors."""
    ok = (
        all(isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous() for t in (points, idx))
        and points.dtype == torch.float32 and points.numel() == b * n * 3
        and idx.dtype == torch.int32 and idx.numel() == b * m
        and (temp is None or (temp.is_cuda and temp.dtype == torch.float32 and temp.numel() >= b * n))
    )
    if not ok:
        raise ValueError("furthest_point_sampling_wrapper needs contiguous CUDA float32 points (b,n,3), "
                         "int32 idx (b,m) and float32 temp (b,n)")
    code = er.lib.furthest_point_sample(
        b, n, m, points.data_ptr(), None if temp is None else temp.data_ptr(), idx.data_ptr(), er._stream()
    )
    if code:
        raise RuntimeError(f"furthest_point_sample error {code}")


def furthest_point_sample(xyz, npoint):
    """First ``npoint`` indices of the farthest-point order of each scene of
    ``xyz`` (CUDA float32 (B, N, 3)); returns int32 (B, npoint)."""
    if not (xyz.is_cuda and xyz.dtype == torch.float32 and xyz.ndim == 3 and xyz.shape[2] == 3):
        raise ValueError("xyz must be CUDA float32 (B, N, 3)")
    xyz = xyz.contiguous()
    b, n = xyz.shape[0], xyz.shape[1]
    if not 0 <= npoint <= n:
        raise ValueError("npoint must be in [0, N]")
    idx = torch.empty((b, npoint), dtype=torch.int32, device=xyz.device)
    temp = torch.empty((b, n), dtype=torch.float32, device=xyz.device) if n > SMALL_MAX else None
    furthest_point_sampling_wrapper(b, n, npoint, xyz, temp, idx)
    if temp is not None:
        err = temp.view(torch.int32)[:, 16]
        if bool((err != 0).any()):
            raise RuntimeError("furthest_point_sample: a grid barrier wait ran out; the order is incomplete")
    return idx
