# SPDX-License-Identifier: Apache-2.0
"""Original-order brute-force query ops (mirror of GSA ``gsa/reference.py``).

``ball_query_wrapper`` and ``three_nn_wrapper`` keep the PointNet++ operator
signatures that the fixed-graph adapter patches
(``docs/integration.md``):

    ball_query_wrapper(B, N, Q, radius, K, queries, support, output_ids)
    three_nn_wrapper(B, Q, N, queries, support, squared_distances, output_ids)
"""

import ctypes

import torch

from ._library import load, stream

lib = load("reference_queries")
P = ctypes.c_void_p
I = ctypes.c_int
lib.ball.argtypes = [I, I, I, ctypes.c_float, I, P, P, P, P]
lib.ball.restype = I
lib.nn3.argtypes = [I, I, I, P, P, P, P, P]
lib.nn3.restype = I


def call(name, *args):
    values = [a.data_ptr() if isinstance(a, torch.Tensor) else a for a in args]
    error = getattr(lib, name)(*values, stream())
    if error:
        raise RuntimeError(f"{name}: CUDA error {error}")


def ball_query_wrapper(b, n, m, radius, k, q, x, out):
    """Ordered first-K radius scan; rows without a hit are left untouched."""
    call("ball", b, n, m, radius, k, q, x, out)


def three_nn_wrapper(b, n, m, q, x, distance, ids):
    """Exact 3NN scan of ``n`` queries against ``m`` support points."""
    call("nn3", b, n, m, q, x, distance, ids)
