# SPDX-License-Identifier: Apache-2.0
"""GPU: bit-exact agreement with the reference's own CUDA kernels.

``oracle/_ref`` holds GSA's ``csrc/gsa_bvh.cu`` (cuBQL build + prefix refit +
``radius_ordered``/``query3``) and ``csrc/reference_queries.cu``
(``ball``/``nn3``) compiled from source for sm_100a by ``oracle/Makefile``.
Both libraries export the same C ABI as ours, so the same calls run on both
and the outputs must be identical.  Skipped when the checker was not built.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from tests import abi

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def _lib(name):
    p = REF / (name + ".so")
    if not p.is_file():
        pytest.skip("reference checker not built (make -C oracle)")
    return ctypes.CDLL(str(p))


def _bind_bvh(lib):
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.build_bvh.argtypes = [P, I, I, I, ctypes.POINTER(P), P]
    lib.query_bvh.argtypes = [P, P, I, I, I, P, P, P, P]
    lib.query_ball_bvh.argtypes = [P, P, I, I, I, F, I, P, P, P]
    lib.free_bvh.argtypes = [P, I, P]
    return lib


def _room(seed, n):
    from gsa_b200 import scenes

    p, start = scenes.room(seed, n=n)
    x = torch.from_numpy(p).cuda()
    order = scenes.fps_order(x, start).cuda()
    return x[order].contiguous()


@pytest.mark.parametrize("seed,n", [(0, 3000), (1, 24000)])
def test_tree_queries_equal_reference_cuda(seed, n):
    ref = _bind_bvh(_lib("gsa_bvh"))
    ours = abi.bvh_lib()
    x = _room(seed, n)
    hr, ho = abi.Handle(ref, x, 1, 16), abi.Handle(ours, x, 1, 16)
    assert hr.code == 0 and ho.code == 0
    sizes = [n >> (2 * l) for l in range(4)]
    for level, r in zip(range(4), [0.1, 0.2, 0.4, 0.8]):
        m = sizes[level]
        q = x[:m]
        for ns in [32, 8]:
            cr, outr, fbr = hr.ball(q, m, level, r, ns)
            co, outo, fbo = ho.ball(q, m, level, r, ns)
            assert cr == 0 and co == 0
            assert torch.equal(outr, outo), (level, ns)
        if level < 3:
            qq = x[: sizes[level]]
            m3 = sizes[level + 1]
            cr, dr, ir, _ = hr.knn(qq, m3, level + 1)
            co, do, io, _ = ho.knn(qq, m3, level + 1)
            assert cr == 0 and co == 0
            assert torch.equal(dr, do) and torch.equal(ir, io), level
    assert hr.free() == 0 and ho.free() == 0


def test_scan_kernels_equal_reference_cuda():
    ref = _lib("reference_queries")
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    ref.ball.argtypes = [I, I, I, F, I, P, P, P, P]
    ref.nn3.argtypes = [I, I, I, P, P, P, P, P]
    rng = np.random.default_rng(3)
    b, n, m = 2, 1000, 400
    x = torch.from_numpy(rng.normal(size=(b, n, 3)).astype(np.float32)).cuda()
    q = torch.cat([x[:, :300], torch.from_numpy(rng.normal(size=(b, 100, 3)).astype(np.float32) * 3).cuda()], 1).contiguous()
    for r, ns in [(0.3, 32), (0.8, 16), (0.0, 4)]:
        out_r = torch.zeros((b, m, ns), dtype=torch.int32, device="cuda")
        assert ref.ball(b, n, m, r, ns, q.data_ptr(), x.data_ptr(), out_r.data_ptr(), abi.stream()) == 0
        code, out_o = abi.scan_ball(q, x, r, ns, init=torch.zeros((b, m, ns), dtype=torch.int32, device="cuda"), b=b)
        assert code == 0 and torch.equal(out_r, out_o)
    d_r = torch.empty((b, m, 3), device="cuda")
    i_r = torch.empty((b, m, 3), dtype=torch.int32, device="cuda")
    assert ref.nn3(b, m, n, q.data_ptr(), x.data_ptr(), d_r.data_ptr(), i_r.data_ptr(), abi.stream()) == 0
    code, d_o, i_o = abi.scan_nn3(q, x, b=b)
    assert code == 0 and torch.equal(d_r, d_o) and torch.equal(i_r, i_o)


def test_scan_nn3_overflow_and_nonfinite_equal_reference_cuda():
    """Squared distances that overflow to +inf, and NaN/inf coordinates: the
    reference's double comparison against 1e40 rejects +inf and NaN exactly
    like the finite test, so outputs agree with ours and with the oracle."""
    from oracle import numpy_oracle as orc

    ref = _lib("reference_queries")
    P, I = ctypes.c_void_p, ctypes.c_int
    ref.nn3.argtypes = [I, I, I, P, P, P, P, P]
    x = np.array([[0, 0, 0], [2e19, 0, 0], [np.inf, 0, 0], [np.nan, 1, 1], [1e19, 1e19, 0], [3, 0, 0], [-2e19, 0, 0]], np.float32)
    q = np.array([[0, 0, 0], [1e19, 0, 0], [-3e19, 5, 5], [np.nan, 0, 0], [1, 1, 1]], np.float32)
    xt = torch.from_numpy(x).cuda()
    qt = torch.from_numpy(q).cuda()
    d_r = torch.empty((1, len(q), 3), device="cuda")
    i_r = torch.empty((1, len(q), 3), dtype=torch.int32, device="cuda")
    assert ref.nn3(1, len(q), len(x), qt.data_ptr(), xt.data_ptr(), d_r.data_ptr(), i_r.data_ptr(), abi.stream()) == 0
    code, d_o, i_o = abi.scan_nn3(qt, xt)
    assert code == 0
    ed, ei = orc.nn_oracle(q, x)
    assert np.array_equal(d_r.cpu().numpy()[0], ed) and np.array_equal(i_r.cpu().numpy()[0], ei)
    assert torch.equal(d_r, d_o) and torch.equal(i_r, i_o)
