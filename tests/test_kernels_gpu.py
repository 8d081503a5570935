# SPDX-License-Identifier: Apache-2.0
"""GPU parity of every kernel, called through the C ABI, against the oracle.

Bar: bit-exact IDs and squared distances (``np.array_equal``) on seeded
inputs, covering the reference's edge rules: duplicates, strict radius,
zero and FLT_MAX radii, FP32 scale extremes, non-finite coordinates,
supports of 1..5 points, K = 1..32, every prefix level, more queries than
support points, unrelated query sets, batched forests, the untouched-row
scan contract and the stack-overflow fallback.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import numpy_oracle as orc
from tests import abi

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def levels_of(n):
    return [n >> (2 * l) for l in range(4)]


def check_ball(h, x, q, m, level, r, ns, unordered=False):
    code, out, fb = h.ball(cuda(q), m, level, r, ns, unordered=unordered)
    assert code == 0
    want = orc.ball_oracle_fast(q, x[:m], r, ns)
    got = out.cpu().numpy()
    assert np.array_equal(got, want), (len(x), m, level, r, ns)
    return fb


def check_knn(h, x, q, m, level, unordered=False):
    code, d, ix, fb = h.knn(cuda(q), m, level, unordered=unordered)
    assert code == 0
    ed, ei = orc.nn_oracle_fast(q, x[:m])
    assert np.array_equal(d.cpu().numpy(), ed), (len(x), m, level)
    assert np.array_equal(ix.cpu().numpy(), ei), (len(x), m, level)
    return fb


# "gsa_bvh" scans support prefixes up to 512 (radius) / 128 (3NN) points and
# walks the tree above (packet-frontier radius and 3NN kernels);
# "gsa_bvh_walk" walks the tree for every size; "gsa_bvh_ordered" does so
# with the per-query walks (ordered radius, nearest-first 3NN).
LIBS = ["gsa_bvh", "gsa_bvh_walk", "gsa_bvh_ordered"]


@pytest.mark.parametrize("lib_name", LIBS)
@pytest.mark.parametrize("n", [1, 2, 3, 5, 16, 17, 33, 100, 257, 1000, 4099, 9000])
@pytest.mark.parametrize("leaf", [1, 4, 16, 32])
def test_prefix_tree_all_levels(n, leaf, lib_name):
    rng = np.random.default_rng(n * 31 + leaf)
    x = rng.normal(size=(n, 3)).astype(np.float32)
    if n > 1:
        x[n // 2] = x[0]  # duplicate
    lib = abi.bvh_lib(lib_name)
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=leaf)
    assert h.code == 0
    for level, m in enumerate(levels_of(n)):
        if m < 1:
            continue
        q = np.concatenate([x[:m], rng.normal(size=(7, 3)).astype(np.float32)])
        for r, ns in [(0.0, 8), (0.5, 1), (0.9, 32), (2.0, 16), (50.0, 32)]:
            fb = check_ball(h, x, q, m, level, r, ns)
            assert fb.item() == 0
        if m >= 3:
            assert check_knn(h, x, q, m, level).item() == 0
    # level -1 uses the all-point bounds with any m
    for m in sorted({1, max(1, n // 3), n}):
        check_ball(h, x, x[: max(1, n // 2)], m, -1, 0.7, 8)
        if m >= 3:
            check_knn(h, x, x[: max(1, n // 2)], m, -1)
    assert h.free() == 0


def test_plain_tree_and_invalid_levels():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(500, 3)).astype(np.float32)
    lib = abi.bvh_lib()
    h = abi.Handle(lib, cuda(x), prefix=0, leaf=16)
    assert h.code == 0
    check_ball(h, x, x[:100], 500, -1, 0.4, 32)
    check_ball(h, x, x[:100], 123, -1, 0.4, 32)
    check_knn(h, x, x[:100], 200, -1)
    q = cuda(x[:10])
    assert h.ball(q, 500, 0, 0.4, 8)[0] == 0  # level 0 == all points
    assert h.ball(q, 125, 1, 0.4, 8)[0] == -2  # no prefix levels stored
    assert h.ball(q, 501, -1, 0.4, 8)[0] == -2
    assert h.ball(q, 0, -1, 0.4, 8)[0] == -2
    assert h.ball(q, 10, -1, 0.4, 33)[0] == -2
    assert h.knn(q, 2, -1)[0] == -2
    assert h.free(async_free=0) == 0
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    assert h.ball(q, 126, 1, 0.4, 8)[0] == -2  # m beyond the level-1 prefix (125)
    assert h.ball(q, 125, 4, 0.4, 8)[0] == -2
    assert h.ball(q, 125, 1, 0.4, 8)[0] == 0
    empty = cuda(np.zeros((0, 3)))
    assert h.ball(empty, 125, 1, 0.4, 8)[0] == 0
    assert h.free() == 0


@pytest.mark.parametrize("lib_name", LIBS)
def test_scales_radii_and_nonfinite(lib_name):
    rng = np.random.default_rng(11)
    lib = abi.bvh_lib(lib_name)
    for scale in [0.0, 1e-25, 1.0, 1e20]:
        x = (rng.normal(size=(300, 3)) * scale).astype(np.float32)
        h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
        s32 = float(np.float32(scale))
        up = float(np.nextafter(np.float32(scale), np.float32(np.inf)))
        for r in [0.0, s32, up, 3.0e38]:
            for ns in [1, 8, 32]:
                check_ball(h, x, x[:40], 300, 0, r, ns)
                check_ball(h, x, x[:18], 75, 1, r, ns)
        check_knn(h, x, x[:40], 300, 0)
        check_knn(h, x, x[:40], 18, 2)
        h.free()
    # non-finite support and query coordinates never qualify and never break pruning
    x = rng.normal(size=(400, 3)).astype(np.float32)
    x[5, 0] = np.nan
    x[9, 1] = np.inf
    x[17, 2] = -np.inf
    x[33] = [np.inf, np.inf, np.inf]
    x[40] = [3e38, 0, 0]
    x[41] = [-3e38, 0, 0]
    q = np.concatenate([x[:60], np.array([[np.nan, 0, 0], [np.inf, 0, 0], [1e30, 1e30, 1e30]], np.float32)])
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=8)
    for r in [0.5, 1.5, 3.0e38]:
        check_ball(h, x, q, 400, 0, r, 32)
        check_ball(h, x, q, 100, 1, r, 5)
    check_knn(h, x, q, 400, 0)
    check_knn(h, x, q, 25, 2)
    h.free()


@pytest.mark.parametrize("lib_name", LIBS)
def test_duplicates_and_ties(lib_name):
    rng = np.random.default_rng(12)
    base = rng.integers(0, 4, size=(64, 3)).astype(np.float32)  # lattice, many equal distances
    x = base[rng.integers(0, 64, size=3000)]
    lib = abi.bvh_lib(lib_name)
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    q = np.concatenate([x[:200], base + 0.5])
    for level, m in enumerate(levels_of(3000)):
        check_ball(h, x, q, m, level, 1.0, 32)
        check_ball(h, x, q, m, level, float(np.sqrt(np.float32(2.0))), 7)
        check_knn(h, x, q, m, level)
    h.free()


@pytest.mark.parametrize("lib_name", LIBS)
def test_dense_neighbourhoods_first_k(lib_name):
    """Queries with 33-256 hits (the dense-neighbourhood frontier), with more
    (the ordered walk) and with fewer in the same packets, K from 1 to 32:
    a lattice of 40 points repeated ~60 times plus scattered points, radii
    taking one lattice point's copies, or its axis neighbours too."""
    rng = np.random.default_rng(17)
    base = rng.integers(0, 5, size=(40, 3)).astype(np.float32)
    x = np.concatenate([base[rng.integers(0, 40, size=2400)],
                        rng.random((600, 3)).astype(np.float32) * 5.0])
    x = x[rng.permutation(len(x))]
    lib = abi.bvh_lib(lib_name)
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    q = np.concatenate([x[:1500], base + np.float32(0.25)])
    for r in (0.5, 1.01):
        for ns in (1, 5, 16, 32):
            check_ball(h, x, q, 3000, 0, r, ns)
        check_ball(h, x, q[:750], 750, 1, r, 32)
    h.free()


@pytest.mark.parametrize("lib_name", LIBS)
def test_queries_outnumber_support_and_unrelated_queries(lib_name):
    rng = np.random.default_rng(13)
    x = rng.random((2000, 3)).astype(np.float32)
    lib = abi.bvh_lib(lib_name)
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    big = np.concatenate([x, rng.random((3000, 3)).astype(np.float32)])
    check_ball(h, x, big, 2000, 0, 0.05, 32)
    check_knn(h, x, big, 500, 1)
    unrelated = rng.random((777, 3)).astype(np.float32) * 1.2 - 0.1
    check_ball(h, x, unrelated, 125, 2, 0.2, 16)
    check_knn(h, x, unrelated, 31, 3)
    h.free()


@pytest.mark.parametrize("lib_name", LIBS)
def test_unordered_entries_for_other_query_sets(lib_name):
    """query_ball_bvh_unordered / query_bvh_unordered (queries walked in
    their own Morton order): the support's points shuffled, unrelated points,
    more queries than support points, non-finite queries; rows equal the
    oracle and the ordered entries.  The default library takes the tree (not
    the scan) only for large query sets, so it runs a 24,000-point room (and
    40,000 queries: the multi-launch key sort above 32,768); the tree-only
    variants run a 6,000-point room."""
    rng = np.random.default_rng(31)
    from gsa_b200 import scenes

    big = lib_name == "gsa_bvh"
    n = 24000 if big else 6000
    x = scenes.room(2, n=n)[0].astype(np.float32)
    lib = abi.bvh_lib(lib_name)
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    shuffled = x[rng.permutation(n)]
    unrelated = scenes.room(3, n=n)[0].astype(np.float32)
    odd = unrelated[: n // 2].copy()
    odd[::97, 1] = np.nan
    odd[5::101, 0] = np.inf
    sets = [shuffled, odd]
    if big:
        sets.append(np.concatenate([unrelated, rng.random((16000, 3)).astype(np.float32) * 3.0]))
    else:
        sets += [unrelated, np.concatenate([unrelated, shuffled[:2000]])]
    for q in sets:
        check_ball(h, x, q, n, 0, 0.1, 32, unordered=True)
        check_knn(h, x, q, n // 4, 1, unordered=True)
    if not big:
        check_ball(h, x, unrelated, n // 4, 1, 0.2, 16, unordered=True)
        check_knn(h, x, unrelated, n // 16, 2, unordered=True)
    # the ordered entries give the same rows
    rows = []
    for unordered in (False, True):
        code, out, _ = h.ball(cuda(shuffled), n, 0, 0.1, 32, unordered=unordered)
        code2, d, ix, _ = h.knn(cuda(shuffled), n // 4, 1, unordered=unordered)
        assert code == code2 == 0
        rows.append((out, d, ix))
    assert all(torch.equal(u, v) for u, v in zip(*rows))
    h.free()


def test_tree_and_session_pick_the_query_order():
    """Tree.ball / Tree.query and the session walk query arrays that start at
    the support's first row in the tree's leaf order and other query sets in
    their own Morton order; both equal the oracle."""
    from gsa_b200 import QuerySession, Tree, scenes

    x = scenes.room(4, n=24000)[0].astype(np.float32)
    X = cuda(x)
    rng = np.random.default_rng(5)
    q = x[rng.permutation(24000)]
    Q = cuda(q)
    t = Tree(X, prefix=True)
    out = torch.empty(24000, 32, dtype=torch.int32, device="cuda")
    t.ball(Q, 24000, 0.1, 32, out)
    assert np.array_equal(out.cpu().numpy(), orc.ball_oracle_fast(q, x, 0.1, 32))
    d = torch.empty(24000, 3, device="cuda")
    ix = torch.empty(24000, 3, dtype=torch.int32, device="cuda")
    t.query(Q, 6000, d, ix)
    ed, ei = orc.nn_oracle_fast(q, x[:6000])
    assert np.array_equal(d.cpu().numpy(), ed) and np.array_equal(ix.cpu().numpy(), ei)
    t.close()
    with QuerySession(threshold=32) as s:
        s.ball_into(Q, X, 0.1, 32, out)
        s.nn_into(Q, X[:6000], d, ix)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), orc.ball_oracle_fast(q, x, 0.1, 32))
        assert np.array_equal(d.cpu().numpy(), ed) and np.array_equal(ix.cpu().numpy(), ei)


@pytest.mark.parametrize("lib_name", LIBS)
def test_knn_bounds_from_sparse_and_tied_supports(lib_name):
    """3NN where most window members are non-finite (queries without a
    finite window bound take the per-query walk), where ties are massive (a
    query's candidate buffer is cut to its best three many times), and with a
    support prefix smaller than the level (window members with ID >= m)."""
    rng = np.random.default_rng(21)
    lib = abi.bvh_lib(lib_name)
    n = 6000
    x = rng.random((n, 3)).astype(np.float32)
    x[rng.random(n) < 0.9] = np.nan  # 90 % non-finite support points
    q = np.concatenate([rng.random((1500, 3)).astype(np.float32), x[:500]])
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    for level, m in enumerate(levels_of(n)):
        check_knn(h, x, q, m, level)
    check_knn(h, x, q, 1000, 1)  # m below the level-1 prefix of 1500
    h.free()
    lattice = rng.integers(0, 3, size=(27, 3)).astype(np.float32)
    x = lattice[rng.integers(0, 27, size=n)]  # ~220 copies of each point
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=16)
    for level, m in enumerate(levels_of(n)):
        check_knn(h, x, x[: m], m, level)
    h.free()


def test_small_stack_fallback_is_exact_and_counted():
    rng = np.random.default_rng(14)
    x = rng.random((5000, 3)).astype(np.float32)
    lib = abi.bvh_lib("gsa_bvh_stack4")
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=4)
    fb = check_ball(h, x, x[:1250], 1250, 1, 0.3, 32)
    assert fb.item() > 0
    fb = check_knn(h, x, x[:600], 5000, 0)
    assert fb.item() > 0
    h.free()


@pytest.mark.parametrize("n,leaf", [(5000, 4), (5000, 16), (700, 32), (60, 4)])
def test_node_capacity_overflow_is_exact_and_counted(n, leaf):
    """A tree whose kept nodes exceed its stored-node capacity (8 in this
    build) is flagged by the build; its queries take the exact scans, are
    counted as fallbacks and equal the oracle on every level."""
    rng = np.random.default_rng(16 + n + leaf)
    x = rng.random((n, 3)).astype(np.float32)
    lib = abi.bvh_lib("gsa_bvh_cap8")
    h = abi.Handle(lib, cuda(x), prefix=1, leaf=leaf)
    assert h.code == 0
    for level in range(4):
        m = n >> (2 * level)
        if m < 3:
            break
        fb = check_ball(h, x, x[:m], m, level, 0.2, 32)
        assert fb.item() > 0
        fb = check_knn(h, x, x[:m], m, level)
        assert fb.item() > 0
    h.free()


@pytest.mark.parametrize("lib_name", LIBS + ["gsa_bvh_cap8"])
def test_forest_batch_equals_oracle_per_scene(lib_name):
    rng = np.random.default_rng(15)
    sizes = [1, 3, 17, 700, 4096, 2500, 12000]
    xs = [rng.normal(size=(n, 3)).astype(np.float32) for n in sizes]
    seg = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    x = cuda(np.concatenate(xs))
    lib = abi.bvh_lib(lib_name)
    h = ctypes.c_void_p()
    seg_c = (ctypes.c_int * len(seg))(*seg.tolist())
    assert lib.build_bvh_batch(x.data_ptr(), seg_c, len(sizes), 1, 16, ctypes.byref(h), abi.stream()) == 0
    trees = ctypes.c_int()
    assert lib.bvh_info(h, ctypes.byref(trees), None, None, None) == 0 and trees.value == len(sizes)
    for level in [0, 1, 2]:
        qs = [xi[: max(0, len(xi) >> (2 * level))] for xi in xs]
        qseg = np.concatenate([[0], np.cumsum([len(a) for a in qs])]).astype(np.int32)
        q = cuda(np.concatenate(qs))
        qseg_d = torch.from_numpy(qseg).cuda()
        qseg_h = (ctypes.c_int * len(qseg))(*qseg.tolist())
        out = torch.full((len(q), 32), -9, dtype=torch.int32, device="cuda")
        fb = torch.zeros(1, dtype=torch.int32, device="cuda")
        code = lib.query_ball_bvh_batch(h, q.data_ptr(), None, qseg_d.data_ptr(), qseg_h, 0, level, 0.3, 32, out.data_ptr(), fb.data_ptr(), abi.stream())
        ok_sizes = all(len(xi) >> (2 * level) >= 1 for xi, qq in zip(xs, qs) if len(qq))
        if not ok_sizes:
            assert code == -2
            continue
        assert code == 0
        got = out.cpu().numpy()
        for i, (xi, qi) in enumerate(zip(xs, qs)):
            m = len(xi) >> (2 * level)
            want = orc.ball_oracle_fast(qi, xi[:m], 0.3, 32)
            assert np.array_equal(got[qseg[i]:qseg[i + 1]], want), (i, level)
        if all(len(xi) >> (2 * level) >= 3 for xi, qq in zip(xs, qs) if len(qq)):
            d = torch.empty((len(q), 3), device="cuda")
            ix = torch.empty((len(q), 3), dtype=torch.int32, device="cuda")
            assert lib.query_bvh_batch(h, q.data_ptr(), None, qseg_d.data_ptr(), qseg_h, 0, level, d.data_ptr(), ix.data_ptr(), fb.data_ptr(), abi.stream()) == 0
            for i, (xi, qi) in enumerate(zip(xs, qs)):
                m = len(xi) >> (2 * level)
                ed, ei = orc.nn_oracle_fast(qi, xi[:m])
                assert np.array_equal(d.cpu().numpy()[qseg[i]:qseg[i + 1]], ed)
                assert np.array_equal(ix.cpu().numpy()[qseg[i]:qseg[i + 1]], ei)
    assert lib.free_bvh(h, 1, abi.stream()) == 0


def test_scan_kernels_contract():
    rng = np.random.default_rng(16)
    b, n, m = 3, 900, 300
    x = rng.normal(size=(b, n, 3)).astype(np.float32)
    x[:, 4] = x[:, 0]
    q = np.concatenate([x[:, :200], rng.normal(size=(b, 100, 3)).astype(np.float32) * 4], axis=1)
    for r, ns in [(0.0, 4), (0.3, 1), (0.6, 32), (1.0, 40)]:
        init = torch.full((b, m, ns), -3, dtype=torch.int32, device="cuda")
        code, out = abi.scan_ball(cuda(q), cuda(x), r, ns, init=init, b=b)
        assert code == 0
        got = out.cpu().numpy()
        for i in range(b):
            want = orc.ball_scan_untouched(q[i], x[i], r, ns, np.full((m, ns), -3, np.int32))
            assert np.array_equal(got[i], want), (r, ns, i)
    code, d, ix = abi.scan_nn3(cuda(q), cuda(x), b=b)
    assert code == 0
    for i in range(b):
        ed, ei = orc.nn_oracle_fast(q[i], x[i])
        assert np.array_equal(d.cpu().numpy()[i], ed) and np.array_equal(ix.cpu().numpy()[i], ei)
    # fewer than three support points: (inf, 0) fill; non-finite skipped
    xs = np.array([[[0, 0, 0], [np.inf, 0, 0]]], np.float32)
    code, d, ix = abi.scan_nn3(cuda(q[:1, :5]), cuda(xs))
    ed, ei = orc.nn_oracle(q[0, :5], xs[0])
    assert np.array_equal(d.cpu().numpy()[0], ed) and np.array_equal(ix.cpu().numpy()[0], ei)


def test_reuse_kernels():
    lib = abi.bvh_lib()
    a = torch.tensor([0.0, 1.0, float("nan"), 2.0, -0.0], device="cuda")
    b = torch.tensor([-0.0, 1.0, float("nan"), 2.0, 0.0], device="cuda")
    big = torch.randn(1 << 20, 3, device="cuda")
    big2 = big.clone()
    big3 = big.clone()
    big3[123457, 1] = torch.nextafter(big3[123457, 1], torch.tensor(float("inf"), device="cuda"))
    pairs = [(a[:2], b[:2]), (a[2:3], b[2:3]), (a[3:], b[3:]), (big, big2), (big, big3), (big[1:], big2[1:])]
    n = len(pairs)
    flags = torch.full((n,), 9, dtype=torch.int32, device="cuda")
    A = (ctypes.c_void_p * n)(*[p[0].data_ptr() for p in pairs])
    B = (ctypes.c_void_p * n)(*[p[1].data_ptr() for p in pairs])
    C = (ctypes.c_longlong * n)(*[p[0].numel() for p in pairs])
    assert lib.coords_mismatch(n, A, B, C, flags.data_ptr(), abi.stream()) == 0
    want = [0 if torch.equal(u, v) else 1 for u, v in pairs]
    assert flags.tolist() == want == [0, 1, 0, 0, 1, 0]
    # reuse_rows picks the first candidate whose two flags are zero
    cached = [torch.randint(0, 1000, (50, 32), dtype=torch.int32, device="cuda") for _ in range(3)]
    fl = torch.tensor([1, 0, 0, 1, 0, 0], dtype=torch.int32, device="cuda")
    src = (ctypes.c_void_p * 3)(*[c.data_ptr() for c in cached])
    for rows, cols in [(50, 32), (17, 5), (1, 1)]:
        out = torch.full((rows, cols), -1, dtype=torch.int32, device="cuda")
        hit = torch.full((1,), -5, dtype=torch.int32, device="cuda")
        assert lib.reuse_rows(3, src, fl.data_ptr(), 32, rows, cols, out.data_ptr(), hit.data_ptr(), abi.stream()) == 0
        assert hit.item() == 2 and torch.equal(out, cached[2][:rows, :cols])
    fl = torch.ones(6, dtype=torch.int32, device="cuda")
    out = torch.full((5, 4), -1, dtype=torch.int32, device="cuda")
    hit = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.reuse_rows(3, src, fl.data_ptr(), 32, 5, 4, out.data_ptr(), hit.data_ptr(), abi.stream()) == 0
    assert hit.item() == -1 and (out == -1).all()
    out = torch.empty((50, 7), dtype=torch.int32, device="cuda")
    assert lib.gather_rows(cached[1].data_ptr(), 32, 50, 7, out.data_ptr(), abi.stream()) == 0
    assert torch.equal(out, cached[1][:, :7])


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("case", ["small", "large", "many_pairs"])
def test_session_lookup_paths(case, pinned):
    """session_lookup: one cluster launch for lookups of a few MB and at
    most 64 pairs (flags written straight into pinned host memory, or copied
    when the host buffer is pageable), the four-operation path otherwise;
    flags as torch.equal, rows of the first fully matching memo candidate."""
    lib = abi.bvh_lib()
    n = {"small": 6000, "large": 1 << 20, "many_pairs": 500}[case]
    x = torch.randn(n, 3, device="cuda")
    x[7, 2] = float("nan")  # NaN never equals itself: x never equals a copy
    y = torch.randn(n, 3, device="cuda")
    z = y.clone()
    z[n - 1, 0] = -0.0 if z[n - 1, 0] == 0 else z[n - 1, 0]
    w = y.clone()
    w[n // 2, 1] = torch.nextafter(w[n // 2, 1], torch.tensor(float("inf"), device="cuda"))
    # memo pairs: candidate 0 (NaN in x, one ulp in w) differs, candidate 1
    # (y, z) / (y[:n//4], z) matches
    pairs = [(x, x.clone()), (y, w), (y, z), (y[: n // 4], z)]
    memo = 2
    if case == "many_pairs":
        pairs += [(y, z) if i % 3 else (y, w) for i in range(70)]
    rows, cols = n // 4, 32
    cached = [torch.randint(0, 1 << 20, (n, 32), dtype=torch.int32, device="cuda") for _ in range(memo)]
    count = len(pairs)
    A = (ctypes.c_void_p * count)(*[p[0].data_ptr() for p in pairs])
    B = (ctypes.c_void_p * count)(*[p[1].data_ptr() for p in pairs])
    C = (ctypes.c_longlong * count)(*[p[0].numel() for p in pairs])
    src = (ctypes.c_void_p * memo)(*[c.data_ptr() for c in cached])
    flags = torch.full((count,), 9, dtype=torch.int32, device="cuda")
    want = [0 if torch.equal(u, v[: u.shape[0]]) else 1 for u, v in pairs]
    assert want[:4] == [1, 1, 0, 0]
    for rep in range(2):  # twice in a row: nothing of the first call leaks
        out = torch.full((rows, cols), -1, dtype=torch.int32, device="cuda")
        if pinned:
            host_t = torch.full((count,), 7, dtype=torch.int32, pin_memory=True)
            host = (ctypes.c_int * count).from_address(host_t.data_ptr())
        else:
            host = (ctypes.c_int * count)(*([7] * count))
        code = lib.session_lookup(count, A, B, C, memo, src, 32, rows, cols, out.data_ptr(),
                                  flags.data_ptr(), host, abi.stream())
        assert code == 0
        assert list(host) == want and flags.tolist() == want
        assert torch.equal(out, cached[1][:rows, :cols])
    # no matching candidate: out untouched
    out = torch.full((rows, cols), -1, dtype=torch.int32, device="cuda")
    host = (ctypes.c_int * count)()
    assert lib.session_lookup(2, A, B, C, 1, src, 32, rows, cols, out.data_ptr(), flags.data_ptr(), host,
                              abi.stream()) == 0
    assert list(host)[:2] == [1, 1] and (out == -1).all()


def test_fps_order_matches_sequential_rule():
    from gsa_b200 import scenes
    from oracle import fps as fps_cpu

    pts = []
    starts = []
    for s in range(3):
        p, st = scenes.room(s, n=3000)
        pts.append(p)
        starts.append(st)
    pts[1][10] = pts[1][20]  # duplicate coordinates
    x = torch.from_numpy(np.stack(pts)).cuda()
    order = scenes.fps_order(x, starts).numpy()
    for i in range(3):
        assert np.array_equal(order[i], fps_cpu.fps_order(pts[i], starts[i]))
        assert sorted(order[i].tolist()) == list(range(3000))


def test_fps_cooperative_grid_matches_single_block():
    from gsa_b200 import scenes

    p, st = scenes.room(7, n=20000)
    p[100] = p[200]
    x = torch.from_numpy(p).cuda()
    small = scenes.fps_order(x, st, large=False)
    large = scenes.fps_order(x, st, large=True)
    assert torch.equal(small, large)


def test_fps_grid_barrier_timeout_sets_error_and_returns():
    """In a test build where one block of the cooperative FPS grid leaves
    before its first barrier, every other block's bounded wait runs out: the
    kernel ends, the error flag reads 1, and the context stays usable (the
    regular library then computes the same order correctly)."""
    from gsa_b200 import _library, scenes

    p, st = scenes.room(9, n=6000)
    x = torch.from_numpy(p).cuda()
    P_, I_ = ctypes.c_void_p, ctypes.c_int
    drop = _library.load("gsa_fps_drop")
    drop.fps_order_large.argtypes = [I_, P_, I_, P_, P_, P_, P_]
    drop.fps_order_large.restype = I_
    order = torch.full((len(p),), -1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(16, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    code = drop.fps_order_large(len(p), x.data_ptr(), int(st), order.data_ptr(), scratch.data_ptr(),
                                err.data_ptr(), abi.stream())
    assert code == 0
    torch.cuda.synchronize()
    assert err.item() == 1
    assert (order[1:] == -1).all()  # no step completed after the first barrier
    small = scenes.fps_order(x, st, large=False)
    large = scenes.fps_order(x, st, large=True)
    assert torch.equal(small, large)


def test_furthest_point_sample_op_matches_sequential_rule():
    """The PointNet++-style FPS op: first m indices from index 0, exact FP32
    distances, ties to the lowest index (a lattice makes many exact ties),
    NaN points chosen first; small scenes in shared memory, a 60,000-point
    scene on the cooperative grid."""
    from gsa_b200 import sampling
    from oracle import fps as fps_cpu

    rng = np.random.default_rng(4)
    lat = np.stack(np.meshgrid(*[np.arange(12, dtype=np.float32)] * 3, indexing="ij"), -1).reshape(-1, 3)
    pts = np.stack([
        rng.normal(size=(1728, 3)).astype(np.float32),
        lat * np.float32(0.25),
        rng.random((1728, 3)).astype(np.float32),
    ])
    pts[2, 5] = pts[2, 9]
    pts[2, 40, 1] = np.nan
    x = torch.from_numpy(pts).cuda()
    for m in (1, 432, 1728):
        idx = sampling.furthest_point_sample(x, m).cpu().numpy()
        for i in range(3):
            assert np.array_equal(idx[i], fps_cpu.fps_order(pts[i], 0, m)), (i, m)
    assert sampling.furthest_point_sample(x, 0).shape == (3, 0)
    big = rng.normal(size=(1, 60000, 3)).astype(np.float32)
    idx = sampling.furthest_point_sample(torch.from_numpy(big).cuda(), 300).cpu().numpy()
    assert np.array_equal(idx[0], fps_cpu.fps_order(big[0], 0, 300))
    with pytest.raises(ValueError):
        sampling.furthest_point_sample(x, 1729)
    lib = abi.bvh_lib()
    assert lib.furthest_point_sample(1, 10, 11, None, None, None, None) == -2
    assert lib.furthest_point_sample(1, 60000, 5, x.data_ptr(), None, x.data_ptr(), None) == -2  # temp needed


def test_pool_reports_usage():
    from gsa_b200 import runtime

    runtime.pool_reset_peak()
    x = torch.randn(100000, 3, device="cuda")
    t = runtime.Tree(x, prefix=True)
    torch.cuda.synchronize()
    mem = runtime.pool_memory()
    assert mem["native_pool_used_peak_bytes"] >= 100000 * 16
    assert mem["native_pool_reserved_peak_bytes"] >= mem["native_pool_used_peak_bytes"]
    t.close()
