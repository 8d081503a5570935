# SPDX-License-Identifier: Apache-2.0
"""CPU: pin the oracle and the session host logic to the reference's goldens.

The fixture ``tests/golden/query_session_correctness.json`` holds, for each
of the 94 calls of the reference test ``tests/check_queries.py``, the SHA-256
of the int32 radius rows and the session statistics after the call, as the
reference committed them (``data/query_session/correctness.json``).
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import numpy_oracle as orc
from tests import sequence
from tests.fake_ops import make_oracle_session

GOLDEN = json.loads((Path(__file__).parent / "golden" / "query_session_correctness.json").read_text())


@pytest.fixture(scope="module")
def replay():
    return sequence.run(make_oracle_session, "cpu")


def test_golden_fixture_shape():
    recs = GOLDEN["records"]
    assert len(recs) == 94
    assert sum(r["op"] == "ball" for r in recs) == 69
    assert sum("ids_sha256" in r for r in recs) == 69


def test_oracle_reproduces_all_69_radius_hashes(replay):
    got = [r for r in replay if r["op"] == "ball"]
    want = [r for r in GOLDEN["records"] if r["op"] == "ball"]
    assert len(got) == len(want) == 69
    for g, w in zip(got, want):
        assert (g["label"], g["n"], g["q"], g["k"]) == (w["label"], w["n"], w["q"], w["k"])
        assert g["r"] == w["r"]
        assert g["ids_sha256"] == w["ids_sha256"], g["label"]


def test_session_host_logic_reproduces_all_94_stats(replay):
    for g, w in zip(replay, GOLDEN["records"]):
        assert (g["op"], g["label"], g["n"], g["q"]) == (w["op"], w["label"], w["n"], w["q"])
        assert g["stats"] == w["stats"], (g["label"], g["stats"], w["stats"])


def test_nn_records_match_literal_oracle(replay):
    for g in replay:
        if g["op"] != "nn":
            continue
        ed, ei = orc.nn_oracle(g["qv"], g["x"])
        assert np.array_equal(g["d"], ed) and np.array_equal(g["ids"], ei)


def test_fast_oracles_equal_literal_ones():
    rng = np.random.default_rng(5)
    for n, nq, scale in [(1, 4, 1.0), (17, 13, 1.0), (300, 64, 1.0), (97, 9, 1e20), (50, 7, 1e-25), (40, 5, 0.0)]:
        x = (rng.normal(size=(n, 3)) * scale).astype(np.float32)
        x[n // 2] = x[0]
        q = np.concatenate([x[: nq // 2], (rng.normal(size=(nq - nq // 2, 3)) * scale).astype(np.float32)])
        for r in [0.0, 0.3 * scale, scale, 2.5 * scale]:
            for k in [1, 5, 32]:
                assert np.array_equal(orc.ball_oracle(q, x, r, k), orc.ball_oracle_fast(q, x, r, k))
        if n >= 1:
            a = orc.nn_oracle(q, x)
            b = orc.nn_oracle_fast(q, x)
            assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_oracle_edge_rules():
    # strict qualification: a point at exactly r is excluded
    x = np.array([[0.25, 0, 0], [0.1, 0, 0], [0, 0, 0]], np.float32)
    q = np.zeros((1, 3), np.float32)
    assert orc.ball_oracle(q, x, 0.25, 4).tolist() == [[1, 2, 1, 1]]
    # no hit -> zero row; scan contract leaves the row untouched
    assert orc.ball_oracle(q, x + 10, 0.25, 3).tolist() == [[0, 0, 0]]
    init = np.full((1, 3), 7, np.int32)
    assert orc.ball_scan_untouched(q, x + 10, 0.25, 3, init).tolist() == [[7, 7, 7]]
    # 3NN: ties by lower ID, non-finite distances skipped, (inf, 0) fill
    x = np.array([[1, 0, 0], [0, 1, 0], [np.inf, 0, 0], [0, 0, 1], [1e30, 0, 0]], np.float32)
    d, i = orc.nn_oracle(q, x)
    assert i.tolist() == [[0, 1, 3]] and d.tolist() == [[1.0, 1.0, 1.0]]
    d, i = orc.nn_oracle(q, x[2:3])
    assert i.tolist() == [[0, 0, 0]] and np.isinf(d).all()


def test_index_candidate_misses_host_logic():
    """Index lookups whose first candidate's root differs: the answer comes
    from the matching or newly built index, the statistics count as GSA's."""
    from tests.index_miss import INDEX_MISS_STATS, index_candidate_misses

    got, want, stats = index_candidate_misses(make_oracle_session, "cpu")
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    for key, value in INDEX_MISS_STATS.items():
        assert stats[key] == value, (key, stats)
