# SPDX-License-Identifier: Apache-2.0
"""GPU: the drop-in Python API against the reference's own tests.

* the 94-call sequence of GSA ``tests/check_queries.py`` through the real
  ``QuerySession``: all 69 radius-row SHA-256 values and all 94 statistics
  dicts equal the reference's committed records, 3NN equals the oracle;
* GSA ``tests/check_integration.py``: fixed-graph ``prefix``/``scale``
  outputs equal the unpatched operators bit for bit with exactly one radius
  hit, wrappers restored after an exception, invalid buffers rejected;
* GSA ``examples/query_session.py``: row reuse and shared-prefix index reuse.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import numpy_oracle as orc
from tests import sequence

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "query_session_correctness.json").read_text())


def test_check_queries_sequence_matches_golden():
    from gsa_b200 import QuerySession

    rows = sequence.run(lambda t: QuerySession(threshold=t), "cuda")
    for g, w in zip(rows, GOLDEN["records"]):
        assert (g["op"], g["label"], g["n"], g["q"]) == (w["op"], w["label"], w["n"], w["q"])
        assert g["stats"] == w["stats"], (g["label"], g["stats"], w["stats"])
        if g["op"] == "ball":
            assert g["ids_sha256"] == w["ids_sha256"], g["label"]
            assert np.array_equal(g["ids"], orc.ball_oracle(g["qv"], g["x"], g["r"], g["k"]))
        else:
            ed, ei = orc.nn_oracle(g["qv"], g["x"])
            assert np.array_equal(g["d"], ed) and np.array_equal(g["ids"], ei), g["label"]


def _graph(ops):
    def graph(inputs):
        root = inputs["pos"]
        sampled = root[:, :1024].contiguous()
        outputs = []
        for support, queries, k in [
            (root, sampled, 16),
            (sampled, sampled, 32),
            (sampled, sampled[:, :256], 8),
            (sampled[:, :256], sampled[:, :64], 16),
        ]:
            result = torch.zeros(1, queries.shape[1], k, device="cuda", dtype=torch.int32)
            ops.ball_query_wrapper(1, support.shape[1], queries.shape[1], 0.5, k, queries, support, result)
            outputs.append(result)
        for support in [sampled, sampled[:, :256], sampled[:, :64]]:
            q = root[:, :79]
            distance = torch.empty(1, 79, 3, device="cuda")
            ids = torch.empty(1, 79, 3, device="cuda", dtype=torch.int32)
            ops.three_nn_wrapper(1, 79, support.shape[1], q, support, distance, ids)
            outputs.extend([distance, ids])
        return outputs

    return graph


def test_fixed_graph_integration():
    from gsa_b200 import QuerySession, fixed_graph_forward
    from gsa_b200 import reference as ops

    torch.manual_seed(123)
    data = {"pos": torch.randn(1, 4096, 3, device="cuda")}
    graph = _graph(ops)
    with torch.inference_mode():
        expected = graph(data)
        original = ops.ball_query_wrapper, ops.three_nn_wrapper
        for policy in ["prefix", "scale"]:
            for verify in [True, False]:
                stats = {}
                actual = fixed_graph_forward(graph, data, ops=ops, policy=policy, threshold=32, verify=verify, stats=stats)
                assert all(torch.equal(a, b) for a, b in zip(actual, expected))
                assert stats["ball_hits"] == 1 and stats["fallbacks"] == 0
                assert stats["builds"] == (2 if policy == "prefix" else 4)
                assert (ops.ball_query_wrapper, ops.three_nn_wrapper) == original
        # oracle check of the unpatched operators themselves
        root = data["pos"][0].cpu().numpy()
        assert np.array_equal(expected[0][0].cpu().numpy(), orc.ball_scan_untouched(root[:1024], root, 0.5, 16, np.zeros((1024, 16), np.int32)))

        def raising(inputs):
            graph(inputs)
            raise RuntimeError("test cleanup")

        with pytest.raises(RuntimeError, match="test cleanup"):
            fixed_graph_forward(raising, data, ops=ops, threshold=32)
        assert (ops.ball_query_wrapper, ops.three_nn_wrapper) == original

        x = data["pos"][0]
        q = x[:8]
        with QuerySession() as session:
            invalid = [
                lambda: session.ball_into(q, x, 0.5, 8, torch.empty(8, 8, device="cuda")),
                lambda: session.nn_into(q, x, torch.empty(8, 3, device="cuda", dtype=torch.float64), torch.empty(8, 3, device="cuda", dtype=torch.int32)),
                lambda: session.ball_into(q, x, -0.5, 8, torch.empty(8, 8, device="cuda", dtype=torch.int32)),
                lambda: session.ball_into(q, x, 0.5, 8, torch.empty(8, 16, device="cuda", dtype=torch.int32)[:, ::2]),
                lambda: session.ball_into(q, x, float("nan"), 8, torch.empty(8, 8, device="cuda", dtype=torch.int32)),
                lambda: session.ball_into(q, x, 0.5, 33, torch.empty(8, 33, device="cuda", dtype=torch.int32)),
                lambda: session.nn_into(q, x[:2], torch.empty(8, 3, device="cuda"), torch.empty(8, 3, device="cuda", dtype=torch.int32)),
            ]
            for op in invalid:
                with pytest.raises(ValueError):
                    op()
        torch.cuda.synchronize()


def test_example_query_session():
    from gsa_b200 import QuerySession

    torch.manual_seed(7)
    with torch.inference_mode():
        support = torch.randn(4096, 3, device="cuda")
        queries = support[:256].clone()
        indices = torch.empty(256, 16, dtype=torch.int32, device="cuda")
        smaller = torch.empty(64, 8, dtype=torch.int32, device="cuda")
        distance = torch.empty(64, 3, device="cuda")
        nearest = torch.empty(64, 3, dtype=torch.int32, device="cuda")
        with QuerySession(threshold=32) as session:
            session.ball_into(queries, support, 0.4, 16, indices)
            session.ball_into(queries[:64].clone(), support.clone(), 0.4, 8, smaller)
            session.nn_into(queries[:64], support[:1024], distance, nearest)
            torch.cuda.synchronize()
            assert torch.equal(smaller, indices[:64, :8])
            assert session.stats["ball_hits"] == 1
            assert session.stats["tree_reuses"] == 1
        s = support.cpu().numpy()
        assert np.array_equal(indices.cpu().numpy(), orc.ball_oracle(s[:256], s, 0.4, 16))
        ed, ei = orc.nn_oracle(s[:64], s[:1024])
        assert np.array_equal(distance.cpu().numpy(), ed) and np.array_equal(nearest.cpu().numpy(), ei)


def test_session_rejects_wrong_stream_and_closed_use():
    from gsa_b200 import QuerySession

    x = torch.randn(100, 3, device="cuda")
    s = QuerySession()
    other = torch.cuda.Stream()
    with torch.cuda.stream(other):
        with pytest.raises(ValueError):
            s.ball_into(x[:4], x, 0.5, 4, torch.empty(4, 4, dtype=torch.int32, device="cuda"))
        with pytest.raises(ValueError):
            s.close()
    s.close()
    with pytest.raises(ValueError):
        s.ball_into(x[:4], x, 0.5, 4, torch.empty(4, 4, dtype=torch.int32, device="cuda"))


def test_index_candidate_misses():
    """Through the real session: index lookups whose first candidate's root
    differs by one ulp answer from the matching or newly built index, and
    the statistics count as GSA's."""
    from gsa_b200 import QuerySession
    from tests.index_miss import INDEX_MISS_STATS, index_candidate_misses

    got, want, stats = index_candidate_misses(lambda t: QuerySession(threshold=t), "cuda")
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    for key, value in INDEX_MISS_STATS.items():
        assert stats[key] == value, (key, stats)
