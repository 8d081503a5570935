# SPDX-License-Identifier: Apache-2.0
"""Replays the reference's 94-call query/state sequence.

The call sequence, inputs and RNG draw order follow GSA
``tests/check_queries.py:84-151`` (seed 20261111): three supports of 17, 257
and 4099 N(0,1) points with a duplicated point, clone/prefix reuse, caller
output edits, zero and changed radii, 3NN at several prefixes, in-place
support/query updates, a support permutation, a return to the original
values, empty queries, an ID-changing sequence and an FP32 scale sweep.

``run(session_factory, device)`` executes it against any session object with
the ``QuerySession`` API and returns one record per call with the output,
its SHA-256 (radius calls), the session statistics and the inputs used.
"""

import hashlib

import numpy as np
import torch

SEED = 20261111


def run(make_session, device):
    rng = np.random.default_rng(SEED)
    rows = []

    def ball(s, x, q, r, k, label):
        out = torch.empty((len(q), k), device=device, dtype=torch.int32)
        s.ball_into(q, x, r, k, out)
        a = out.cpu().numpy()
        rows.append(
            {
                "op": "ball",
                "label": label,
                "n": len(x),
                "q": len(q),
                "r": r,
                "k": k,
                "ids": a,
                "ids_sha256": hashlib.sha256(a.tobytes()).hexdigest(),
                "stats": dict(s.stats),
                "x": x.cpu().numpy().copy(),
                "qv": q.cpu().numpy().copy(),
            }
        )
        return out

    def nn(s, x, q, label):
        d = torch.empty((len(q), 3), device=device, dtype=torch.float32)
        ids = torch.empty((len(q), 3), device=device, dtype=torch.int32)
        s.nn_into(q, x, d, ids)
        rows.append(
            {
                "op": "nn",
                "label": label,
                "n": len(x),
                "q": len(q),
                "d": d.cpu().numpy(),
                "ids": ids.cpu().numpy(),
                "stats": dict(s.stats),
                "x": x.cpu().numpy().copy(),
                "qv": q.cpu().numpy().copy(),
            }
        )

    with torch.inference_mode():
        for n in [17, 257, 4099]:
            original = rng.normal(size=(n, 3)).astype(np.float32)
            original[1] = original[0]
            x = torch.from_numpy(original.copy()).to(device)
            q = x[:13].clone()
            s = make_session(32)
            first = ball(s, x, q, 1.0, 8, "initial")
            hits = s.stats["ball_hits"]
            ball(s, x.clone(), q[:7].clone(), 1.0, 1, "value_equal_clones_and_query_prefix")
            assert s.stats["ball_hits"] == hits + 1
            first.fill_(-123)
            hits = s.stats["ball_hits"]
            ball(s, x, q, 1.0, 32, "private_cached_rows_after_caller_output_edit")
            assert s.stats["ball_hits"] == hits + 1
            ball(s, x, q, 0.0, 32, "strict_zero_radius")
            ball(s, x, q, 4.0, 8, "changed_radius")
            for m in [n, max(3, n // 4), max(3, n // 16), max(3, n - 3)]:
                nn(s, x[:m].contiguous(), q, "prefix_and_independent_support")
            x.add_(0.37)
            ball(s, x, q, 1.0, 8, "inplace_support_update")
            nn(s, x, q, "nn_after_support_update")
            x.copy_(x.flip(0))
            ball(s, x, q, 1.0, 8, "support_permutation")
            nn(s, x, q, "nn_after_permutation")
            q.add_(0.19)
            ball(s, x, q, 1.0, 8, "inplace_query_update")
            old = torch.from_numpy(original.copy()).to(device)
            ball(s, old, old[:13].clone(), 1.0, 8, "return_to_original_coordinate_values")
            ball(s, old, old[:0], 1.0, 8, "empty_query")
            nn(s, old, old[:0], "empty_nn_query")
            s.close(collect=True)
            assert s.stats["fallbacks"] == 0
        x = torch.tensor([[0.0, 0.0, 0.0], [2.0, 0.0, 0.0], [3.0, 0.0, 0.0]], device=device)
        q = torch.zeros((1, 3), device=device)
        s = make_session(32)
        assert ball(s, x, q, 0.1, 1, "id_change_start").item() == 0
        x.copy_(x[[1, 0, 2]])
        assert ball(s, x, q, 0.1, 1, "id_change_after_permutation").item() == 1
        x[1, 0] = 3.0
        x[2, 0] = 0.0
        assert ball(s, x, q, 0.1, 1, "id_change_after_inplace_mutation").item() == 2
        s.close()
        for scale in [0.0, 1e-25, 1.0, 1e20]:
            a = (rng.normal(size=(97, 3)) * scale).astype(np.float32)
            x = torch.from_numpy(a).to(device)
            q = x[:9].clone()
            s = make_session(32)
            for r in [
                0.0,
                float(np.float32(scale)),
                float(np.nextafter(np.float32(scale), np.float32(np.inf))),
            ]:
                for k in [1, 8, 32]:
                    ball(s, x, q, r, k, "scale_radius_K_contract")
            nn(s, x, q, "scaled_nn")
            s.close(collect=True)
            assert s.stats["fallbacks"] == 0
    assert len(rows) == 94
    return rows
