# SPDX-License-Identifier: Apache-2.0
"""Index lookups whose first candidate has a different root.

When the first index candidate's root differs from the support (here by
one ulp), the answer must come from a later candidate or a newly built
index, and the statistics must count as GSA ``gsa/session.py:65-81``
counts.  Used by a CPU test (oracle-backed session) and a GPU test (the
real session).
"""

import torch

from oracle import numpy_oracle as orc


def index_candidate_misses(make_session, device):
    """Calls whose first index candidate has a different root, so the
    answer must come from a later candidate or a new index.  Returns the
    outputs (numpy) with the oracle's answers and the final statistics."""
    g = torch.Generator().manual_seed(7)
    x1 = torch.rand(512, 3, generator=g)
    x2 = x1.clone()
    x2[100, 1] = torch.nextafter(x2[100, 1], torch.tensor(2.0))
    q = torch.rand(96, 3, generator=g)
    X1, X2, Q = x1.to(device), x2.to(device), q.to(device)
    got, want = [], []
    with make_session(32) as s:
        for sup in (X1, X2, X2):  # build; root differs -> build; reuse 2nd
            d = torch.empty(96, 3, device=device)
            ids = torch.empty(96, 3, dtype=torch.int32, device=device)
            s.nn_into(Q, sup, d, ids)
            got += [d.cpu().numpy(), ids.cpu().numpy()]
            want += list(orc.nn_oracle(q.numpy(), sup.cpu().numpy()))
        out = torch.empty(96, 16, dtype=torch.int32, device=device)
        s.ball_into(Q, X2, 0.2, 16, out)  # no memo entry; first index differs
        got.append(out.cpu().numpy())
        want.append(orc.ball_oracle(q.numpy(), x2.numpy(), 0.2, 16))
        stats = dict(s.stats)
    return got, want, stats


INDEX_MISS_STATS = {"builds": 2, "tree_reuses": 2, "coordinate_comparisons": 5, "nn_calls": 3, "ball_calls": 1}
