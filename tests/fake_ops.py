# SPDX-License-Identifier: Apache-2.0
"""CPU stand-ins for the session's device operations, backed by the oracle.

Used only by CPU tests of the session's host logic (admission, candidate
ordering, statistics replay).  Every device result comes from
``oracle.numpy_oracle``; comparisons use ``torch.equal`` one pair at a time,
exactly like the reference session.
"""

import numpy as np
import torch

from gsa_b200.session import QuerySession
from oracle import numpy_oracle as orc


class OracleTree:
    def __init__(self, root):
        self.x = root
        self.fallback = torch.zeros(1, dtype=torch.int32)

    def ball(self, q, m, r, ns, out):
        out.copy_(torch.from_numpy(orc.ball_oracle(q.numpy(), self.x[:m].numpy(), r, ns)))

    def query(self, q, m, d, ids):
        ed, ei = orc.nn_oracle(q.numpy(), self.x[:m].numpy())
        d.copy_(torch.from_numpy(ed))
        ids.copy_(torch.from_numpy(ei))

    def close(self):
        pass


def _ball_scan(b, n, m, r, k, q, x, out):
    for i in range(b):
        res = orc.ball_scan_untouched(q[i].numpy(), x[i].numpy(), r, k, out[i].numpy())
        out[i].copy_(torch.from_numpy(res))


def _nn_scan(b, n, m, q, x, d, ids):
    for i in range(b):
        ed, ei = orc.nn_oracle(q[i].numpy(), x[i].numpy())
        d[i].copy_(torch.from_numpy(ed))
        ids[i].copy_(torch.from_numpy(ei))


class OracleOps:
    comparisons = 0

    @staticmethod
    def current():
        return 0, 0

    @staticmethod
    def on_device(x, device):
        return not x.is_cuda

    def lookup(self, pairs, cached, rows, cols, out, device):
        flags = [0 if torch.equal(a, b[: a.shape[0]]) else 1 for a, b in pairs]
        for c, rows_c in enumerate(cached):
            if not (flags[2 * c] or flags[2 * c + 1]):
                out.copy_(rows_c[:rows, :cols])
                break
        return flags

    def mismatch(self, pairs, device):
        return torch.tensor([0 if torch.equal(a, b) else 1 for a, b in pairs], dtype=torch.int32)

    def reuse(self, cached, flags, rows, cols, out):
        f = flags.tolist()
        for c, rows_c in enumerate(cached):
            if not (f[2 * c] or f[2 * c + 1]):
                out.copy_(rows_c[:rows, :cols])
                return

    @staticmethod
    def fetch(flags):
        return flags.tolist()

    @staticmethod
    def copy_cols(out, result, k):
        out.copy_(result[: out.shape[0], :k])

    @staticmethod
    def scan_ball(n, nq, r, cap, q, x, out):
        _ball_scan(1, n, nq, r, cap, q[None], x[None], out[None])

    @staticmethod
    def scan_nn(nq, n, q, x, d, ids):
        _nn_scan(1, nq, n, q[None], x[None], d[None], ids[None])

    @staticmethod
    def tree_ball(tree, q, x, m, r, cap, out):
        tree.ball(q, m, r, cap, out)

    @staticmethod
    def tree_query(tree, q, x, m, d, ids):
        tree.query(q, m, d, ids)

    @staticmethod
    def zeros(rows, device):
        return torch.zeros((rows, 32), dtype=torch.int32)

    @staticmethod
    def rows(rows, device):
        # not zero-filled, like the device session's tree result rows: the
        # tree query must write every row
        return torch.full((rows, 32), -7, dtype=torch.int32)

    @staticmethod
    def snapshot(x):
        return x.clone()

    @staticmethod
    def tree(root):
        return OracleTree(root)

    @staticmethod
    def collect(tree):
        return int(tree.fallback.item())

    default_ball = staticmethod(_ball_scan)
    default_nn = staticmethod(_nn_scan)


class OracleSession(QuerySession):
    _ops_class = OracleOps


def make_oracle_session(threshold):
    return OracleSession(threshold=threshold)
