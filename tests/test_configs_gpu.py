# SPDX-License-Identifier: Apache-2.0
"""GPU parity on the five benchmark workloads (seeded synthetic stand-ins).

* unit case: 4096 N(0,1) points, radius 0.4 K16 for the first 128, 3NN of
  all points against the first 1024, at threshold 1024 (scan 3NN) and 32;
* room hierarchy: 24,000-point FPS-ordered room, prefixes
  24000/6000/1500/375/94, r = 0.1/0.2/0.4/0.8, K = 32, reuse enabled --
  every output equals the oracle, statistics as the reference would count;
* batched scenes: ``hierarchy.Batch`` over many rooms equals the per-scene
  ``QuerySession`` run bit for bit (oracle-checked on a sample of scenes);
* exactness stress: 200,000 clustered points (sigma 1e-3, 20 % duplicates,
  5 % points at exactly f32(0.25)^2 from a query), radius and 3NN on oracle
  samples, then a 1-ulp support change must miss the reuse cache and
  recompute correctly.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import numpy_oracle as orc

pytestmark = pytest.mark.gpu


def test_unit_case():
    from gsa_b200 import QuerySession, scenes

    x_np = scenes.unit_case()
    x = torch.from_numpy(x_np).cuda()
    for threshold in [1024, 32]:
        with QuerySession(threshold=threshold) as s:
            out = torch.empty((128, 16), dtype=torch.int32, device="cuda")
            s.ball_into(x[:128], x, 0.4, 16, out)
            d = torch.empty((4096, 3), device="cuda")
            i = torch.empty((4096, 3), dtype=torch.int32, device="cuda")
            s.nn_into(x, x[:1024], d, i)
            assert np.array_equal(out.cpu().numpy(), orc.ball_oracle(x_np[:128], x_np, 0.4, 16))
            ed, ei = orc.nn_oracle_fast(x_np, x_np[:1024])
            assert np.array_equal(d.cpu().numpy(), ed) and np.array_equal(i.cpu().numpy(), ei)
            assert s.stats["builds"] == 1 and s.stats["tree_reuses"] == (1 if threshold == 32 else 0)


def _room(seeds):
    from gsa_b200 import scenes

    return scenes.room_batch(seeds)


def _check_hierarchy_against_oracle(P_np, out, sizes, radii):
    for s in range(4):
        ps = P_np[: sizes[s]]
        want = orc.ball_oracle_fast(ps, ps, radii[s], 32)
        assert np.array_equal(out[f"ball{s}"].cpu().numpy(), want), s
        assert np.array_equal(out[f"hit{s}"].cpu().numpy(), want[: sizes[s + 1]]), s
        ed, ei = orc.nn_oracle_fast(ps, P_np[: sizes[s + 1]])
        assert np.array_equal(out[f"nnd{s}"].cpu().numpy(), ed), s
        assert np.array_equal(out[f"nni{s}"].cpu().numpy(), ei), s


def test_room_hierarchy_session():
    from gsa_b200 import QuerySession, hierarchy as hz

    P = _room([0])[0]
    with QuerySession() as s:
        out = hz.run_session(s, P)
        torch.cuda.synchronize()
        st = dict(s.stats)
    _check_hierarchy_against_oracle(P.cpu().numpy(), out, hz.ROOM_SIZES, hz.ROOM_RADII)
    # one prefix tree serves supports 24000/6000/1500 (radius stages 1-2 and
    # the 3NN supports 6000/1500 reuse it); 375 and 94 take the scan
    assert st["builds"] == 1 and st["ball_hits"] == 4 and st["ball_calls"] == 8
    assert st["nn_calls"] == 4 and st["tree_reuses"] == 4
    assert st["fallbacks"] == 0


def test_batch_equals_session_per_scene():
    from gsa_b200 import QuerySession, hierarchy as hz

    seeds = list(range(16))
    X = _room(seeds)
    eng = hz.Batch()
    out = eng.run(X)
    assert out["hits"].sum().item() == 4 * len(seeds)
    serial = eng.run(X, eng.allocate(len(seeds), X.device), concurrent=False)
    for key in out:
        if key.startswith(("ball", "hit", "nn")):
            assert torch.equal(out[key], serial[key]), key
    torch.cuda.synchronize()
    for b in range(len(seeds)):
        with QuerySession() as s:
            ref = hz.run_session(s, X[b])
        for key, t in ref.items():
            rows = t.shape[0]
            got = out[key][b * rows:(b + 1) * rows]
            assert torch.equal(got, t), (b, key)
    _check_hierarchy_against_oracle(X[3].cpu().numpy(), {k: v[3 * v.shape[0] // 16:4 * v.shape[0] // 16] for k, v in out.items() if k.startswith(("ball", "hit", "nn"))}, hz.ROOM_SIZES, hz.ROOM_RADII)


def test_large_scene_hierarchy():
    """1,000,000-point room in a 20x20x3 m box, FPS-ordered, prefixes
    1M/250k/62.5k/15.6k(/3.9k), r = 0.05/0.1/0.2/0.4, K = 32: the session and
    the batched engine agree on every row, oracle samples of every stage
    match, reuse rows are prefixes of the self rows."""
    from gsa_b200 import QuerySession, hierarchy as hz, scenes

    sizes, radii = hz.LARGE_SIZES, hz.LARGE_RADII
    P = scenes.room_batch([11], n=sizes[0], box=(20.0, 20.0, 3.0))
    with QuerySession() as s:
        out = hz.run_session(s, P[0], sizes, radii)
        st = dict(s.stats)
    # the 3,906-point support of the last decoder stage is not one of the
    # root's prefix sizes (1M, 250k, 62.5k, 15.6k), so it gets its own tree
    assert st["builds"] == 2 and st["ball_hits"] == 4 and st["tree_reuses"] == 6
    batch = hz.Batch(sizes, radii).run(P)
    torch.cuda.synchronize()
    for key, t in out.items():
        assert torch.equal(batch[key], t), key
    Pn = P[0].cpu().numpy()
    rng = np.random.default_rng(3)
    for s_ in range(4):
        n_s = sizes[s_]
        rows = out[f"ball{s_}"].cpu().numpy()
        assert np.array_equal(out[f"hit{s_}"].cpu().numpy(), rows[: sizes[s_ + 1]])
        pick = np.unique(np.concatenate([rng.choice(n_s, 200, replace=False), [0, n_s - 1]]))
        want = orc.ball_oracle_fast(Pn[pick], Pn[:n_s], radii[s_], 32)
        assert np.array_equal(rows[pick], want), s_
        ed, ei = orc.nn_oracle_fast(Pn[pick], Pn[: sizes[s_ + 1]])
        assert np.array_equal(out[f"nnd{s_}"].cpu().numpy()[pick], ed), s_
        assert np.array_equal(out[f"nni{s_}"].cpu().numpy()[pick], ei), s_


def test_batched_reuse_admission_rejects_changed_scene():
    from tests import abi

    lib = abi.bvh_lib()
    B, N, n_q = 4, 1000, 250
    X = torch.randn(B, N, 3, device="cuda")
    snap = X.clone()
    snap[2, 700, 1] += 1e-3  # support differs beyond the query prefix
    snap[3, 10, 0] = float("nan")  # NaN never compares equal
    flags = torch.full((2 * B,), 7, dtype=torch.int32, device="cuda")
    st = abi.stream()
    assert lib.coords_mismatch_strided(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, N * 3, flags.data_ptr(), 2, st) == 0
    assert lib.coords_mismatch_strided(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, n_q * 3, flags.data_ptr() + 4, 2, st) == 0
    assert flags.tolist() == [0, 0, 0, 0, 1, 0, 1, 1]
    rows = torch.randint(0, 999, (B * N, 32), dtype=torch.int32, device="cuda")
    dst = torch.full((B * n_q, 32), -1, dtype=torch.int32, device="cuda")
    hits = torch.full((B,), 9, dtype=torch.int32, device="cuda")
    assert lib.reuse_rows_batch(B, rows.data_ptr(), N * 32, 32, flags.data_ptr(), n_q, 32, dst.data_ptr(), n_q * 32, hits.data_ptr(), st) == 0
    assert hits.tolist() == [1, 1, 0, 0]
    for b in range(B):
        got = dst[b * n_q:(b + 1) * n_q]
        if b < 2:
            assert torch.equal(got, rows[b * N:b * N + n_q])
        else:
            assert (got == -1).all()


@pytest.mark.parametrize("N,n_q,shift,B", [(1000, 250, 0, 6), (24000, 6000, 0, 6), (24000, 6000, 0, 24),
                                           (1001, 333, 1, 6), (94, 23, 0, 6), (7, 7, 1, 6)])
def test_fused_stage_reuse_equals_two_step_path(N, n_q, shift, B):
    """reuse_prefix_batch against coords_mismatch_strided twice +
    reuse_rows_batch: same flags, hits and rows; rows of a miss stay
    untouched.  Six 24,000-point scenes take its grid-wide form (their
    clusters would not cover the SMs), 24 take one 8-CTA cluster per scene,
    small scenes smaller clusters.  shift=1 offsets every buffer by one
    element (scalar path)."""
    from tests import abi

    lib = abi.bvh_lib()
    K = 32
    g = torch.Generator(device="cpu").manual_seed(N + n_q)
    X = torch.randn(B * N * 3 + shift, generator=g).cuda()[shift:].view(B, N, 3)
    snap = torch.empty(B * N * 3 + shift, device="cuda")[shift:].view(B, N, 3)
    snap.copy_(X)
    if N > n_q:
        snap[1, N - 1, 2] += 1e-3  # support differs beyond the query prefix
    snap[2, n_q - 1, 2] = torch.nextafter(snap[2, n_q - 1, 2], torch.tensor(float("inf"), device="cuda"))  # last query element
    snap[3, 0, 0] = float("nan")  # NaN never compares equal
    X[4, 0, 1] = 0.0
    snap[4, 0, 1] = -0.0  # -0 == +0: still a hit
    X[5, n_q // 2, 0] = float("nan")
    snap[5, n_q // 2, 0] = float("nan")
    st = abi.stream()
    want_flags = torch.full((2 * B,), 7, dtype=torch.int32, device="cuda")
    assert lib.coords_mismatch_strided(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, N * 3, want_flags.data_ptr(), 2, st) == 0
    assert lib.coords_mismatch_strided(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, n_q * 3, want_flags.data_ptr() + 4, 2, st) == 0
    rows = torch.randint(0, 999, (B * N * K + shift,), dtype=torch.int32, device="cuda")[shift:].view(B * N, K)
    want = torch.full((B * n_q * K + shift,), -1, dtype=torch.int32, device="cuda")[shift:].view(B * n_q, K)
    got = want.clone()
    want_hits = torch.full((B,), 9, dtype=torch.int32, device="cuda")
    assert lib.reuse_rows_batch(B, rows.data_ptr(), N * K, K, want_flags.data_ptr(), n_q, K, want.data_ptr(), n_q * K, want_hits.data_ptr(), st) == 0
    flags = torch.full((2 * B,), 7, dtype=torch.int32, device="cuda")
    hits = torch.full((B,), 9, dtype=torch.int32, device="cuda")
    for _ in range(2):  # flags and hits are written whole on every call
        assert lib.reuse_prefix_batch(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, N * 3, n_q * 3,
                                      rows.data_ptr(), N * K, K, n_q, K, got.data_ptr(), n_q * K,
                                      flags.data_ptr(), hits.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert flags.tolist() == want_flags.tolist()
        assert hits.tolist() == want_hits.tolist()
        assert torch.equal(got, want)
    expect_hits = [1, 0 if N > n_q else 1, 0, 0, 1, 0] + [1] * (B - 6)
    assert hits.tolist() == expect_hits
    assert lib.reuse_prefix_batch(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, n_q * 3, N * 3,
                                  rows.data_ptr(), N * K, K, n_q, K, got.data_ptr(), n_q * K,
                                  flags.data_ptr(), hits.data_ptr(), st) == (-2 if N > n_q else 0)


@pytest.mark.parametrize("N,B", [(24000, 64), (24000, 4), (1001, 5)])
def test_all_stage_reuse_equals_per_stage_calls(N, B):
    """reuse_prefix_stages (the four hierarchy stages in one launch) against
    reuse_prefix_batch per stage: same flags, hits and rows, with scenes whose
    support differs at some stages only.  Four 24,000-point
    scenes take the per-stage grid-wide form."""
    from tests import abi

    lib = abi.bvh_lib()
    K = 32
    sizes = [N, N // 4, N // 16, N // 64, max(1, N // 256)]
    g = torch.Generator(device="cpu").manual_seed(N + B)
    X = torch.randn(B, N, 3, generator=g).cuda()
    snap = X.clone()
    snap[1, sizes[1] + 3, 0] += 1.0    # stage 0 support differs only
    snap[2, sizes[3], 2] = float("nan")  # supports of stages 0-2 only
    snap[B - 1, 0, 1] = -snap[B - 1, 0, 1] if snap[B - 1, 0, 1] != 0 else 1.0  # every stage
    rows = [torch.randint(0, 1 << 20, (B * sizes[s], K), dtype=torch.int32, device="cuda") for s in range(4)]
    st = abi.stream()
    want, got = [], []
    for s in range(4):
        n_s, n_q = sizes[s], sizes[s + 1]
        w = {"rows": torch.full((B * n_q, K), -1, dtype=torch.int32, device="cuda"),
             "flags": torch.full((2 * B,), 7, dtype=torch.int32, device="cuda"),
             "hits": torch.full((B,), 9, dtype=torch.int32, device="cuda")}
        assert lib.reuse_prefix_batch(B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3, n_s * 3, n_q * 3,
                                      rows[s].data_ptr(), n_s * K, K, n_q, K, w["rows"].data_ptr(), n_q * K,
                                      w["flags"].data_ptr(), w["hits"].data_ptr(), st) == 0
        want.append(w)
        got.append({k: torch.full_like(v, -1 if k == "rows" else 5) for k, v in w.items()})
    LLa, Pa, Ia = ctypes.c_longlong * 4, ctypes.c_void_p * 4, ctypes.c_int * 4
    for _ in range(2):  # flags and hits are written whole on every call
        code = lib.reuse_prefix_stages(
            4, B, X.data_ptr(), N * 3, snap.data_ptr(), N * 3,
            LLa(*[sizes[s] * 3 for s in range(4)]), LLa(*[sizes[s + 1] * 3 for s in range(4)]),
            Pa(*[rows[s].data_ptr() for s in range(4)]), LLa(*[sizes[s] * K for s in range(4)]), K,
            Ia(*[sizes[s + 1] for s in range(4)]), K, Pa(*[got[s]["rows"].data_ptr() for s in range(4)]),
            LLa(*[sizes[s + 1] * K for s in range(4)]), Pa(*[got[s]["flags"].data_ptr() for s in range(4)]),
            Pa(*[got[s]["hits"].data_ptr() for s in range(4)]), st)
        assert code == 0
        torch.cuda.synchronize()
        for s in range(4):
            for k in ("flags", "hits", "rows"):
                assert torch.equal(got[s][k], want[s][k]), (s, k)
    assert [h.item() for h in want[0]["hits"][:3]] == [1, 0, 0]
    assert want[3]["hits"][2].item() == 1 and want[2]["hits"][2].item() == 0
    assert all(w["hits"][B - 1].item() == 0 for w in want)


def test_clustered_exactness_stress():
    from gsa_b200 import QuerySession, scenes

    pts, info = scenes.clustered(seed=0)
    assert info["exact_points"] >= 9000
    r2 = np.float32(0.25) * np.float32(0.25)
    for pid, qi in info["anchors"][:200]:
        d = pts[qi] - pts[pid]
        sq = d * d
        assert (sq[0] + sq[1]) + sq[2] == r2
    x = torch.from_numpy(pts).cuda()
    nq = info["queries"]
    rng = np.random.default_rng(1)
    anchor_q = np.array(sorted({qi for _, qi in info["anchors"]}))
    sample = np.unique(np.concatenate([rng.choice(nq, 1500, replace=False), anchor_q[:500]]))
    with QuerySession() as s:
        out = torch.empty((nq, 32), dtype=torch.int32, device="cuda")
        s.ball_into(x[:nq], x, 0.25, 32, out)
        d = torch.empty((len(pts), 3), device="cuda")
        ids = torch.empty((len(pts), 3), dtype=torch.int32, device="cuda")
        s.nn_into(x, x[:nq], d, ids)
        got = out.cpu().numpy()
        assert np.array_equal(got[sample], orc.ball_oracle_fast(pts[sample], pts, 0.25, 32))
        nn_sample = np.unique(np.concatenate([rng.choice(len(pts), 2000, replace=False), np.arange(0, 200)]))
        ed, ei = orc.nn_oracle_fast(pts[nn_sample], pts[:nq])
        assert np.array_equal(d.cpu().numpy()[nn_sample], ed) and np.array_equal(ids.cpu().numpy()[nn_sample], ei)
        # exact-r points: strict qualification on a support of anchors only
        anchors = np.array(info["anchors"][:2000])
        sub = np.concatenate([pts[anchors[:, 1]], pts[anchors[:, 0]]])
        xs = torch.from_numpy(sub).cuda()
        o2 = torch.empty((len(anchors), 32), dtype=torch.int32, device="cuda")
        s.ball_into(xs[: len(anchors)], xs, 0.25, 32, o2)
        assert np.array_equal(o2.cpu().numpy(), orc.ball_oracle_fast(sub[: len(anchors)], sub, 0.25, 32))
        # 1-ulp change of one support coordinate: reuse miss and exact recompute
        hits, builds = s.stats["ball_hits"], s.stats["builds"]
        j = int(anchors[0, 0])
        x2 = x.clone()
        x2[j, 0] = torch.nextafter(x2[j, 0], torch.tensor(np.inf, device="cuda"))
        out2 = torch.empty((nq, 32), dtype=torch.int32, device="cuda")
        s.ball_into(x2[:nq], x2, 0.25, 32, out2)
        assert s.stats["ball_hits"] == hits and s.stats["builds"] == builds + 1
        p2 = x2.cpu().numpy()
        sample2 = np.unique(np.concatenate([sample[:300], [int(anchors[0, 1])]]))
        assert np.array_equal(out2.cpu().numpy()[sample2], orc.ball_oracle_fast(p2[sample2], p2, 0.25, 32))
        # the unchanged values still hit
        out3 = torch.empty((nq // 2, 8), dtype=torch.int32, device="cuda")
        s.ball_into(x[: nq // 2].clone(), x.clone(), 0.25, 8, out3)
        assert s.stats["ball_hits"] == hits + 1
        assert torch.equal(out3, out[: nq // 2, :8])
        s.close(collect=True)
        assert s.stats["fallbacks"] == 0
