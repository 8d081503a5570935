# SPDX-License-Identifier: Apache-2.0
"""CPU: host-side pieces that need no GPU.

* The package and its build module import without touching the native
  libraries, so ``python -m gsa_b200._build`` works in a fresh checkout.
* ``hierarchy.session_outputs`` lays one scene's outputs over one flat
  buffer: every output once, contiguous, with the shapes and types the
  session calls require, and no two outputs sharing a word.
"""

import subprocess
import sys
from pathlib import Path

import torch

from gsa_b200 import hierarchy as hz

ROOT = Path(__file__).resolve().parents[1]


def test_package_and_build_module_import_without_native_libraries():
    code = (
        "import sys\n"
        "import gsa_b200, gsa_b200._build\n"
        "loaded = [m for m in ('gsa_b200.runtime', 'gsa_b200.session', 'gsa_b200.reference') if m in sys.modules]\n"
        "assert not loaded, loaded\n"
    )
    subprocess.run([sys.executable, "-c", code], cwd=ROOT, check=True)


def test_session_outputs_cover_one_flat_buffer():
    sizes = hz.ROOM_SIZES
    flat, out = hz.session_outputs(sizes, "cpu")
    assert flat.dtype == torch.int32 and flat.numel() == hz.session_words(sizes)
    want = {}
    for s in range(4):
        want[f"ball{s}"] = ((sizes[s], hz.K), torch.int32)
        want[f"hit{s}"] = ((sizes[s + 1], hz.K), torch.int32)
        want[f"nnd{s}"] = ((sizes[s], 3), torch.float32)
        want[f"nni{s}"] = ((sizes[s], 3), torch.int32)
    assert set(out) == set(want)
    spans = []
    base = flat.data_ptr()
    for key, t in out.items():
        shape, dtype = want[key]
        assert tuple(t.shape) == shape and t.dtype == dtype and t.is_contiguous(), key
        start = (t.data_ptr() - base) // 4
        spans.append((start, start + t.numel()))
    spans.sort()
    assert spans[0][0] == 0 and spans[-1][1] == flat.numel()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0  # adjacent, no overlap, no gap
    # writes through the views land in the flat buffer (one copy moves all)
    out["nnd0"][5, 1] = 2.5
    out["ball3"][-1, -1] = 7
    assert (flat.view(torch.float32) == 2.5).sum() == 1
    assert (flat == 7).sum() == 1


def test_session_outputs_reuse_a_given_buffer():
    flat = torch.zeros(hz.session_words(), dtype=torch.int32)
    same, out = hz.session_outputs(hz.ROOM_SIZES, "cpu", flat)
    assert same.data_ptr() == flat.data_ptr()
    assert out["ball0"].data_ptr() == flat.data_ptr()


def test_traffic_profile_parses_ncu_csv_and_pins_the_sources(tmp_path):
    """``bench.py --write-traffic-profile``: per kernel, launches in ID order
    are stages 0..2, DRAM bytes per query are read + write over the stage's
    queries, and the profile records the SHA-256 of the sources it was taken
    of, which ``measured_traffic`` then requires."""
    import bench

    head = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
            '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"\n')
    rows = []
    for i, (kern, stage) in enumerate([("radius_frontier_kernel", 0), ("knn3_frontier_kernel", 0),
                                       ("radius_frontier_kernel", 1), ("knn3_frontier_kernel", 1),
                                       ("radius_frontier_kernel", 2), ("knn3_frontier_kernel", 2)]):
        name = f"void <unnamed>::{kern}<128>(<unnamed>::QArgs)"
        q = bench.SCENES * bench.SIZES[stage]
        for metric, unit, val in [("dram__bytes_read.sum", "byte", 100 * q), ("dram__bytes_write.sum", "byte", 40 * q),
                                  ("gpu__time_duration.sum", "nsecond", 1000 + i), ("smsp__inst_executed.sum", "inst", 250 * q)]:
            rows.append(f'"{i}","1","python","h","{name}","1","7","(64, 1, 1)","(375, 64, 1)","0","10.0",'
                        f'"Command line profiler metrics","{metric}","{unit}","{val:,}"\n')
    csv_path = tmp_path / "dram.csv"
    csv_path.write_text("==PROF== Connected\n" + head + "".join(rows))
    out = tmp_path / "profile.json"
    prof = bench.write_traffic_profile(str(csv_path), out)
    assert sorted(prof["kernels"]) == ["knn3_frontier_kernel", "radius_frontier_kernel"]
    for entry in prof["kernels"].values():
        assert abs(entry["dram_bytes_per_query"] - 140.0) < 1e-9
        assert [s["stage"] for s in entry["per_stage"]] == [0, 1, 2]
        assert all(abs(s["warp_inst_per_32_queries"] - 8000.0) < 1e-9 for s in entry["per_stage"])
    assert prof["sources_sha256"] == bench.kernel_sources_sha(bench.TRAFFIC_SOURCES)
