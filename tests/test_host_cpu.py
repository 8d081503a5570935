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
