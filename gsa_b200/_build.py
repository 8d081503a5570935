# SPDX-License-Identifier: Apache-2.0
"""Compile the native libraries in-tree for B200 (sm_100a).

``python -m gsa_b200._build`` writes ``gsa_b200/_native/gsa_bvh.so`` and
``gsa_b200/_native/reference_queries.so`` (the two library names GSA's
``gsa/_library.py`` loads), plus three test variants: ``gsa_bvh_walk.so``
answers every support size with the tree walk (the default library scans
small prefixes), ``gsa_bvh_ordered.so`` does so with the per-query walks
(ordered radius, nearest-first 3NN) instead of the packet-frontier kernels
and builds every tree with the multi-launch sort instead of the cluster sort,
``gsa_bvh_stack4.so`` has a 4-entry traversal stack (8-entry frontier)
so that the per-query-walk and exact full-scan fallbacks are exercised, and
``gsa_bvh_cap8.so`` caps every tree's stored nodes at 8 so that the
node-capacity overflow path (exact scans) is exercised; ``gsa_fps_drop.so``
(FPS only) has one grid block that never arrives at the FPS grid barrier,
so the barrier's bounded wait runs out and reports its error flag.  Flags keep GSA's arithmetic contract (``scripts/build.py:25-34``:
``--fmad=false --ftz=false``); the kernels also use explicit round-to-nearest
intrinsics for every distance operation.
"""

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
NATIVE = PKG / "_native"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "--fmad=false",
    "--ftz=false",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-shared",
    "-I" + str(ROOT / "include"),
]

_BVH = [
    "launches.cu", "pool.cu", "build.cu", "query.cu", "reuse.cu", "reuse_static.cu", "fps.cu", "gsa_bvh_abi.cu",
]
_WALK_ONLY = ["-DGSA_RADIUS_SCAN_MAX=0", "-DGSA_KNN_SCAN_MAX=0"]
LIBS = {
    "gsa_bvh": (_BVH, []),
    "reference_queries": (["launches.cu", "reference_queries.cu"], []),
    # test variants: tree walks for every support size (packet frontier;
    # per-query walks); and the frontier with a 4-entry stack
    "gsa_bvh_walk": (_BVH, _WALK_ONLY),
    "gsa_bvh_ordered": (_BVH, _WALK_ONLY + ["-DGSA_RADIUS_FRONTIER=0", "-DGSA_KNN_FRONTIER=0", "-DGSA_CLUSTER_SORT=0"]),
    "gsa_bvh_stack4": (_BVH, ["-DGSA_STACK=4"] + _WALK_ONLY),
    # every tree of more than ~100 points overflows a node capacity of 8, so
    # its queries take the exact scans
    "gsa_bvh_cap8": (_BVH, ["-DGSA_NODE_CAP_LIMIT=8"] + _WALK_ONLY),
    # FPS only: one block of the cooperative grid never arrives at the
    # barrier and the others' waits are short, so the timeout path runs
    "gsa_fps_drop": (["launches.cu", "fps.cu"],
                     ["-DGSA_FPS_DROP_BLOCK=1", "-DGSA_FPS_BARRIER_SPINS=65536"]),
}


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build gsa_b200")
    return path


def _stale(out, sources):
    if not out.exists():
        return True
    t = out.stat().st_mtime
    deps = list(sources) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps) or Path(__file__).stat().st_mtime > t


def build(names=None, force=False, verbose=False, extra=()):
    """Build the named libraries (default: all); returns their paths."""
    NATIVE.mkdir(exist_ok=True)
    out_paths = []
    for name, (files, defs) in LIBS.items():
        if names and name not in names:
            continue
        sources = [CSRC / f for f in files]
        out = NATIVE / (name + ".so")
        out_paths.append(out)
        if not force and not _stale(out, sources):
            continue
        tmp = out.with_suffix(".so.tmp%d" % os.getpid())
        cmd = [nvcc()] + ARCH + FLAGS + list(defs) + list(extra) + [str(s) for s in sources] + ["-o", str(tmp)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, out)
    return out_paths


if __name__ == "__main__":
    force = "--force" in sys.argv
    extra = [a for a in sys.argv[1:] if a.startswith("-X") or a.startswith("--resource-usage")]
    for p in build(force=force, verbose=True, extra=extra):
        print("built", p)
