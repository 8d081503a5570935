# SPDX-License-Identifier: Apache-2.0
"""Load the in-tree native libraries (mirror of GSA ``gsa/_library.py``).

``load(name)`` opens ``gsa_b200/_native/<name>.so``.  There is no CPU
fallback: a missing library raises immediately.
"""

import ctypes
from pathlib import Path

NATIVE_DIR = Path(__file__).resolve().parent / "_native"
_loaded = {}


def path(name):
    return NATIVE_DIR / (name + ".so")


def load(name):
    """Return the ``ctypes.CDLL`` of ``_native/<name>.so`` (cached)."""
    if name in _loaded:
        return _loaded[name]
    p = path(name)
    if not p.is_file():
        raise RuntimeError(
            "Compile gsa_b200 first: python -m gsa_b200._build "
            "(needs nvcc; builds sm_100a libraries in gsa_b200/_native)"
        )
    lib = ctypes.CDLL(str(p))
    _loaded[name] = lib
    return lib
