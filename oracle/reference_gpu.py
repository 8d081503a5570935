# SPDX-License-Identifier: Apache-2.0
"""The reference's own GPU path, unmodified, as a checker and a timing bar.

TEST AND BASELINE INFRASTRUCTURE, not product code.  ``oracle/Makefile``
(``make -C oracle install``) installs the reference's Python package
(qmkkk/GSA ``gsa/``: ``QuerySession``, ``Tree``, ``fixed_graph``) into
``baseline/_ref`` with pip and places beside it the reference's
``csrc/gsa_bvh.cu`` and ``csrc/reference_queries.cu`` built from source for
sm_100a (``gsa/_native/*.so``, the layout the reference's
``scripts/build.py`` writes).  ``load()`` imports that package, so a GPU test
can run the very call sequence a reference user runs
(``gsa.QuerySession.ball_into`` / ``nn_into``, ``gsa/session.py:83-151``)
and compare every output row with this repository's, and the reference arm
of ``bench.py`` can time it on the same box.
"""

import importlib
import sys
from pathlib import Path

BASE = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def available():
    """Why the reference package cannot be loaded, or None when it can."""
    if not (BASE / "gsa" / "__init__.py").is_file():
        return "reference package not installed (make -C oracle install)"
    for name in ("gsa_bvh", "reference_queries"):
        if not (BASE / "gsa" / "_native" / (name + ".so")).is_file():
            return f"reference library {name}.so not built (make -C oracle install)"
    return None


def load():
    """Import and return the reference's ``gsa`` package (raises
    RuntimeError with the reason when it is not installed)."""
    why = available()
    if why:
        raise RuntimeError(why)
    if str(BASE) not in sys.path:
        sys.path.insert(0, str(BASE))
    gsa = importlib.import_module("gsa")
    if Path(gsa.__file__).resolve().parent != (BASE / "gsa").resolve():
        raise RuntimeError(f"a different 'gsa' package is importable: {gsa.__file__}")
    return gsa
