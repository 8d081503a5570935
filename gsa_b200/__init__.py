# SPDX-License-Identifier: Apache-2.0
"""B200-native exact point queries with geometry-state reuse.

Drop-in for GSA's Python API (``gsa/__init__.py:4-6``): ``QuerySession``,
``Tree``, ``pool_memory`` and ``fixed_graph_forward``, backed by hand-written
sm_100a kernels in ``gsa_b200/_native``.  ``Forest`` adds multi-scene batches.

The public names load on first use, so that ``python -m gsa_b200._build``
can compile the libraries in a fresh checkout; using any of them before the
libraries exist raises (there is no CPU fallback).
"""

import importlib

__version__ = "0.1.0"

_EXPORTS = {
    "QuerySession": (".session", "QuerySession"),
    "Tree": (".runtime", "Tree"),
    "pool_memory": (".runtime", "pool_memory"),
    "fixed_graph_forward": (".fixed_graph", "forward"),
    "Forest": (".forest", "Forest"),
}
__all__ = list(_EXPORTS)


def __getattr__(name):
    try:
        module, attr = _EXPORTS[name]
    except KeyError:
        raise AttributeError(f"module 'gsa_b200' has no attribute {name!r}") from None
    value = getattr(importlib.import_module(module, __name__), attr)
    globals()[name] = value
    return value
