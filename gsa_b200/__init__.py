# SPDX-License-Identifier: Apache-2.0
"""B200-native exact point queries with geometry-state reuse.

Drop-in for GSA's Python API (``gsa/__init__.py:4-6``): ``QuerySession``,
``Tree``, ``pool_memory`` and ``fixed_graph_forward``, backed by hand-written
sm_100a kernels in ``gsa_b200/_native``.  ``Forest`` adds multi-scene batches.
"""

from .session import QuerySession
from .runtime import Tree, pool_memory
from .fixed_graph import forward as fixed_graph_forward
from .forest import Forest

__version__ = "0.1.0"
