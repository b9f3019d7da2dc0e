"""CPU oracle of the dendritic tick -- TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg, as the checker or the timed CPU baseline; the product package
never imports it.  See ``tick.py`` (C restatement loaded through ctypes, plus
numpy restatements of the weight formats).
"""

from .tick import *  # noqa: F401,F403
from .tick import CSR, build_oracle, max_threads  # noqa: F401
