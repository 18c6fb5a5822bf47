"""CPU oracle for the AdaAttention forward path.

Test infrastructure only: ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` may import this package, and only as the checker or as the
timed CPU baseline. The product path (``adaattn_b200``) never imports it.
"""

from .ada_oracle import *  # noqa: F401,F403
