"""CPU checker for the block-sparse prefill attention path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package. The product
(``exp3_b200``) never imports it: its ops fail loudly when the CUDA library is
missing instead of falling back to a CPU path.
"""

from .attention_oracle import *  # noqa: F401,F403
