"""CPU oracle for the low-bit linear layer (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import this package.  The product path (``apsi_b200``) never imports it.
"""
from .lowbit_oracle import *  # noqa: F401,F403
