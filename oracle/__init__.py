"""CPU oracle for the gated block-sparse attention path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import this package, and only as the checker or
the timed CPU baseline. The product package ``tasft_b200`` never imports it.
"""
from oracle.tasft_oracle import *  # noqa: F401,F403
