"""CPU oracle for the Pearl mining hot path.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` as the
checker.  The product package ``pearl_b200`` never imports it.
"""

from .oracle import *  # noqa: F401,F403
