"""CPU oracle for the MEDUSA tree-verify hot path.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` as the
checker.  The product package never imports it.
"""
