"""CPU oracle (test infrastructure only): restatements of the reference's hot path.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` -- never by the ``xanosmerks_b200`` package.
"""
