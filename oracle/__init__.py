"""CPU oracle for easy_as_b200 parity tests.  TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline arm
of ``bench.py`` as the checker; never by the ``easy_as_b200`` package.
"""
