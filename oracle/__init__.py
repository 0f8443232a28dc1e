"""CPU oracle for the Cherimoya hot path.  TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` as the checker and the CPU baseline; never by the engine.
"""
