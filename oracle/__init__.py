"""CPU oracle for the MoE hot path -- test infrastructure, never product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package.
"""
