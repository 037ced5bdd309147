"""CPU oracle and CPU baseline of the entropy-gated path -- test infrastructure only.

Imported by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py``; never by the engine package.
"""
