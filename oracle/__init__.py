"""Parity oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and the
CPU-baseline legs of ``bench.py``. The shipped library never imports it.
"""
