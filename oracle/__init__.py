"""CPU oracle for the decode hot path -- TEST INFRASTRUCTURE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this package, and only as the checker (or the timed CPU baseline).  The
product package ``nurostream_b200`` never imports it and has no CPU fallback.
"""
