"""CPU oracle for the Mamba TP hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu-baseline
leg may import this package, and only as the checker / the timed CPU
baseline.  The product (``mamba_tp_lite_b200``) never imports it and has no
CPU fallback.
"""
