"""CPU oracle for the HERM forward hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the host and in plain torch/numpy, the algorithms of
the Koemi-5HOM reference that the B200 kernels implement. Each function cites
the reference file:line it follows. It is pinned against golden fixtures
generated from the reference itself (tests/golden/make_golden.py).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline. The product path (``koemi_5hom_b200``)
never imports it and has no CPU fallback.
"""
