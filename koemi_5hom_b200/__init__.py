"""B200-native HERM forward hot path for Koemi-5HOM.

Subpackages:
- ``cuda_kernels``: the four native operator fronts (core, dense, think, moe),
  drop-in for ``koemi.cuda_kernels``;
- ``model``: the HERM block (``KoemiModel``-compatible forward) on those kernels;
- ``runtime``: fixed-shape batched decode with CUDA-graph replay.

Kernels live in ``lib/libkoemi_b200.so`` (built by ``koemi_5hom_b200.build``).
"""

__version__ = "0.1.0"
