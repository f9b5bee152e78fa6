"""xb200: B200-native (sm_100a) implementation of the Triton-XDNA example operator set.

Layers:
  * ``libxb200.so`` -- hand-written CUDA kernels behind a C ABI (``include/xb200.h``);
  * ``xb200._lib``  -- ctypes binding generated from that header;
  * ``xb200.ops``   -- tensor-level operators on CUDA tensors;
  * ``xb200.kernels`` -- ``kernel[grid](...)`` launchers with the reference
    examples' signatures and host-copy semantics;
  * ``xb200.benchmark`` -- ``select_b200_backend`` / ``measure``, standing in for
    the reference's examples/benchmark.py.
"""

from ._lib import XbError  # noqa: F401

__all__ = ["XbError"]
