"""vkcuda_b200: the hot path of junka/vkcuda's demos (flash-attention forward,
cooperative-matrix GEMM, vadd / reduce) rebuilt for NVIDIA B200 (sm_100a)
behind the reference's own runtime API.

* ``vkcuda_b200.vc``    - Python mirror of the VC runtime API over the C ABI.
* ``vkcuda_b200.build`` - nvcc build of ``lib/libVCRuntime.so``.
"""
from . import vc  # noqa: F401

__all__ = ["vc"]
