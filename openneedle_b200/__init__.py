"""B200 (sm_100a) build of OpenNeedle's quantized hot path.

The CUDA kernels and the C ABI live in ``libneedle2_b200.so`` (built from
``csrc/`` by :mod:`openneedle_b200.build`); :mod:`openneedle_b200.native`
mirrors the reference's ctypes layer on top of it.
"""
from .native import NativeCQ, available, features, library_path, sdot_available  # noqa: F401

__all__ = ["NativeCQ", "available", "features", "library_path", "sdot_available"]
