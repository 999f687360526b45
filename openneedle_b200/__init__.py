"""B200 (sm_100a) build of OpenNeedle's quantized hot path behind its C ABI."""
from .native import DeviceMatrix, available, features, library_path, sdot_available  # noqa: F401

__all__ = ["DeviceMatrix", "available", "features", "library_path", "sdot_available"]
