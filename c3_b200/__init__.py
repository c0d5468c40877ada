"""C3 B200: the fused hot path of ShengFlow/C3 (MatMul+Add+ReLU region, its captured
backward, elementwise chains) as hand-written sm_100a kernels behind a C ABI
(include/c3cu.h), with a C++ mirror of C3's install-and-dispatch API."""
from . import _lib
from ._lib import C3CUError, device_check, fault_status, load
from . import linear, elementwise

__all__ = ["C3CUError", "device_check", "fault_status", "load", "linear", "elementwise", "_lib"]
