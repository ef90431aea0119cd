"""B200-native (sm_100a) backend for ZillaPHP's training hot path.

The product is the C-ABI library ``lib/libzilla_b200.so`` (include/zilla_b200.h);
this package builds it, loads it and mirrors ZillaPHP's CudaBackend on top of it.
"""
from . import configs, synthetic  # noqa: F401
from .native import LIB_PATH, load  # noqa: F401
