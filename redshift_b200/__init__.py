"""B200 (sm_100a) build of the Redshift attention / gated-DeltaNet hot path.

The product is the C-ABI library ``build/libqvelox.so`` (see
``include/runtime.h``); this package holds its CUDA sources (``csrc/``), the
build script and the ctypes bindings.
"""
from .runtime import DEFAULT_LIBRARY, HotPath, NativeError, load_library  # noqa: F401
