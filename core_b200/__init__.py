"""CORE KV-compression step on B200 (sm_100a).

The compute path is the CUDA library ``libcore_b200.so`` (C ABI in
``include/core_b200.h``), bound with ctypes in :mod:`core_b200._lib`;
:mod:`core_b200.ops` wraps each entry point for torch tensors,
:mod:`core_b200.engine` runs one layer's compression step and
:mod:`core_b200.press` provides the KVPress-compatible presses.
"""

__version__ = "0.1.0"
