"""ctypes binding of ``libcore_b200.so`` (the C ABI declared in include/core_b200.h).

The library is the product: there is no fallback.  Loading fails loudly when
the shared object is missing or lacks a symbol.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcore_b200.so"

CORE_OK = 0
CORE_DTYPE_BF16 = 1
CORE_DTYPE_F32 = 2
CORE_DTYPE_F16 = 3

CORE_ERR_INVALID_ARG = -1
CORE_ERR_UNSUPPORTED = -2
CORE_ERR_NONFINITE = -3
CORE_ERR_TIMEOUT = -4
CORE_ERR_CUDA = -5
CORE_ERR_WORKSPACE = -6
ERRORS = {
    -1: "invalid argument",
    -2: "unsupported",
    -3: "non-finite value",
    -4: "timeout",
    -5: "CUDA error",
    -6: "workspace too small",
}


class CoreDims(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("n_q_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_queries", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class CoreLayerWeights(ctypes.Structure):
    _fields_ = [
        ("geometry_ext", ctypes.c_void_p),
        ("prototypes", ctypes.c_void_p),
        ("mlp", ctypes.c_void_p),
        ("theta_split", ctypes.c_void_p),
        ("d_mem", ctypes.c_int32),
    ]


class CoreCompressArgs(ctypes.Structure):
    _fields_ = [
        ("n_kept", ctypes.c_int32),
        ("n_sink", ctypes.c_int32),
        ("topk_qk", ctypes.c_int32),
        ("n_recent_queries", ctypes.c_int32),
        ("shrinkage_rho", ctypes.c_float),
        ("original_length", ctypes.c_int32),
        ("is_prefill", ctypes.c_int32),
        ("gamma", ctypes.c_float),
        ("eta", ctypes.c_float),
        ("student_temp", ctypes.c_float),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_F = ctypes.c_float
_S = ctypes.c_size_t
_D = ctypes.POINTER(CoreDims)

# name -> (restype, argtypes); mirrors include/core_b200.h
SIGNATURES = {
    "core_version": (ctypes.c_int, []),
    "core_last_error": (ctypes.c_int, [ctypes.c_char_p, _S]),
    "core_check_device_status": (ctypes.c_int, [_P]),
    "core_qk_features_workspace_bytes": (_S, [_D]),
    "core_qk_features": (ctypes.c_int, [_D, _P, _P, _I, _I, _P, _P, _P, _I, _P, _S, _P]),
    "core_coverage_workspace_bytes": (_S, [_D]),
    "core_coverage_features": (ctypes.c_int, [_D, _P, _P, _P, _F, _P, _I, _I, _P, _S, _P]),
    "core_prepare_geometry": (ctypes.c_int, [_P, _P, _I, _P, _P]),
    "core_indexer_scores": (ctypes.c_int, [_D, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "core_indexer_mlp_bytes": (_S, []),
    "core_prepare_indexer_mlp": (ctypes.c_int, [_P, _P]),
    "core_topb_workspace_bytes": (_S, [_I, _I]),
    "core_topb_select": (ctypes.c_int, [_P, _I, _I, _I, _I, _P, _P, _P, _S, _P]),
    "core_memory_write_workspace_bytes": (_S, [_D, _I, _I]),
    "core_memory_write": (ctypes.c_int, [_D, _P, _P, _P, _P, _I, _P, _I, _F, _F, _F, _P, _P, _P,
                                         _P, _S, _P]),
    "core_compact_kv": (ctypes.c_int, [_D, _P, _P, _P, _I, _P, _P, _P]),
    "core_memory_readout_workspace_bytes": (_S, [_D, _I, _I, _I]),
    "core_memory_readout": (ctypes.c_int, [_D, _I, _P, _P, _P, _P, _P, _P, _I, _I, _F, _P, _P, _P,
                                           _I, _P, _P, _S, _P]),
    "core_memory_readout_noalloc": (ctypes.c_int, [_D, _I, _P, _P, _P, _P, _P, _P, _I, _I, _F,
                                                   _P, _P, _P, _I, _P, _P]),
    "core_set_sm_budget": (ctypes.c_int, [_I]),
    "core_selftest_wait_timeout": (ctypes.c_int, [_I, _P]),
    "core_split_bf16": (ctypes.c_int, [_P, ctypes.c_int64, _I, _P, _P]),
    "core_qk_summary_words": (_I, [_I]),
    "core_qk_head_summary": (ctypes.c_int, [_D, _P, _P, _I, _I, _P, _P, _P, _S, _P]),
    "core_qk_merge_summaries": (ctypes.c_int, [_P, _I, ctypes.c_int64, _I, _I, _I, _I, _I, _I, _I,
                                               _P, _I, _P]),
    "core_coverage_partial_projection": (ctypes.c_int, [_D, _P, _P, _P, _P, _S, _P]),
    "core_coverage_range_workspace_bytes": (_S, [_I]),
    "core_coverage_range_totals": (ctypes.c_int, [_P, _I, _P, _P, _P, _P, _P, _S, _P]),
    "core_coverage_range_assign": (ctypes.c_int, [_P, _I, _F, _P, _P, _I, _P, _P, _P, _P, _I, _I,
                                                  _P, _S, _P]),
    "core_coverage_range_occupancy": (ctypes.c_int, [_P, _P, _I, _P, _I, _I, _P]),
    "core_value_head_sums": (ctypes.c_int, [_D, _P, _P, ctypes.c_int64, _P]),
    "core_indexer_scores_from_sums": (ctypes.c_int, [_I, _I, _P, ctypes.c_int64, _P, _P, _I, _I,
                                                     _I, _P, _P, _P, _P]),
    "core_memory_write_gathered": (ctypes.c_int, [_D, _P, _P, _P, _P, _I, _P, _I, _F, _F, _F, _P,
                                                  _P, _P, _P, _S, _P]),
    "core_rope_queries": (ctypes.c_int, [_I, _I, _I, _I, _I, _P, ctypes.c_int64, _P, _P, _F, _P,
                                         _P, _I, _P, _P]),
    "core_attention_prefill": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _F, _P]),
    "core_compress_layer_workspace_bytes": (_S, [_D, _I, _I]),
    "core_compress_layer": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P,
                                           ctypes.POINTER(CoreLayerWeights),
                                           ctypes.POINTER(CoreCompressArgs), _P, _P, _P, _P, _P,
                                           _P, _P, _P, _P, _P, _S, _P, _P, _P]),
}


class CoreError(RuntimeError):
    """A non-zero status returned by the CUDA library."""

    def __init__(self, code: int, message: str):
        super().__init__(f"core_b200 error {code} ({ERRORS.get(code, '?')}): {message}")
        self.code = code


_lib = None


def load(path: str | os.PathLike | None = None):
    """Load the shared library (once) and bind every declared symbol."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m core_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is missing
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().core_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != CORE_OK:
        raise CoreError(rc, last_error())
