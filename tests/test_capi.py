"""The C-ABI library loads and exports every entry point declared in
include/core_b200.h; argument validation fails cleanly without touching a GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from core_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "core_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|int32_t|size_t)\s+(core_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_version_and_error_buffer():
    lib = _lib.load()
    assert lib.core_version() == 100
    assert lib.core_last_error(None, 0) != 0


def test_invalid_arguments_rejected_on_host():
    lib = _lib.load()
    # NULL tensors: rejected before any CUDA call
    rc = lib.core_topb_select(None, 1, 16, 4, 4, None, None, None, 0, None)
    assert rc == -1 and "NULL" in _lib.last_error()
    dims = _lib.CoreDims(1, 32, 8, 64, 16, 128, _lib.CORE_DTYPE_BF16)  # head_dim 64
    rc = lib.core_qk_features(ctypes.byref(dims), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 16,
                              None, None, ctypes.c_void_p(16), 14, None, 0, None)
    assert rc == -2 and "head_dim" in _lib.last_error()
    dims = _lib.CoreDims(1, 40, 8, 128, 16, 128, _lib.CORE_DTYPE_BF16)  # GQA 5
    rc = lib.core_qk_features(ctypes.byref(dims), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 16,
                              None, None, ctypes.c_void_p(16), 14, None, 0, None)
    assert rc == -2 and "group size" in _lib.last_error()
    dims = _lib.CoreDims(1, 32, 8, 128, 16, 128, 99)  # unknown dtype code
    rc = lib.core_qk_features(ctypes.byref(dims), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 16,
                              None, None, ctypes.c_void_p(16), 14, None, 0, None)
    assert rc == -2 and "dtype" in _lib.last_error()
    # f32 caches pass the dimension checks and stop at the (missing) workspace
    dims = _lib.CoreDims(1, 32, 8, 128, 16, 128, _lib.CORE_DTYPE_F32)
    rc = lib.core_qk_features(ctypes.byref(dims), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 16,
                              None, None, ctypes.c_void_p(16), 14, None, 0, None)
    assert rc == -6 and "workspace" in _lib.last_error()
    dims = _lib.CoreDims(1, 32, 8, 128, 256, 128, _lib.CORE_DTYPE_BF16)  # nq > L
    rc = lib.core_qk_features(ctypes.byref(dims), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 16,
                              None, None, ctypes.c_void_p(16), 14, None, 0, None)
    assert rc == -1
    rc = lib.core_split_bf16(None, 10, 2, None, None)
    assert rc == -1


def test_workspace_queries_are_host_only():
    lib = _lib.load()
    dims = _lib.CoreDims(1, 32, 8, 128, 128, 16384, _lib.CORE_DTYPE_BF16)
    # size queries need the SM count (a CUDA call); without a device they must not crash
    try:
        import torch
        if not torch.cuda.is_available():
            pytest.skip("SM-count dependent sizes need a device")
    except ImportError:
        pytest.skip("torch missing")
    assert lib.core_qk_features_workspace_bytes(ctypes.byref(dims)) > 0


def test_ops_refuse_cpu_tensors():
    import torch
    from core_b200 import ops
    q = torch.zeros(1, 8, 4, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.qk_features(q, k)


def test_readout_workspace_covers_a_call_without_gate():
    """The readout carves at least one gate float even when gate_hidden is 0
    (a fixed gate); the size query must count it too (pure host arithmetic)."""
    lib = _lib.load()
    dims = _lib.CoreDims(1, 32, 8, 128, 1, 1, _lib.CORE_DTYPE_BF16)
    f = lib.core_memory_readout_workspace_bytes
    assert f(ctypes.byref(dims), 1, 512, 0) == f(ctypes.byref(dims), 1, 512, 1)
    assert f(ctypes.byref(dims), 1, 512, 64) >= 4 * (512 + 64 + 8 * 128)


def test_attention_arguments_rejected_on_host():
    """core_attention_prefill refuses bad shapes before any CUDA call."""
    lib = _lib.load()
    f = lib.core_attention_prefill
    s = (ctypes.c_int64 * 3)(1 << 20, 1 << 14, 128)
    sp = ctypes.cast(s, ctypes.c_void_p)
    p = ctypes.c_void_p(256)
    dims = _lib.CoreDims(1, 8, 2, 128, 64, 64, _lib.CORE_DTYPE_BF16)
    assert f(ctypes.byref(dims), None, sp, p, sp, p, sp, p, p, 0.08, None) == -1
    dims = _lib.CoreDims(1, 8, 2, 64, 64, 64, _lib.CORE_DTYPE_BF16)
    assert f(ctypes.byref(dims), p, sp, p, sp, p, sp, p, p, 0.08, None) == -2
    assert "head_dim" in _lib.last_error()
    dims = _lib.CoreDims(1, 8, 2, 128, 65, 64, _lib.CORE_DTYPE_BF16)  # more queries than keys
    assert f(ctypes.byref(dims), p, sp, p, sp, p, sp, p, p, 0.08, None) == -2
    dims = _lib.CoreDims(1, 8, 2, 128, 64, 64, _lib.CORE_DTYPE_F32)
    assert f(ctypes.byref(dims), p, sp, p, sp, p, sp, p, p, 0.08, None) == -2
    assert "dtype" in _lib.last_error()
    dims = _lib.CoreDims(1, 8, 3, 128, 64, 64, _lib.CORE_DTYPE_BF16)  # 8 heads over 3 KV heads
    assert f(ctypes.byref(dims), p, sp, p, sp, p, sp, p, p, 0.08, None) == -1
    dims = _lib.CoreDims(1, 8, 2, 128, 64, 64, _lib.CORE_DTYPE_BF16)
    assert f(ctypes.byref(dims), p, sp, p, sp, p, sp, p, p, -1.0, None) == -1
    assert "softmax_scale" in _lib.last_error()
