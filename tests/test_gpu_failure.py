"""Failure handling on the GPU without a fault: a bounded device-side wait
that nothing completes gives up after its limit, the library reports
CORE_ERR_TIMEOUT through the device status, and the context stays usable."""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def test_bounded_wait_gives_up_and_context_stays_usable():
    from core_b200 import _lib, ops
    dev = _dev()
    ops.status(dev)  # start clean
    lib = _lib.load()
    t0 = time.perf_counter()
    _lib.check(lib.core_selftest_wait_timeout(2000, ops._stream(dev)))  # 2 ms limit
    with pytest.raises(_lib.CoreError) as err:
        ops.status(dev)
    elapsed = time.perf_counter() - t0
    assert err.value.code == _lib.CORE_ERR_TIMEOUT
    assert "where=990" in str(err.value)
    assert elapsed < 5.0  # the wait ended by its own limit
    # the status was cleared and the context still runs kernels
    ops.status(dev)
    s = torch.arange(10000, dtype=torch.float32, device=dev)[None] % 97
    keep, _ = ops.topb_select(s, 1000, 4)
    ops.status(dev)
    from oracle import core_oracle as O
    assert np.array_equal(keep[0].cpu().numpy(), O.topb_select(s.cpu().numpy(), 1000, 4)[0])


def test_selftest_rejects_bad_limits():
    from core_b200 import _lib, ops
    dev = _dev()
    lib = _lib.load()
    assert lib.core_selftest_wait_timeout(0, ops._stream(dev)) == _lib.CORE_ERR_INVALID_ARG
    assert lib.core_selftest_wait_timeout(2_000_000, ops._stream(dev)) == _lib.CORE_ERR_INVALID_ARG
