"""core_memory_readout_noalloc (static device scratch) against core_memory_readout.

Collected last (file name) so it also runs after every other GPU test has
used the library.  Calls the new entry point directly through the C-ABI.
"""

import ctypes

import numpy as np
import pytest
import torch

from helpers import TWO_STEP_CASE, load_case

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _inputs(dev):
    from core_b200 import engine
    d, m = load_case(TWO_STEP_CASE)
    hkv, hq = m["hkv"], m["hq"]
    def f32(x):
        return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev).contiguous()

    def bf16(x):
        return f32(x).to(torch.bfloat16).contiguous()

    w = dict(theta=f32(d["theta"]), w1=f32(d["gate_w1"]), b1=f32(d["gate_b1"]),
             w2=f32(d["gate_w2"]).reshape(-1).contiguous(), b2=f32(d["gate_b2"]).reshape(-1).contiguous(),
             M=f32(d["M2"])[None].contiguous(), b=f32(d["b2"])[None].contiguous(),
             ofold=engine.fold_groups(f32(d["o_proj"]), hkv, hq // hkv, 128).contiguous())
    cases = [(bf16(d[f"readout_q{ql}"])[None].contiguous(), bf16(d[f"readout_attn{ql}"]).contiguous())
             for ql in (1, 3)]
    return w, cases, hkv


def _call(lib, name, q, w, attn, hkv, ws=None):
    from core_b200 import _lib
    B, hq, q_len, d = q.shape
    dims = _lib.CoreDims(B, hq, hkv, d, q_len, q_len, _lib.CORE_DTYPE_BF16)
    d_mem, gh, hidden = w["theta"].shape[0], w["w1"].shape[0], w["ofold"].shape[0]
    args = [ctypes.byref(dims), q_len, q.data_ptr(), w["theta"].data_ptr(), w["w1"].data_ptr(),
            w["b1"].data_ptr(), w["w2"].data_ptr(), w["b2"].data_ptr(), d_mem, gh, float("nan"),
            w["M"].data_ptr(), w["b"].data_ptr(), w["ofold"].data_ptr(), hidden, attn.data_ptr()]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    args.append(torch.cuda.current_stream(q.device).cuda_stream)
    rc = getattr(lib, name)(*args)
    assert rc == 0, _lib.last_error()


def test_noalloc_readout_matches_workspace_readout_twice():
    from core_b200 import _lib, ops
    dev = _dev()
    lib = _lib.load()
    w, cases, hkv = _inputs(dev)
    for _ in range(2):  # two calls in a row reuse the static scratch
        for q, attn in cases:
            B, hq, q_len, d = q.shape
            dims = _lib.CoreDims(B, hq, hkv, d, q_len, q_len, _lib.CORE_DTYPE_BF16)
            nbytes = lib.core_memory_readout_workspace_bytes(ctypes.byref(dims), q_len,
                                                             w["theta"].shape[0], w["w1"].shape[0])
            ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            ref = attn.clone()
            _call(lib, "core_memory_readout", q, w, ref, hkv, ws)
            got = attn.clone()
            _call(lib, "core_memory_readout_noalloc", q, w, got, hkv)
            torch.cuda.synchronize()
            ops.status(dev)
            # same kernels on the same inputs: bit-identical bf16 outputs
            assert torch.equal(got, ref)
            assert not torch.equal(got, attn)  # the readout did add to the output


def test_noalloc_readout_rejects_oversized_call():
    from core_b200 import _lib
    dev = _dev()
    lib = _lib.load()
    w, cases, hkv = _inputs(dev)
    q, attn = cases[1]
    # B=64 x q_len=3 overflows the 256 KB scratch; every operand is sized for
    # B=64 so that the call stays in bounds even if it were not rejected
    big_q = q.expand(64, -1, -1, -1).contiguous()
    big_attn = attn.expand(64, -1, -1).contiguous()
    w = dict(w, M=w["M"].expand(64, -1, -1).contiguous(), b=w["b"].expand(64, -1).contiguous())
    B, hq, q_len, d = big_q.shape
    dims = _lib.CoreDims(B, hq, hkv, d, q_len, q_len, _lib.CORE_DTYPE_BF16)
    rc = lib.core_memory_readout_noalloc(
        ctypes.byref(dims), q_len, big_q.data_ptr(), w["theta"].data_ptr(), w["w1"].data_ptr(),
        w["b1"].data_ptr(), w["w2"].data_ptr(), w["b2"].data_ptr(), w["theta"].shape[0],
        w["w1"].shape[0], float("nan"), w["M"].data_ptr(), w["b"].data_ptr(), w["ofold"].data_ptr(),
        w["ofold"].shape[0], big_attn.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -1  # CORE_ERR_INVALID_ARG, before any launch
    assert "static scratch" in _lib.last_error()
