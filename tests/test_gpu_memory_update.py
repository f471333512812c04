"""The memory recurrence M, b <- (gamma Z M + pi_E eta M_bar) / Z' has two
kernels: four columns of M per thread when M is 16-byte aligned, one element
per thread otherwise.  Both evaluate every element with the same expressions
in the same split order, so an M that starts 4 bytes past an aligned address
must give the same bits as an aligned one."""

import numpy as np
import pytest
import torch

from oracle import core_oracle as O

pytestmark = pytest.mark.gpu


def test_unaligned_memory_state_gives_the_same_bits():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from core_b200 import engine, ops
    dev = torch.device("cuda", 0)
    hkv, hq, L, d_mem = 8, 32, 3000, 256
    rng = np.random.default_rng(11)
    k = O.bf16_round(rng.standard_normal((hkv, L, 128), dtype=np.float32) / np.float32(np.sqrt(128)))
    v = O.bf16_round(rng.standard_normal((hkv, L, 128), dtype=np.float32))
    scores = (rng.standard_normal(L) * 0.05).astype(np.float32)
    theta = (rng.standard_normal((d_mem, hq * 128)) / np.sqrt(hq * 128)).astype(np.float32)
    keep = O.topb_select(scores[None], L // 4, 4)[0]
    evict = torch.from_numpy(np.setdiff1d(np.arange(L), keep).astype(np.int32)).to(dev)[None]
    kt = torch.from_numpy(k).to(dev, torch.bfloat16)[None]
    vt = torch.from_numpy(v).to(dev, torch.bfloat16)[None]
    st = torch.from_numpy(scores).to(dev)[None]
    ts = ops.split_bf16(engine.fold_groups(torch.from_numpy(theta).to(dev), hkv, 4, 128), 2)
    n = d_mem * hkv * 128
    M0 = torch.from_numpy(rng.standard_normal((1, d_mem, hkv * 128)).astype(np.float32)).to(dev)
    b0 = torch.from_numpy(rng.standard_normal((1, d_mem)).astype(np.float32)).to(dev)
    states = []
    for offset in (0, 1):  # floats past a 256-byte aligned allocation
        buf = torch.empty(n + 4, device=dev)
        M = buf[offset:offset + n].view(1, d_mem, hkv * 128)
        assert (M.data_ptr() % 16 == 0) == (offset == 0)
        M.copy_(M0)
        b = b0.clone()
        Z = torch.full((1,), 2.5, device=dev)
        for _ in range(2):  # two writes in a row: the second starts from the first's state
            ops.memory_write(kt, vt, st, evict, ts, M, b, Z, gamma=0.9, eta=1.0, student_temp=1.0)
        ops.status()
        states.append((M.clone(), b.clone(), Z.clone()))
    (Ma, ba, Za), (Mu, bu, Zu) = states
    assert torch.equal(Ma, Mu)
    assert torch.equal(ba, bu)
    assert torch.equal(Za, Zu)
    assert bool(torch.isfinite(Ma).all()) and not torch.equal(Ma, M0)
