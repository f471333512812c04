"""The head-sharded layer step (KV heads split across ranks) against the
unsharded one, with the ranks emulated in one process on one GPU; and, where
two GPUs are present, with two real ranks over NCCL."""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from helpers import rel_err

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
L, NQ, HKV, HQ, D_MEM = 3001, 200, 8, 32, 128
LAYER = 3


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _layer(dev, ratio=0.75):
    from core_b200 import engine, synthetic
    q, k, v = synthetic.make_layer_inputs(seed=31, batch=1, n_kv_heads=HKV, n_q_heads=HQ,
                                          seq_len=L, n_queries=NQ, device=dev)
    w = synthetic.make_layer_weights(seed=32, n_kv_heads=HKV, n_q_heads=HQ, d_mem=D_MEM)
    return q, k, v, w, engine.n_kept_for(L, ratio, 4)


def _unsharded(q, k, v, w, n_kept, dev):
    from core_b200 import engine, ops
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                     n_kv_heads=HKV, n_q_heads=HQ, device=dev)
    mem = engine.MemoryState.zeros(1, D_MEM, HKV * 128, dev)
    out = engine.compress_layer(q, k, v, lw, n_kept=n_kept,
                                positions=torch.arange(L, device=dev)[None], original_length=L,
                                is_prefill=False, memory=mem)
    ops.status()
    return out, mem


def _sharded(world, q, k, v, w, n_kept, dev):
    from core_b200 import engine, ops
    from core_b200.sharded import HeadShard, LocalExchange, ShardWeights, compress_layer_sharded
    G = HQ // HKV
    shards = [HeadShard(r, world, HKV, L) for r in range(world)]
    inputs = [dict(q=q[:, s.h0 * G:s.h1 * G].contiguous(), keys=k[:, s.h0:s.h1].contiguous(),
                   values=v[:, s.h0:s.h1].contiguous()) for s in shards]
    weights = [ShardWeights.prepare(s, geometry=w["geometry"], prototypes=w["prototypes"],
                                    hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                    n_q_heads=HQ, device=dev) for s in shards]
    mem = engine.MemoryState.zeros(1, D_MEM, HKV * 128, dev)
    outs = compress_layer_sharded(LocalExchange(world), shards, inputs, weights, layer_idx=LAYER,
                                  n_kept=n_kept, positions=torch.arange(L, device=dev),
                                  original_length=L, is_prefill=False, memory=mem,
                                  keep_features=True)
    ops.status()
    return shards, outs, mem


# r = 0.75: the owner receives the compacted evicted rows; r = 0.9: whole caches
@pytest.mark.parametrize("world,ratio", [(2, 0.75), (4, 0.75), (8, 0.75), (2, 0.9), (8, 0.9)])
def test_head_sharded_step_matches_unsharded(world, ratio):
    dev = _dev()
    q, k, v, w, n_kept = _layer(dev, ratio)
    ref, ref_mem = _unsharded(q, k, v, w, n_kept, dev)
    shards, outs, mem = _sharded(world, q, k, v, w, n_kept, dev)
    feats = torch.cat([o["features"] for o in outs]).cpu().numpy()
    want = ref["features"][0].cpu().numpy()
    assert feats.shape == want.shape
    # continuous QK and coverage features: the same arithmetic up to summation order
    cont = [0, 1, 2, 3, 7, 8, 9]
    err = rel_err(feats[:, cont], want[:, cont], floor=1e-2)
    assert np.quantile(err, 0.999) < 1e-4 and err.max() < 1e-2, err.max(0)
    # discrete ones (f5, f6, occupancy) agree on nearly every key
    for c in (4, 5, 6):
        assert (np.abs(feats[:, c] - want[:, c]) > 1e-6).mean() <= 0.005, c
    # auxiliary features: the same bf16 arithmetic, bit for bit
    assert np.array_equal(feats[:, 10:], want[:, 10:])
    # every rank holds all scores and the same keep set
    for o in outs[1:]:
        assert torch.equal(o["scores"], outs[0]["scores"])
        assert torch.equal(o["keep"], outs[0]["keep"])
    s = outs[0]["scores"][0].cpu().numpy()
    s_ref = ref["scores"][0].cpu().numpy()
    serr = np.abs(s - s_ref) / np.maximum(np.abs(s_ref), 1e-3)
    assert np.quantile(serr, 0.999) < 1e-4, serr.max()
    keep = outs[0]["keep"][0].cpu().numpy()
    keep_ref = ref["keep"][0].cpu().numpy()
    sat = s_ref.copy()
    sat[:4] = sat.max() + 1
    boundary = np.sort(sat)[::-1][n_kept - 1]
    diff = np.setxor1d(keep, keep_ref)
    assert np.all(np.abs(sat[diff] - boundary) <= 1e-3 * abs(boundary)), diff
    # each rank keeps its own heads' rows of the kept tokens
    idx = outs[0]["keep"].long()[:, None, :, None].expand(-1, HKV, -1, 128)
    kk, vv = k.gather(2, idx), v.gather(2, idx)
    for sh, o in zip(shards, outs):
        assert torch.equal(o["keys"], kk[:, sh.h0:sh.h1])
        assert torch.equal(o["values"], vv[:, sh.h0:sh.h1])
    # the memory written on the owner from all heads' evicted rows
    if diff.size == 0:
        for got, exp in ((mem.M, ref_mem.M), (mem.b, ref_mem.b)):
            g, e = got.cpu().numpy(), exp.cpu().numpy()
            assert np.abs(g - e).max() <= 1e-4 * np.abs(e).max()
        assert abs(float(mem.Z[0]) - float(ref_mem.Z[0])) <= 1e-6


def test_gathered_memory_write_equals_indexed_write():
    """core_memory_write_gathered on pre-gathered rows gives the same state,
    bit for bit, as core_memory_write gathering the rows itself."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    _, k, v = synthetic.make_layer_inputs(seed=41, batch=1, n_kv_heads=HKV, n_q_heads=HQ,
                                          seq_len=2000, n_queries=8, device=dev)
    w = synthetic.make_layer_weights(seed=42, n_kv_heads=HKV, n_q_heads=HQ, d_mem=256)
    theta = engine.fold_groups(w["theta"].to(dev), HKV, HQ // HKV, 128)
    ts = ops.split_bf16(theta, 2)
    scores = torch.randn(1, 2000, device=dev) * 0.05
    keep, evict = ops.topb_select(scores, 500, 4)
    states = [engine.MemoryState.zeros(1, 256, HKV * 128, dev) for _ in range(2)]
    for st in states:
        st.Z.fill_(0.5)
        st.b.fill_(0.25)
    ops.memory_write(k, v, scores, evict, ts, states[0].M, states[0].b, states[0].Z, gamma=0.9,
                     eta=1.0, student_temp=1.0)
    ke, ve = ops.compact_kv(k, v, evict)
    ops.memory_write_gathered(ke, ve, scores, evict, ts, states[1].M, states[1].b, states[1].Z,
                              gamma=0.9, eta=1.0, student_temp=1.0)
    ops.status()
    assert torch.equal(states[0].M, states[1].M)
    assert torch.equal(states[0].b, states[1].b)
    assert torch.equal(states[0].Z, states[1].Z)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_nccl_ranks_match_emulation(tmp_path):
    """Two processes, one GPU each, over NCCL (skipped with fewer GPUs)."""
    _dev()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = _free_port()
    script = os.path.join(ROOT, "tests", "sharded_worker.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), script, str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = [torch.load(tmp_path / f"rank{i}.pt") for i in range(2)]
    dev = torch.device("cuda", 0)
    q, k, v, w, n_kept = _layer(dev)
    shards, outs, mem = _sharded(2, q, k, v, w, n_kept, dev)
    for i in range(2):
        assert torch.equal(got[i]["keep"], outs[i]["keep"].cpu())
        assert torch.allclose(got[i]["features"], outs[i]["features"].cpu(), rtol=1e-5, atol=1e-6)
        assert torch.equal(got[i]["keys"], outs[i]["keys"].cpu())
    owner = LAYER % 2
    assert torch.allclose(got[owner]["M"], mem.M.cpu(), rtol=1e-4, atol=1e-6)
