"""Parity of the f32 cache path (the reference's fp32 arithmetic, on CUDA
cores) with the oracle and the reference's fp32 golden fixture.  Needs a B200
and the built library."""

import numpy as np
import pytest
import torch

from helpers import f3_flip_consistent, layer_weights, load_case, rel_err
from oracle import core_oracle as O

pytestmark = pytest.mark.gpu

CASE = "fp32_decode_L512_Q64"
# f32 everywhere: only summation orders differ from the oracle (which sums in
# f64), so continuous outputs agree to 1e-4 relative (floored at 1e-3
# absolute scale) and f32 state to 1e-5 of its largest entry.
FEAT_TOL = 1e-4
STATE_TOL = 1e-5
# d_proto and delta_proto are differences of O(1) cosines: their absolute
# precision is a few f32 ulps of 1.0 however small they are, so their relative
# error is floored at 1e-2 (absolute 1e-6).
COV_FLOOR = 1e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _f32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)


def _prepared(d, m, dev):
    from core_b200 import engine
    w = layer_weights(d)
    return engine.LayerWeights.prepare(geometry=_f32(w.geometry, dev),
                                       prototypes=_f32(w.prototypes, dev),
                                       hadamard=_f32(w.hadamard, dev),
                                       mlp_params=[_f32(x, dev) for x in w.mlp],
                                       theta=_f32(w.theta, dev), n_kv_heads=m["hkv"],
                                       n_q_heads=m["hq"], device=dev)


def test_coverage_f32_matches_golden():
    from core_b200 import ops
    dev = _dev()
    d, m = load_case(CASE)
    geo = ops.prepare_geometry(_f32(d["geometry"], dev), _f32(d["hadamard"], dev))
    cov = ops.coverage_features(_f32(d["k"], dev)[None], geo, _f32(d["prototypes"], dev))
    ops.status()
    got = cov[0].cpu().numpy()
    ref = O.coverage_features(d["k"], d["geometry"], d["prototypes"], d["hadamard"])
    for want in (ref, d["features"][:, 6:10]):
        # occupancy log1p(count): the same counts, the log within one f32 ulp
        assert np.array_equal(np.rint(np.expm1(got[:, 0])), np.rint(np.expm1(want[:, 0])))
        np.testing.assert_allclose(got[:, 0], want[:, 0], rtol=2.4e-7, atol=0)
        assert rel_err(got[:, 1:], want[:, 1:], floor=COV_FLOOR).max() < FEAT_TOL


def test_indexer_f32_matches_golden():
    from core_b200 import ops
    dev = _dev()
    d, m = load_case(CASE)
    L = m["L"]
    feats = torch.zeros(1, L, 14, device=dev)
    feats[0, :, :10] = _f32(d["features"][:, :10], dev)
    w = layer_weights(d)
    mlp = ops.pack_mlp([_f32(x, dev) for x in w.mlp])
    scores = ops.indexer_scores(_f32(d["v"], dev)[None], torch.arange(L, device=dev)[None], feats,
                                mlp, original_length=L, is_prefill=bool(m["prefill"]), n_sink=4)
    ops.status()
    aux = O.auxiliary_features(d["v"], np.arange(L), seq_len=L, is_prefill=bool(m["prefill"]),
                               round_bf16=False)
    np.testing.assert_allclose(feats[0, :, 10:].cpu().numpy(), aux, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(feats[0, :, 10:].cpu().numpy(), d["features"][:, 10:],
                               rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(scores[0].cpu().numpy(), d["scores"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("d_mem,L,hkv,n_kept", [(64, 512, 2, 128), (512, 1300, 8, 300),
                                                (128, 700, 4, 699)])
def test_memory_write_f32_matches_oracle(d_mem, L, hkv, n_kept):
    from core_b200 import engine, ops
    dev = _dev()
    hq = 4 * hkv
    rng = np.random.default_rng(d_mem * 7 + L)
    k = (rng.standard_normal((hkv, L, 128)) / np.sqrt(128)).astype(np.float32)
    v = rng.standard_normal((hkv, L, 128)).astype(np.float32)
    scores = (rng.standard_normal(L) * 0.05).astype(np.float32)
    theta = (rng.standard_normal((d_mem, hq * 128)) / np.sqrt(hq * 128)).astype(np.float32)
    keep = O.topb_select(scores[None], n_kept, 4)[0]
    evict = np.setdiff1d(np.arange(L), keep)
    mask = np.zeros(L, bool)
    mask[evict] = True
    M0 = (rng.standard_normal((d_mem, hkv * 128)) * 0.1).astype(np.float32)
    b0 = np.abs(rng.standard_normal(d_mem)).astype(np.float32)
    Z0 = np.float32(0.7)
    ref_M, ref_b, ref_Z = O.memory_write(k, v, scores, mask, theta, groups=4, M=M0, b=b0, Z=Z0)
    fold = engine.fold_groups(_f32(theta, dev), hkv, 4, 128)
    M = _f32(M0, dev)[None].contiguous()
    b = _f32(b0, dev)[None].contiguous()
    Z = torch.full((1,), float(Z0), device=dev)
    ops.memory_write(_f32(k, dev)[None], _f32(v, dev)[None], _f32(scores, dev)[None],
                     torch.from_numpy(evict.astype(np.int32)).to(dev)[None], fold, M, b, Z,
                     gamma=0.9, eta=1.0, student_temp=1.0)
    ops.status()
    assert np.abs(M[0].cpu().numpy() - ref_M).max() <= STATE_TOL * np.abs(ref_M).max()
    assert np.abs(b[0].cpu().numpy() - ref_b).max() <= STATE_TOL * np.abs(ref_b).max()
    assert abs(float(Z[0]) - float(ref_Z)) <= 1e-6


def test_compact_kv_f32_is_exact_gather():
    from core_b200 import ops, synthetic
    dev = _dev()
    _, k, v = synthetic.make_layer_inputs(seed=6, batch=2, n_kv_heads=4, n_q_heads=16,
                                          seq_len=900, n_queries=8, device=dev,
                                          dtype=torch.float32)
    rng = np.random.default_rng(1)
    keep = np.stack([np.sort(rng.choice(900, 301, replace=False)) for _ in range(2)]).astype(np.int32)
    kt = torch.from_numpy(keep).to(dev)
    ok, ov = ops.compact_kv(k, v, kt)
    idx = kt.long()[:, None, :, None].expand(-1, 4, -1, 128)
    assert ok.dtype == torch.float32
    assert torch.equal(ok, k.gather(2, idx))
    assert torch.equal(ov, v.gather(2, idx))


@pytest.mark.parametrize("q_len,gate_override", [(1, None), (3, None), (2, 0.5)])
def test_memory_readout_f32_matches_oracle(q_len, gate_override):
    from core_b200 import ops
    dev = _dev()
    hkv, hq, d_mem, gh, hidden = 2, 8, 64, 32, 256
    rng = np.random.default_rng(q_len)
    q = rng.standard_normal((q_len, hq * 128)).astype(np.float32)
    theta = (rng.standard_normal((d_mem, hq * 128)) / 32).astype(np.float32)
    w1 = (rng.standard_normal((gh, hq * 128)) / 32).astype(np.float32)
    b1 = rng.standard_normal(gh).astype(np.float32) * 0.1
    w2 = rng.standard_normal(gh).astype(np.float32) * 0.1
    b2 = np.float32([0.2])
    M = rng.standard_normal((d_mem, hkv * 128)).astype(np.float32)
    b = np.abs(rng.standard_normal(d_mem)).astype(np.float32)
    ofold = (rng.standard_normal((hidden, hkv * 128)) / 16).astype(np.float32)
    attn = rng.standard_normal((q_len, hidden)).astype(np.float32)
    ref = O.memory_readout(q, theta, w1, b1, w2[None], b2, M, b, ofold, attn,
                           gate_override=gate_override, out_bf16=False)
    qt = _f32(q, dev).reshape(q_len, hq, 128).permute(1, 0, 2)[None].contiguous()
    out = _f32(attn, dev)[None].contiguous()
    ops.memory_readout(qt, _f32(theta, dev), (_f32(w1, dev), _f32(b1, dev), _f32(w2, dev),
                                              _f32(b2, dev)),
                       _f32(M, dev)[None], _f32(b, dev)[None], _f32(ofold, dev), out,
                       n_kv_heads=hkv, gate_override=gate_override)
    ops.status()
    assert out.dtype == torch.float32
    np.testing.assert_allclose(out[0].cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


def test_compress_layer_f32_matches_golden():
    """The whole layer step on f32 caches through the public engine call:
    features, scores, the retained set and K/V, and the memory state."""
    from core_b200 import engine, ops
    dev = _dev()
    d, m = load_case(CASE)
    L, hkv = m["L"], m["hkv"]
    lw = _prepared(d, m, dev)
    mem = engine.MemoryState.zeros(1, m["d_mem"], hkv * 128, dev)
    n_kept = engine.n_kept_for(L, m["ratio"], 4)
    k = _f32(d["k"], dev)[None]
    v = _f32(d["v"], dev)[None]
    out = engine.compress_layer(_f32(d["q"], dev)[None], k, v, lw, n_kept=n_kept,
                                positions=torch.arange(L, device=dev)[None], original_length=L,
                                is_prefill=bool(m["prefill"]), memory=mem)
    ops.status()
    f = out["features"][0].cpu().numpy()
    g = d["features"]
    assert rel_err(f[:, :4], g[:, :4]).max() < FEAT_TOL
    assert rel_err(f[:, 7:10], g[:, 7:10], floor=COV_FLOOR).max() < FEAT_TOL
    for c in (4, 5, 6):  # f5, f6, occupancy: discrete
        assert (np.abs(f[:, c] - g[:, c]) > 1e-6).mean() <= 0.002, c
    np.testing.assert_allclose(f[:, 10:], g[:, 10:], rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(out["scores"][0].cpu().numpy(), d["scores"], rtol=2e-4, atol=1e-5)
    keep = out["keep"][0].cpu().numpy()
    assert np.array_equal(keep, d["keep"])
    assert out["keys"].dtype == torch.float32
    assert np.array_equal(out["keys"][0].cpu().numpy(), d["out_k"])
    assert np.array_equal(out["values"][0].cpu().numpy(), d["out_v"])
    gM, gb = d["M"], d["b"]
    assert np.abs(mem.M[0].cpu().numpy() - gM).max() <= STATE_TOL * np.abs(gM).max()
    assert np.abs(mem.b[0].cpu().numpy() - gb).max() <= STATE_TOL * np.abs(gb).max()
    assert abs(float(mem.Z[0]) - float(d["Z"][0])) <= 1e-6


def test_compress_layer_f32_single_layer_4096():
    """The single-layer fp32 workload: batch 1, 4096 cached tokens, 8 KV heads
    x 128, 32 query heads, 128 buffered queries, compression ratio 0.75, with
    the seeded Gaussian-with-outlier inputs; every output against the oracle."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L, nq, hkv, hq, d_mem = 4096, 128, 8, 32, 128
    q, k, v = synthetic.make_layer_inputs(seed=0, batch=1, n_kv_heads=hkv, n_q_heads=hq,
                                          seq_len=L, n_queries=nq, device=dev,
                                          dtype=torch.float32)
    w = synthetic.make_layer_weights(seed=1, n_kv_heads=hkv, n_q_heads=hq, d_mem=d_mem)
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"],
                                     theta=w["theta"], n_kv_heads=hkv, n_q_heads=hq, device=dev)
    mem = engine.MemoryState.zeros(1, d_mem, hkv * 128, dev)
    n_kept = engine.n_kept_for(L, 0.75, 4)
    out = engine.compress_layer(q, k, v, lw, n_kept=n_kept,
                                positions=torch.arange(L, device=dev)[None], original_length=L,
                                is_prefill=False, memory=mem)
    ops.status()
    ow = O.LayerWeights(mlp=tuple(x.float().cpu().numpy() for x in w["mlp"]),
                        geometry=w["geometry"].float().cpu().numpy(),
                        prototypes=w["prototypes"].float().cpu().numpy(),
                        hadamard=w["hadamard"].float().cpu().numpy(),
                        theta=w["theta"].float().cpu().numpy())
    qn = q[0].reshape(hq, nq, 128).cpu().numpy()
    kn = k[0].cpu().numpy()
    ref = O.compress_layer(qn, kn, v[0].cpu().numpy(), ow, compression_ratio=0.75,
                           is_prefill=False, round_bf16=False)
    _, _, R = O.qk_features(qn, kn, groups=4, round_bf16=False)
    f = out["features"][0].cpu().numpy()
    g = ref["features"]
    err = rel_err(f[:, :4], g[:, :4])
    assert err[:, [0, 1, 3]].max() < FEAT_TOL
    # f3 up to sign flips of relation values within f32 rounding of 0
    bad = np.nonzero(err[:, 2] > FEAT_TOL)[0]
    assert len(bad) <= 0.002 * L, len(bad)
    ok, key = f3_flip_consistent(f[:, 2], R, bad, rtol=FEAT_TOL, near=1e-5)
    assert ok, (key, f[key, 2], g[key, 2])
    assert rel_err(f[:, 7:10], g[:, 7:10], floor=COV_FLOOR).max() < FEAT_TOL
    for c in (4, 5, 6):
        assert (np.abs(f[:, c] - g[:, c]) > 1e-6).mean() <= 0.002, c
    s = out["scores"][0].cpu().numpy()
    # the MLP on this path's own features, the Top-B of its own scores
    np.testing.assert_allclose(s, O.indexer_mlp(f, *ow.mlp), rtol=1e-5, atol=1e-6)
    keep = out["keep"][0].cpu().numpy()
    assert np.array_equal(keep, O.topb_select(s[None], n_kept, 4)[0])
    unflipped = np.ones(L, bool)
    unflipped[bad] = False
    np.testing.assert_allclose(s[unflipped], ref["scores"][unflipped], rtol=2e-4, atol=1e-5)
    # the retained set differs from the oracle's only at the Top-B boundary or a flipped key
    diff = np.setxor1d(keep, ref["keep"])
    sr = ref["scores"].copy()
    sr[:4] = sr.max() + 1
    boundary = np.sort(sr)[::-1][n_kept - 1]
    assert np.all((np.abs(sr[diff] - boundary) <= 1e-4 * abs(boundary)) | ~unflipped[diff]), diff
    # the memory write over this path's evicted set
    evicted = np.ones(L, bool)
    evicted[keep] = False
    rM, rb, rZ = O.memory_write(kn, v[0].cpu().numpy(), s, evicted, ow.theta, groups=4)
    assert np.abs(mem.M[0].cpu().numpy() - rM).max() <= STATE_TOL * np.abs(rM).max()
    assert np.abs(mem.b[0].cpu().numpy() - rb).max() <= STATE_TOL * np.abs(rb).max()
    assert abs(float(mem.Z[0]) - float(rZ)) <= 1e-6
