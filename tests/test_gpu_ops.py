"""Parity of each CUDA entry point with the oracle (and through it, with the
reference's golden fixtures).  Needs a B200 and the built library."""

import numpy as np
import pytest
import torch

from helpers import (SINGLE_STEP_CASES, TWO_STEP_CASE, check_qk_features_bounded,
                     check_scores_explained, flip_bound, layer_weights, load_case, rel_err)
from oracle import core_oracle as O

pytestmark = pytest.mark.gpu

BF16_CASES = [c for c in SINGLE_STEP_CASES if c.startswith("bf16")]
# Tolerances (bf16 compute): relative, floored at 1e-3 absolute scale, on
# every key.  Logits are rounded to bf16 after an f32 dot product whose
# summation order differs between the tensor cores and the oracle, so a rare
# logit lands one bf16 ulp away; a key outside FEATURE_TOL must be explained
# by such flips (helpers.check_qk_features_bounded counts and bounds them).
FEATURE_TOL = 2e-3
LSE_TOL = 2e-5


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(torch.bfloat16)


def _f32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)


def _discrete_mismatch(a, b, step):
    """Fraction of entries that differ, and the largest difference in units of step."""
    d = np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))
    return float((d > 1e-6).mean()), float(d.max() / step)


def _check_qk(q, k, got, ref, lse, ref_lse, R, max_frac=0.01):
    lse_err = float(np.abs(lse - ref_lse).max())
    assert lse_err <= LSE_TOL * np.abs(ref_lse).max()
    return check_qk_features_bounded(got, ref, R, flip_bound(q, k, lse_err), rtol=FEATURE_TOL,
                                     max_frac=max_frac)


@pytest.mark.parametrize("name", BF16_CASES)
def test_qk_features_match_oracle(name):
    from core_b200 import ops
    dev = _dev()
    d, m = load_case(name)
    q = _bf16(d["q"], dev)[None]
    k = _bf16(d["k"], dev)[None]
    feats, lse = ops.qk_features(q, k)
    ops.status()
    ref, ref_lse, R = O.qk_features(d["q"], d["k"], groups=m["hq"] // m["hkv"], round_bf16=True)
    _check_qk(d["q"], d["k"], feats[0].cpu().numpy(), ref, lse[0].cpu().numpy(), ref_lse, R)


def test_qk_features_llama_shapes_4096():
    from core_b200 import ops, synthetic
    dev = _dev()
    q, k, _ = synthetic.make_layer_inputs(seed=11, batch=1, n_kv_heads=8, n_q_heads=32,
                                          seq_len=4096, n_queries=128, device=dev)
    feats, lse = ops.qk_features(q, k)
    ops.status()
    qn = q[0].float().cpu().numpy()
    kn = k[0].float().cpu().numpy()
    ref, ref_lse, R = O.qk_features(qn, kn, groups=4, round_bf16=True)
    _check_qk(qn, kn, feats[0].cpu().numpy(), ref, lse[0].cpu().numpy(), ref_lse, R)


def test_qk_features_full_scope_prefill_2048():
    """Full-scope prefill (every cached token also a query, Q = L, the
    reference's prefill_qk_scope="all") at the largest supported query count."""
    from core_b200 import ops, synthetic
    dev = _dev()
    L = 2048
    q, k, _ = synthetic.make_layer_inputs(seed=12, batch=1, n_kv_heads=4, n_q_heads=16,
                                          seq_len=L, n_queries=L, device=dev)
    feats, lse = ops.qk_features(q, k)
    ops.status()
    qn = q[0].float().cpu().numpy()
    kn = k[0].float().cpu().numpy()
    ref, ref_lse, R = O.qk_features(qn, kn, groups=4, round_bf16=True)
    _check_qk(qn, kn, feats[0].cpu().numpy(), ref, lse[0].cpu().numpy(), ref_lse, R)


def test_qk_features_full_scope_prefill_8192():
    """Full-scope prefill beyond 2048 queries (every cached token a query):
    fully masked units above the diagonal are skipped, the merge reads only
    the query blocks that see each key, and undecided f6 heads go through the
    radix-select resolver."""
    from core_b200 import ops, synthetic
    dev = _dev()
    L = 8192
    q, k, _ = synthetic.make_layer_inputs(seed=14, batch=1, n_kv_heads=2, n_q_heads=8,
                                          seq_len=L, n_queries=L, device=dev)
    feats, lse = ops.qk_features(q, k)
    ops.status()
    qn = q[0].float().cpu().numpy()
    kn = k[0].float().cpu().numpy()
    ref, ref_lse, R = O.qk_features(qn, kn, groups=4, round_bf16=True)
    # a key is seen by up to 8192 queries here, so the keys touched by some
    # one-ulp logit flip (each one still bounded) grow with the query count
    _check_qk(qn, kn, feats[0].cpu().numpy(), ref, lse[0].cpu().numpy(), ref_lse, R, max_frac=0.05)


def test_compress_layer_full_scope_16k():
    """A 16K prefill scored by all its queries (the reference's default
    prefill_qk_scope="all") through the fused layer step: it runs, keeps the
    budget with the sinks, and its features are finite and in range."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L, hkv, hq = 16384, 8, 32
    q, k, v = synthetic.make_layer_inputs(seed=15, batch=1, n_kv_heads=hkv, n_q_heads=hq,
                                          seq_len=L, n_queries=L, device=dev)
    w = synthetic.make_layer_weights(seed=16, n_kv_heads=hkv, n_q_heads=hq, d_mem=512)
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                     n_kv_heads=hkv, n_q_heads=hq, device=dev)
    mem = engine.MemoryState.zeros(1, 512, hkv * 128, dev)
    n_kept = engine.n_kept_for(L, 0.75, 4)
    out = engine.compress_layer(q, k, v, lw, n_kept=n_kept, positions=torch.arange(L, device=dev)[None],
                                original_length=L, is_prefill=True, memory=mem)
    ops.status()
    f = out["features"][0].cpu().numpy()
    assert np.isfinite(f).all()
    assert ((f[:, 4] >= 0) & (f[:, 4] <= 1) & (f[:, 5] >= 0) & (f[:, 5] <= 1)).all()
    keep = out["keep"][0].cpu().numpy()
    assert keep.size == n_kept and np.all(np.diff(keep) > 0) and np.all(keep[:4] == np.arange(4))
    assert np.isfinite(mem.M.cpu().numpy()).all() and float(mem.Z[0]) > 0


def test_qk_features_q512_L32768():
    """The long-context query buffer (512 queries) over 32768 cached keys."""
    from core_b200 import ops, synthetic
    dev = _dev()
    q, k, _ = synthetic.make_layer_inputs(seed=13, batch=1, n_kv_heads=2, n_q_heads=8,
                                          seq_len=32768, n_queries=512, device=dev)
    feats, lse = ops.qk_features(q, k)
    ops.status()
    qn = q[0].float().cpu().numpy()
    kn = k[0].float().cpu().numpy()
    ref, ref_lse, R = O.qk_features(qn, kn, groups=4, round_bf16=True)
    _check_qk(qn, kn, feats[0].cpu().numpy(), ref, lse[0].cpu().numpy(), ref_lse, R)


def test_qk_features_batch_rows_are_independent():
    from core_b200 import ops, synthetic
    dev = _dev()
    q, k, _ = synthetic.make_layer_inputs(seed=3, batch=2, n_kv_heads=2, n_q_heads=8,
                                          seq_len=700, n_queries=96, device=dev)
    both, lse2 = ops.qk_features(q, k)
    one, lse1 = ops.qk_features(q[1:].contiguous(), k[1:].contiguous())
    ops.status()
    assert torch.equal(both[1], one[0])
    assert torch.equal(lse2[1], lse1[0])


# f32 caches: CUDA-core path with unrounded f32 logits.  Only the summation
# order differs from the oracle, so the continuous features agree to 1e-4
# relative (floored at 1e-3 absolute scale) and the discrete ones almost
# everywhere (a relation value within f32 rounding of 0 may flip).
F32_FEATURE_TOL = 1e-4
F32_LSE_TOL = 2e-6


def test_qk_features_f32_matches_golden():
    from core_b200 import ops
    dev = _dev()
    d, m = load_case("fp32_decode_L512_Q64")
    q = _f32(d["q"], dev)[None]
    k = _f32(d["k"], dev)[None]
    feats, lse = ops.qk_features(q, k)
    ops.status()
    ref, ref_lse, _ = O.qk_features(d["q"], d["k"], groups=m["hq"] // m["hkv"],
                                    round_bf16=False)
    got = feats[0].cpu().numpy()
    assert np.abs(lse[0].cpu().numpy() - ref_lse).max() <= F32_LSE_TOL * np.abs(ref_lse).max()
    assert rel_err(got[:, :4], ref[:, :4]).max() < F32_FEATURE_TOL
    assert rel_err(got[:, :4], d["features"][:, :4]).max() < F32_FEATURE_TOL
    nq, hkv = m["nq"], m["hkv"]
    f5_frac, f5_steps = _discrete_mismatch(got[:, 4], d["features"][:, 4], 1.0 / nq)
    f6_frac, f6_steps = _discrete_mismatch(got[:, 5], d["features"][:, 5], 1.0 / hkv)
    assert f5_frac <= 0.002 and f5_steps <= 1.01, (f5_frac, f5_steps)
    assert f6_frac <= 0.002 and f6_steps <= 1.01, (f6_frac, f6_steps)


def test_qk_features_f32_ragged_and_given_lse():
    """f32 path at a ragged length with several q-blocks, batch 2, group 4, and
    with the LSE supplied by the caller (the decode readout order)."""
    from core_b200 import ops
    dev = _dev()
    g = torch.Generator().manual_seed(21)
    B, hkv, hq, L, nq = 2, 2, 8, 1000, 200
    q = (torch.randn(B, hq, nq, 128, generator=g) * 0.5).to(dev)
    k = (torch.randn(B, hkv, L, 128, generator=g) * 0.5).to(dev)
    feats, lse = ops.qk_features(q, k)
    feats2, lse2 = ops.qk_features(q, k, lse=lse)
    ops.status()
    assert torch.equal(feats, feats2)
    for b in range(B):
        ref, ref_lse, _ = O.qk_features(q[b].cpu().numpy(), k[b].cpu().numpy(), groups=4,
                                        round_bf16=False)
        got = feats[b].cpu().numpy()
        assert np.abs(lse[b].cpu().numpy() - ref_lse).max() <= F32_LSE_TOL * np.abs(ref_lse).max()
        assert rel_err(got[:, :4], ref[:, :4]).max() < F32_FEATURE_TOL
        f5_frac, _ = _discrete_mismatch(got[:, 4], ref[:, 4], 1.0 / nq)
        f6_frac, _ = _discrete_mismatch(got[:, 5], ref[:, 5], 1.0 / hkv)
        assert f5_frac <= 0.002 and f6_frac <= 0.002, (f5_frac, f6_frac)


@pytest.mark.parametrize("name", BF16_CASES)
def test_coverage_matches_oracle(name):
    from core_b200 import ops
    dev = _dev()
    d, m = load_case(name)
    k = _bf16(d["k"], dev)[None]
    geo = ops.prepare_geometry(_f32(d["geometry"], dev), _f32(d["hadamard"], dev))
    cov = ops.coverage_features(k, geo, _f32(d["prototypes"], dev))
    ops.status()
    got = cov[0].cpu().numpy()
    ref = O.coverage_features(d["k"], d["geometry"], d["prototypes"], d["hadamard"])
    check_coverage(got, ref)


def check_coverage(got, ref, cos_err=2e-5):
    """d_proto and delta_proto are (differences of) cosines computed to f32
    accuracy: within FEATURE_TOL relative or ``cos_err`` absolute.  g within
    FEATURE_TOL.  Occupancy counts change only when some key's top two
    prototypes tie within ``cos_err`` (a reassignment moves two counts)."""
    err = rel_err(got[:, 1:3], ref[:, 1:3])
    absd = np.abs(got[:, 1:3] - ref[:, 1:3])
    assert np.all((err <= FEATURE_TOL) | (absd <= cos_err)), (err.max(0), absd.max(0))
    assert rel_err(got[:, 3], ref[:, 3]).max() <= FEATURE_TOL
    occ = np.abs(got[:, 0] - ref[:, 0]) > 1e-5
    assert occ.mean() <= 0.01, occ.mean()
    if occ.any():
        assert (ref[:, 2] <= cos_err).any(), "occupancy changed without a near tie"


@pytest.mark.parametrize("name", BF16_CASES)
def test_indexer_scores_match_oracle(name):
    from core_b200 import ops
    dev = _dev()
    d, m = load_case(name)
    L = m["L"]
    feats = torch.zeros(1, L, 14, device=dev)
    feats[0, :, :10] = _f32(d["features"][:, :10], dev)
    w = layer_weights(d)
    mlp = ops.pack_mlp([_f32(x, dev) for x in w.mlp])
    pos = torch.arange(L, device=dev)[None]
    scores = ops.indexer_scores(_bf16(d["v"], dev)[None], pos, feats, mlp, original_length=L,
                                is_prefill=bool(m["prefill"]), n_sink=4)
    ops.status()
    aux = O.auxiliary_features(d["v"], np.arange(L), seq_len=L, is_prefill=bool(m["prefill"]),
                               round_bf16=True)
    np.testing.assert_allclose(feats[0, :, 10:].cpu().numpy(), aux, rtol=1e-6, atol=1e-7)
    ref = O.indexer_mlp(d["features"], *w.mlp)
    np.testing.assert_allclose(scores[0].cpu().numpy(), ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(scores[0].cpu().numpy(), d["scores"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("L,n_kept,n_sink", [(5, 4, 4), (96, 48, 4), (333, 133, 4), (4096, 1024, 4),
                                             (16384, 4096, 4), (1000, 1000, 4), (300, 4, 4),
                                             (65536, 16384, 4), (2049, 700, 0), (8191, 3000, 4),
                                             (8192, 2000, 4), (8193, 8192, 4), (131072, 13107, 4),
                                             (131072, 4, 4), (100003, 99000, 0), (400000, 40000, 4)])
def test_topb_matches_stable_argsort(L, n_kept, n_sink):
    from core_b200 import ops
    dev = _dev()
    rng = np.random.default_rng(L)
    s = rng.standard_normal((2, L)).astype(np.float32)
    s[:, ::7] = np.round(s[:, ::7], 1)  # plenty of exact ties
    s[1, 10:20] = 0.0
    s[1, 20:22] = -0.0
    keep, evict = ops.topb_select(_f32(s, dev), n_kept, n_sink)
    ops.status()
    for b in range(2):
        ref = O.topb_select(s[b:b + 1], n_kept, n_sink)[0]
        assert np.array_equal(keep[b].cpu().numpy(), ref)
        ev = np.setdiff1d(np.arange(L), ref)
        assert np.array_equal(evict[b].cpu().numpy(), ev)


@pytest.mark.parametrize("L,n_kept", [(4096, 1000), (70000, 5000), (131072, 13107)])
def test_topb_all_equal_scores_keep_lowest_indices(L, n_kept):
    from core_b200 import ops
    dev = _dev()
    s = np.full((1, L), 0.25, np.float32)
    keep, evict = ops.topb_select(_f32(s, dev), n_kept, 4)
    ops.status()
    assert np.array_equal(keep[0].cpu().numpy(), np.arange(n_kept))
    assert np.array_equal(evict[0].cpu().numpy(), np.arange(n_kept, L))


@pytest.mark.parametrize("name", BF16_CASES + [TWO_STEP_CASE])
def test_memory_write_matches_reference(name):
    from core_b200 import engine, ops
    dev = _dev()
    d, m = load_case(name)
    scores = d["scores"] if "scores" in d else d["scores1"]
    keep = d["keep"] if "keep" in d else d["keep1"]
    L = m["L"]
    evict = np.setdiff1d(np.arange(L), keep)
    if evict.size == 0:
        pytest.skip("nothing evicted")
    hkv, hq, dm = m["hkv"], m["hq"], m["d_mem"]
    theta_f = engine.fold_groups(_f32(d["theta"], dev), hkv, hq // hkv, 128)
    ts = ops.split_bf16(theta_f, 2)
    M = torch.zeros(1, dm, hkv * 128, device=dev)
    b = torch.zeros(1, dm, device=dev)
    Z = torch.zeros(1, device=dev)
    ops.memory_write(_bf16(d["k"], dev)[None], _bf16(d["v"], dev)[None], _f32(scores, dev)[None],
                     torch.from_numpy(evict.astype(np.int32)).to(dev)[None], ts, M, b, Z,
                     gamma=0.9, eta=1.0, student_temp=1.0)
    ops.status()
    gM = d["M"] if "M" in d else d["M1"]
    gb = d["b"] if "b" in d else d["b1"]
    gZ = d["Z"] if "Z" in d else d["Z1"]
    tol = 2e-3
    assert np.abs(M[0].cpu().numpy() - gM).max() <= tol * np.abs(gM).max()
    assert np.abs(b[0].cpu().numpy() - gb).max() <= tol * np.abs(gb).max()
    assert abs(float(Z[0]) - float(gZ[0])) <= 1e-6


@pytest.mark.parametrize("d_mem,L,hkv", [(512, 1536, 8), (256, 1000, 8), (384, 700, 4),
                                         (256, 16384, 8), (128, 70001, 2)])
def test_memory_write_matches_oracle_wide_memory(d_mem, L, hkv):
    """Memory widths whose M_bar tiles pair up (d_mem a multiple of 256) and
    ones that do not; evicted counts that are not multiples of the tiles."""
    from core_b200 import engine, ops
    dev = _dev()
    hq = 4 * hkv
    rng = np.random.default_rng(d_mem + L)
    k = O.bf16_round(rng.standard_normal((hkv, L, 128), dtype=np.float32) / np.float32(np.sqrt(128)))
    v = O.bf16_round(rng.standard_normal((hkv, L, 128), dtype=np.float32))
    scores = (rng.standard_normal(L) * 0.05).astype(np.float32)
    theta = (rng.standard_normal((d_mem, hq * 128)) / np.sqrt(hq * 128)).astype(np.float32)
    n_kept = L // 4
    keep = O.topb_select(scores[None], n_kept, 4)[0]
    evict = np.setdiff1d(np.arange(L), keep)
    mask = np.zeros(L, bool)
    mask[evict] = True
    ref_M, ref_b, ref_Z = O.memory_write(k, v, scores, mask, theta, groups=4)
    ts = ops.split_bf16(engine.fold_groups(_f32(theta, dev), hkv, 4, 128), 2)
    M = torch.zeros(1, d_mem, hkv * 128, device=dev)
    b = torch.zeros(1, d_mem, device=dev)
    Z = torch.zeros(1, device=dev)
    ops.memory_write(_bf16(k, dev)[None], _bf16(v, dev)[None], _f32(scores, dev)[None],
                     torch.from_numpy(evict.astype(np.int32)).to(dev)[None], ts, M, b, Z,
                     gamma=0.9, eta=1.0, student_temp=1.0)
    ops.status()
    tol = 2e-3
    assert np.abs(M[0].cpu().numpy() - ref_M).max() <= tol * np.abs(ref_M).max()
    assert np.abs(b[0].cpu().numpy() - ref_b).max() <= tol * np.abs(ref_b).max()
    assert abs(float(Z[0]) - float(ref_Z)) <= 1e-6


def test_topb_cluster_rows_are_independent():
    """Three batch rows of a long cache (one cluster each) equal each row alone."""
    from core_b200 import ops
    dev = _dev()
    rng = np.random.default_rng(7)
    s = rng.standard_normal((3, 50000)).astype(np.float32)
    s[1, ::3] = 0.5
    keep, evict = ops.topb_select(_f32(s, dev), 9000, 4)
    for b in range(3):
        k1, e1 = ops.topb_select(_f32(s[b:b + 1], dev), 9000, 4)
        assert torch.equal(keep[b], k1[0]) and torch.equal(evict[b], e1[0])
        assert np.array_equal(keep[b].cpu().numpy(), O.topb_select(s[b:b + 1], 9000, 4)[0])
    ops.status()


def test_layer_step_indexer_equals_public_entry():
    """The fused layer step computes the value sums in a separate launch; its
    auxiliary features and scores equal core_indexer_scores' bit for bit."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L = 3000
    q, k, v = synthetic.make_layer_inputs(seed=17, batch=2, n_kv_heads=8, n_q_heads=32,
                                          seq_len=L, n_queries=64, device=dev)
    w = synthetic.make_layer_weights(seed=18, n_kv_heads=8, n_q_heads=32, d_mem=128)
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                     n_kv_heads=8, n_q_heads=32, device=dev)
    pos = torch.arange(L, device=dev)[None].expand(2, L).contiguous()
    out = engine.compress_layer(q, k, v, lw, n_kept=700, positions=pos, original_length=L + 5,
                                is_prefill=False)
    feats = out["features"].clone()
    feats[:, :, 10:] = 0
    scores = ops.indexer_scores(v, pos, feats, lw.mlp, original_length=L + 5, is_prefill=False)
    ops.status()
    assert torch.equal(feats, out["features"])
    assert torch.equal(scores, out["scores"])


def test_compact_kv_is_exact_gather():
    from core_b200 import ops, synthetic
    dev = _dev()
    _, k, v = synthetic.make_layer_inputs(seed=5, batch=2, n_kv_heads=8, n_q_heads=32,
                                          seq_len=1000, n_queries=8, device=dev)
    rng = np.random.default_rng(0)
    keep = np.stack([np.sort(rng.choice(1000, 250, replace=False)) for _ in range(2)]).astype(np.int32)
    kt = torch.from_numpy(keep).to(dev)
    ok, ov = ops.compact_kv(k, v, kt)
    idx = kt.long()[:, None, :, None].expand(-1, 8, -1, 128)
    assert torch.equal(ok, k.gather(2, idx))
    assert torch.equal(ov, v.gather(2, idx))


def test_memory_readout_matches_reference():
    from core_b200 import engine, ops
    dev = _dev()
    d, m = load_case(TWO_STEP_CASE)
    hkv, hq = m["hkv"], m["hq"]
    ofold = engine.fold_groups(_f32(d["o_proj"], dev), hkv, hq // hkv, 128)
    gate = (_f32(d["gate_w1"], dev), _f32(d["gate_b1"], dev), _f32(d["gate_w2"], dev).reshape(-1),
            _f32(d["gate_b2"], dev).reshape(-1))
    for ql in (1, 3):
        q = _bf16(d[f"readout_q{ql}"], dev)[None]
        attn = _bf16(d[f"readout_attn{ql}"], dev).contiguous()
        out = ops.memory_readout(q, _f32(d["theta"], dev), gate, _f32(d["M2"], dev)[None],
                                 _f32(d["b2"], dev)[None], ofold, attn, n_kv_heads=hkv)
        ops.status()
        ref = d[f"readout_out{ql}"][0]
        diff = np.abs(out[0].float().cpu().numpy() - ref)
        # bf16 output: equal up to one bf16 ulp of the residual sum on a few entries
        assert (diff > 0).mean() < 0.02 and diff.max() <= 2 ** -7 * np.abs(ref).max(), diff.max()


# (Hkv, Hq, d_mem, gate_hidden, hidden, q_len): one decode query at the
# benchmark's sizes and at sizes where most blocks hold no rows, the register
# kernels with 8 and 16 float4 a lane, ragged row slices and partial warps, and
# (Hq not a multiple of 4, d_mem above 1024, Hkv*d above 2048) the general kernels
READOUT_SHAPES = [(8, 32, 512, 64, 4096, 1), (1, 4, 20, 8, 40, 1), (16, 64, 700, 48, 96, 3),
                  (1, 4, 20, 8, 40, 5), (18, 18, 1100, 16, 64, 2)]


@pytest.mark.parametrize("shape", READOUT_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_memory_readout_shapes_match_oracle(shape, dtype):
    from core_b200 import ops
    dev = _dev()
    hkv, hq, d_mem, gh, hidden, ql = shape
    rng = np.random.default_rng(sum(shape))
    f = np.float32
    q = rng.standard_normal((ql, hq * 128)).astype(f)
    theta = (rng.standard_normal((d_mem, hq * 128)) / np.sqrt(hq * 128)).astype(f)
    w1 = (rng.standard_normal((gh, hq * 128)) / np.sqrt(hq * 128)).astype(f)
    b1 = (rng.standard_normal(gh) * 0.1).astype(f)
    w2 = (rng.standard_normal(gh) * 0.1).astype(f)
    b2 = f([0.2])
    M = rng.standard_normal((d_mem, hkv * 128)).astype(f)
    b = np.abs(rng.standard_normal(d_mem)).astype(f)
    ofold = (rng.standard_normal((hidden, hkv * 128)) / np.sqrt(hkv * 128)).astype(f)
    attn = rng.standard_normal((ql, hidden)).astype(f)
    bf = dtype == "bf16"
    if bf:  # the inputs the bf16 path sees
        q = O.bf16_round(q)
        attn = O.bf16_round(attn)
    ref = O.memory_readout(q, theta, w1, b1, w2[None], b2, M, b, ofold, attn, out_bf16=bf)
    cast = _bf16 if bf else _f32
    qt = cast(q, dev).reshape(ql, hq, 128).permute(1, 0, 2)[None].contiguous()
    out = cast(attn, dev)[None].contiguous()
    ops.memory_readout(qt, _f32(theta, dev), (_f32(w1, dev), _f32(b1, dev), _f32(w2, dev),
                                              _f32(b2, dev)),
                       _f32(M, dev)[None], _f32(b, dev)[None], _f32(ofold, dev), out,
                       n_kv_heads=hkv)
    ops.status()
    got = out[0].float().cpu().numpy()
    if bf:
        # equal up to one bf16 ulp of the residual or of the sum on a few entries
        diff = np.abs(got - ref)
        assert (diff > 0).mean() < 0.02 and diff.max() <= 2 ** -7 * np.abs(ref).max(), diff.max()
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", BF16_CASES)
def test_compress_layer_keep_set_matches_reference(name):
    from core_b200 import engine, ops
    dev = _dev()
    d, m = load_case(name)
    L = m["L"]
    w = layer_weights(d)
    lw = engine.LayerWeights.prepare(geometry=_f32(w.geometry, dev),
                                     prototypes=_f32(w.prototypes, dev),
                                     hadamard=_f32(w.hadamard, dev),
                                     mlp_params=[_f32(x, dev) for x in w.mlp],
                                     theta=_f32(w.theta, dev), n_kv_heads=m["hkv"],
                                     n_q_heads=m["hq"], device=dev)
    n_kept = engine.n_kept_for(L, m["ratio"], 4)
    out = engine.compress_layer(_bf16(d["q"], dev)[None], _bf16(d["k"], dev)[None],
                                _bf16(d["v"], dev)[None], lw, n_kept=n_kept,
                                positions=torch.arange(L, device=dev)[None], original_length=L,
                                is_prefill=bool(m["prefill"]))
    ops.status()
    got_scores = out["scores"][0].cpu().numpy()
    ref_scores = d["scores"]
    # every score within 2e-3, or (a counted few) explained by its own features,
    # which are checked against the reference's with the flip bound
    n_expl = check_scores_explained(got_scores, ref_scores, out["features"][0].cpu().numpy(),
                                    w.mlp)
    assert n_expl <= max(2, 0.01 * L), n_expl
    _, ref_lse, R = O.qk_features(d["q"], d["k"], groups=m["hq"] // m["hkv"], round_bf16=True)
    gf = out["features"][0].cpu().numpy()
    check_qk_features_bounded(gf[:, :6], d["features"][:, :6], R,
                              flip_bound(d["q"], d["k"], LSE_TOL * np.abs(ref_lse).max()))
    if n_kept >= L:
        return
    keep = out["keep"][0].cpu().numpy()
    gk = d["keep"]
    # bit-exact except keys within 1e-3 relative of the Top-B boundary score
    s = ref_scores.copy()
    s[:4] = s.max() + 1
    boundary = np.sort(s)[::-1][n_kept - 1]
    near = np.abs(s - boundary) <= 1e-3 * abs(boundary)
    diff = np.setxor1d(keep, gk)
    assert np.all(near[diff]), (diff, s[diff], boundary)


def test_compress_layers_concurrent_equals_sequential():
    """Layers on two streams with an SM budget give the same results as one
    layer after another under the same budget."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L, nq, hkv, hq = 2048, 64, 8, 32
    jobs_a, jobs_b = [], []
    for l in range(4):
        q, k, v = synthetic.make_layer_inputs(seed=100 + l, batch=1, n_kv_heads=hkv, n_q_heads=hq,
                                              seq_len=L, n_queries=nq, device=dev)
        w = synthetic.make_layer_weights(seed=200 + l, n_kv_heads=hkv, n_q_heads=hq, d_mem=128)
        lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                         hadamard=w["hadamard"], mlp_params=w["mlp"],
                                         theta=w["theta"], n_kv_heads=hkv, n_q_heads=hq, device=dev)
        pos = torch.arange(L, device=dev)[None]
        for jobs in (jobs_a, jobs_b):
            jobs.append(dict(q=q, keys=k, values=v, weights=lw, positions=pos,
                             memory=engine.MemoryState.zeros(1, 128, hkv * 128, dev)))
    n_kept = engine.n_kept_for(L, 0.75, 4)
    with ops.sm_budget(torch.cuda.get_device_properties(dev).multi_processor_count - 2):
        seq = [engine.compress_layer(**j, n_kept=n_kept, original_length=L, is_prefill=True)
               for j in jobs_a]
        par = engine.compress_layers(jobs_b, n_streams=2, n_kept=n_kept, original_length=L,
                                     is_prefill=True)
        torch.cuda.synchronize()
    ops.status()
    for a, b, ja, jb in zip(seq, par, jobs_a, jobs_b):
        assert torch.equal(a["keep"], b["keep"])
        assert torch.equal(a["scores"], b["scores"])
        assert torch.equal(a["keys"], b["keys"]) and torch.equal(a["values"], b["values"])
        assert torch.equal(ja["memory"].M, jb["memory"].M)


def test_repeated_calls_are_bitwise_deterministic():
    """Same inputs, fresh (uninitialised) workspaces, twenty repetitions: the
    coverage features and the fused layer step reproduce bit for bit."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L, nq, hkv, hq = 2048, 64, 8, 32
    q, k, v = synthetic.make_layer_inputs(seed=102, batch=1, n_kv_heads=hkv, n_q_heads=hq,
                                          seq_len=L, n_queries=nq, device=dev)
    w = synthetic.make_layer_weights(seed=202, n_kv_heads=hkv, n_q_heads=hq, d_mem=128)
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                     n_kv_heads=hkv, n_q_heads=hq, device=dev)
    ref = ops.coverage_features(k, lw.geometry_ext, lw.prototypes).clone()
    for _ in range(20):
        scratch = torch.randn(1 << 20, device=dev)  # leave different garbage behind
        del scratch
        assert torch.equal(ops.coverage_features(k, lw.geometry_ext, lw.prototypes), ref)
    pos = torch.arange(L, device=dev)[None]
    n_kept = engine.n_kept_for(L, 0.75, 4)
    outs = [engine.compress_layer(q, k, v, lw, n_kept=n_kept, positions=pos, original_length=L,
                                  is_prefill=True,
                                  memory=engine.MemoryState.zeros(1, 128, hkv * 128, dev))
            for _ in range(5)]
    ops.status()
    for o in outs[1:]:
        assert torch.equal(o["features"], outs[0]["features"])
        assert torch.equal(o["keep"], outs[0]["keep"])


def test_memory_readout_sees_writes_of_the_kernels_just_before_it():
    """The state and weights written by the kernels right before the call are
    the ones read: the result equals a readout on the same values made after a
    full synchronisation, bit for bit."""
    from core_b200 import ops
    dev = _dev()
    hkv, hq, d_mem, gh, hidden = 8, 32, 512, 64, 4096
    g = torch.Generator(device=dev).manual_seed(5)
    q = (torch.randn(1, hq, 1, 128, device=dev, generator=g)).to(torch.bfloat16)
    theta = torch.randn(d_mem, hq * 128, device=dev, generator=g) / 64
    gate = (torch.randn(gh, hq * 128, device=dev, generator=g) / 64,
            torch.randn(gh, device=dev, generator=g) * 0.1,
            torch.randn(gh, device=dev, generator=g) * 0.1, torch.full((1,), 0.2, device=dev))
    M = torch.randn(1, d_mem, hkv * 128, device=dev, generator=g)
    b = torch.rand(1, d_mem, device=dev, generator=g) + 0.5
    ofold = torch.randn(hidden, hkv * 128, device=dev, generator=g) / 32
    attn = torch.randn(1, 1, hidden, device=dev, generator=g).to(torch.bfloat16)

    def scaled():
        return theta * 1.5, M * 2.0, b * 3.0, ofold * 0.5, attn * 2

    th2, M2, b2, of2, at2 = scaled()
    torch.cuda.synchronize()
    want = ops.memory_readout(q, th2, gate, M2, b2, of2, at2.clone(), n_kv_heads=hkv)
    torch.cuda.synchronize()
    for _ in range(3):
        th, Mx, bx, of, at = theta.clone(), M.clone(), b.clone(), ofold.clone(), attn.clone()
        torch.cuda.synchronize()
        # each in-place scale is a kernel of the same stream, the last right before the call
        th.mul_(1.5)
        Mx.mul_(2.0)
        bx.mul_(3.0)
        at.mul_(2)
        of.mul_(0.5)
        got = ops.memory_readout(q, th, gate, Mx, bx, of, at, n_kv_heads=hkv)
        ops.status()
        assert torch.equal(got, want)



def test_compress_layer_headline_shape():
    """One layer at the benchmark's shape (bf16, 8 KV / 32 query heads,
    L = 16384, 128 scoring queries in the prefill's question scope,
    r = 0.75, d_mem = 512) through the fused layer step, against the
    oracle: keep set (boundary band only), every score, the features, the
    retained K/V bit for bit and the memory state."""
    from core_b200 import engine, ops, synthetic
    dev = _dev()
    L, nq, hkv, hq, dm = 16384, 128, 8, 32, 512
    q, k, v = synthetic.make_layer_inputs(seed=31, batch=1, n_kv_heads=hkv, n_q_heads=hq,
                                          seq_len=L, n_queries=nq, device=dev)
    w = synthetic.make_layer_weights(seed=32, n_kv_heads=hkv, n_q_heads=hq, d_mem=dm)
    lw = engine.LayerWeights.prepare(geometry=w["geometry"], prototypes=w["prototypes"],
                                     hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                     n_kv_heads=hkv, n_q_heads=hq, device=dev)
    mem = engine.MemoryState.zeros(1, dm, hkv * 128, dev)
    n_kept = engine.n_kept_for(L, 0.75, 4)
    out = engine.compress_layer(q, k, v, lw, n_kept=n_kept, positions=torch.arange(L, device=dev)[None],
                                original_length=L, is_prefill=True, memory=mem)
    ops.status()
    qn, kn, vn = (t[0].float().cpu().numpy() for t in (q, k, v))
    ow = O.LayerWeights(mlp=tuple(t.numpy() for t in w["mlp"]), geometry=w["geometry"].numpy(),
                        prototypes=w["prototypes"].numpy(), hadamard=w["hadamard"].numpy(),
                        theta=w["theta"].numpy())
    ref = O.compress_layer(qn, kn, vn, ow, compression_ratio=0.75, is_prefill=True,
                           round_bf16=True)
    gf = out["features"][0].cpu().numpy()
    _, ref_lse, R = O.qk_features(qn, kn, groups=4, round_bf16=True)
    n_qk = check_qk_features_bounded(gf[:, :6], ref["features"][:, :6], R,
                                     flip_bound(qn, kn, LSE_TOL * np.abs(ref_lse).max()))
    check_coverage(gf[:, 6:10], ref["features"][:, 6:10])
    np.testing.assert_allclose(gf[:, 10:], ref["features"][:, 10:], rtol=1e-6, atol=1e-7)
    gs = out["scores"][0].cpu().numpy()
    n_sc = check_scores_explained(gs, ref["scores"], gf, ow.mlp)
    assert n_sc <= 0.01 * L, (n_qk, n_sc)
    keep = out["keep"][0].cpu().numpy()
    s = ref["scores"].astype(np.float64).copy()
    s[:4] = s.max() + 1
    boundary = np.sort(s)[::-1][n_kept - 1]
    near = np.abs(s - boundary) <= 1e-3 * abs(boundary)
    diff = np.setxor1d(keep, ref["keep"])
    assert np.all(near[diff]), (diff, boundary)
    idx = out["keep"].long()[:, None, :, None].expand(-1, hkv, -1, 128)
    assert torch.equal(out["keys"], k.gather(2, idx)) and torch.equal(out["values"], v.gather(2, idx))
    # the memory write of the evicted set this path chose (the reference's
    # unless a boundary key flipped)
    M_ref, b_ref, Z_ref = ref["M"], ref["b"], ref["Z"]
    if diff.size:
        evict = np.ones(L, bool)
        evict[keep] = False
        M_ref, b_ref, Z_ref = O.memory_write(kn, vn, ref["scores"], evict, ow.theta, groups=4)
    for got, want in ((mem.M[0], M_ref), (mem.b[0], b_ref)):
        g = got.cpu().numpy()
        assert np.abs(g - want).max() <= 2e-3 * np.abs(want).max()
    assert abs(float(mem.Z[0]) - float(Z_ref)) <= 1e-6
