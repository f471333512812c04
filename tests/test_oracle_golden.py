"""Pin the numpy oracle to the reference: every golden fixture was produced by
the reference press itself (tests/golden/make_golden.py)."""

import numpy as np
import pytest

from helpers import SINGLE_STEP_CASES, TWO_STEP_CASE, layer_weights, load_case, rel_err
from oracle import core_oracle as O

# Continuous features: relative error (floored at 1e-3 absolute scale).
FEATURE_TOL = 5e-4
# Discrete features (f5, f6, occupancy, sink, phase; a_value too when it is
# computed in bfloat16) take the same discrete value; occupancy is log1p(count)
# and may differ by one float32 ulp between libm implementations.
def discrete_cols(dtype):
    return [4, 5, 6, 11, 12, 13] if dtype == "bfloat16" else [4, 5, 6, 11, 13]


@pytest.mark.parametrize("name", SINGLE_STEP_CASES)
def test_compress_layer_matches_reference(name):
    d, m = load_case(name)
    out = O.compress_layer(d["q"], d["k"], d["v"], layer_weights(d),
                           compression_ratio=m["ratio"], is_prefill=bool(m["prefill"]),
                           round_bf16=m["dtype"] == "bfloat16")
    f, g = out["features"], d["features"]
    assert f.shape == g.shape
    cols = discrete_cols(m["dtype"])
    np.testing.assert_allclose(f[:, cols], g[:, cols], rtol=2.5e-7, atol=0)
    assert rel_err(f, g).max() < FEATURE_TOL
    assert np.abs(out["scores"] - d["scores"]).max() < 1e-6
    assert np.array_equal(out["keep"], d["keep"])
    assert np.array_equal(out["out_k"], d["out_k"]) and np.array_equal(out["out_v"], d["out_v"])
    tol = 1e-5
    assert np.abs(out["M"] - d["M"]).max() <= tol * np.abs(d["M"]).max()
    assert np.abs(out["b"] - d["b"]).max() <= tol * np.abs(d["b"]).max()
    assert abs(float(out["Z"]) - float(d["Z"][0])) <= 1e-6


def test_two_step_recurrence_and_readout_match_reference():
    d, m = load_case(TWO_STEP_CASE)
    w = layer_weights(d)
    o1 = O.compress_layer(d["q"], d["k"], d["v"], w, compression_ratio=m["ratio"],
                          is_prefill=True, round_bf16=True)
    assert np.array_equal(o1["keep"], d["keep1"])
    k = np.concatenate([o1["out_k"], d["k_new"]], axis=1)
    v = np.concatenate([o1["out_v"], d["v_new"]], axis=1)
    pos = np.concatenate([o1["keep"], m["L"] + np.arange(m["nq"])])
    ratio = O.find_target_compression_ratio(k.shape[1], m["target"])
    o2 = O.compress_layer(d["q1"], k, v, w, compression_ratio=ratio, is_prefill=False,
                          positions=pos, seq_len=m["L"] + m["nq"], round_bf16=True,
                          memory=(o1["M"], o1["b"], o1["Z"]))
    assert np.array_equal(o2["keep"], d["keep2"])
    assert rel_err(o2["features"], d["features2"]).max() < FEATURE_TOL
    assert np.abs(o2["M"] - d["M2"]).max() <= 1e-5 * np.abs(d["M2"]).max()
    assert abs(float(o2["Z"]) - float(d["Z2"][0])) <= 1e-6
    of = O.fold_groups(d["o_proj"], m["hkv"], m["hq"] // m["hkv"], m["d"])
    for ql in (1, 3):
        q = d[f"readout_q{ql}"].transpose(1, 0, 2).reshape(ql, m["hq"] * m["d"])
        out = O.memory_readout(q, d["theta"], d["gate_w1"], d["gate_b1"], d["gate_w2"],
                               d["gate_b2"], o2["M"], o2["b"], of, d[f"readout_attn{ql}"][0])
        assert np.array_equal(out, d[f"readout_out{ql}"][0])


def test_noop_when_budget_covers_cache():
    """n_kept >= L returns the cache unchanged (kvpress_adapter.py:1012-1013)."""
    assert O.n_kept_for(4, 0.75, 4) == 4
    assert O.n_kept_for(5, 0.75, 4) == 4
    assert O.n_kept_for(16384, 0.75, 4) == 4096
    assert O.n_kept_for(333, 0.6, 4) == 133


def test_target_ratio_search_hits_target():
    for L, t in [(4224, 4096), (8320, 8192), (256, 192), (1000, 999), (17, 4)]:
        r = O.find_target_compression_ratio(L, t)
        assert int(L * (1 - r)) == t


def test_topb_is_stable_and_forces_sinks():
    s = np.array([[0.5, 0.1, 0.1, 0.1, 0.9, 0.5, 0.5, 0.2]], np.float32)
    keep = O.topb_select(s, 6, 4)
    # sinks 0..3 saturated; ties at 0.5 broken toward lower index (stable sort)
    assert keep.tolist() == [[0, 1, 2, 3, 4, 5]]
