"""Fixture loading shared by the tests."""

from __future__ import annotations

import ast
import os

import numpy as np

from oracle import core_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

SINGLE_STEP_CASES = [
    "fp32_decode_L512_Q64",
    "bf16_prefillq_L640_Q128",
    "bf16_decode_ragged_L333_Q40",
    "bf16_prefill_all_L96",
    "bf16_tiny_L5",
    "bf16_llama_heads_L256_Q32",
]
TWO_STEP_CASE = "bf16_two_step_L384_Q64"


def load_case(name: str):
    """Return (arrays, meta); bf16 arrays stored as uint16 bits come back as float32."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        d = {k: z[k] for k in z.files}
    meta = ast.literal_eval(str(d.pop("meta")))
    for k, v in list(d.items()):
        if v.dtype == np.uint16:
            d[k] = O.bits_to_f32(v)
    return d, meta


def layer_weights(d) -> O.LayerWeights:
    return O.LayerWeights(
        mlp=tuple(d[x] for x in ("mlp_w1", "mlp_b1", "mlp_w2", "mlp_b2", "mlp_w3", "mlp_b3")),
        geometry=d["geometry"], prototypes=d["prototypes"], hadamard=d["hadamard"],
        theta=d["theta"])


def rel_err(a, b, floor=1e-3):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b) / np.maximum(np.abs(b), floor)


def f3_flip_consistent(got_f3, R, bad_keys, *, rtol, near=2e-3):
    """f3 is the mean of the positive relation values of a key.  A relation
    value within rounding of 0 can take either sign in another summation order
    (one bf16 ulp of a logit moves it by up to ~1e-3; in f32 far less), which
    moves the count by one and the sum by about nothing.  Accept a key whose f3
    equals psum / (pcnt + j) for j within the number of values with
    |R| <= ``near``.  Returns (ok, first failing key)."""
    nkv, nq, L = R.shape
    flat = R.reshape(nkv * nq, L).astype(np.float64)
    for k in bad_keys:
        col = flat[:, k]
        pos = col > 0
        psum, pcnt = col[pos].sum(), int(pos.sum())
        close = np.abs(col) <= near
        n_minus, n_plus = int((close & pos).sum()), int((close & ~pos & np.isfinite(col)).sum())
        cands = [psum / max(pcnt + j, 1) for j in range(-n_minus, n_plus + 1)]
        tol = rtol * max(abs(psum / max(pcnt, 1)), 1e-3)
        if min(abs(got_f3[k] - c) for c in cands) > tol:
            return False, k
    return True, None


HOOK_CASE = "bf16_hook_decode_L256"


def hook_rotary(meta, device="cpu"):
    """The Llama-3.1 rotary embedding the hook fixture was written with."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = LlamaConfig(hidden_size=meta["hidden"], num_attention_heads=meta["hq"],
                      num_key_value_heads=meta["hkv"], head_dim=meta["d"],
                      max_position_embeddings=131072, rope_parameters=dict(meta["rope"]))
    return LlamaRotaryEmbedding(cfg).to(device)


def hook_decode_steps(d):
    """Per decode forward: (first token index into the decode_* arrays, n tokens)."""
    starts = np.concatenate([[0], np.cumsum(d["decode_tokens"])[:-1]])
    return list(zip(starts.tolist(), d["decode_tokens"].tolist()))


def hook_events(d, meta):
    """Per compression, in order: (layer, keep indices, calibrated scores).
    Every compression of the case keeps the prefill budget, meta["target"]."""
    out, off_s = [], 0
    n = int(meta["target"])
    for i, (layer, ln) in enumerate(zip(d["event_layer"].tolist(), d["event_len"].tolist())):
        out.append((int(layer), d["event_keep"][i * n:(i + 1) * n], d["event_scores"][off_s:off_s + ln]))
        off_s += ln
    return out


def flip_bound(q, k, lse_err: float) -> float:
    """Largest change of any relation value that one-bf16-ulp changes of the
    logits can cause, plus the LSE difference.

    A logit is an f32 dot product rounded to bf16; another summation order can
    land on the neighbouring bf16 value, 1 ulp <= 2^-7 |logit| away, and
    |logit| <= |q| |k|.  The relation r = scale * logit - lse + log|C| (and
    its logaddexp with the floor, a 1-Lipschitz map) moves by at most
    scale * 2^-7 * max|q| max|k| + |delta lse|; the head mean, maxima and
    top-k means of such values move by no more."""
    qn = np.sqrt((np.asarray(q, np.float64) ** 2).sum(-1)).max()
    kn = np.sqrt((np.asarray(k, np.float64) ** 2).sum(-1)).max()
    d = np.asarray(q).shape[-1]
    return float(d ** -0.5 * 2.0 ** -7 * qn * kn + lse_err)


def check_qk_features_bounded(got, ref, R, bound, *, rtol=2e-3, max_frac=0.01):
    """f1..f6 of the CUDA path against the oracle's, every key within ``rtol``
    relative (floored at 1e-3) or, for at most ``max_frac`` of the keys,
    within what logit flips of size ``bound`` can explain:
      f1, f2, f4 : |delta| <= bound;
      f3         : psum / (pcnt + j), j within the number of values |R| <= bound;
      f5         : |delta| * nq <= queries whose head maximum |max_h R| <= bound;
      f6         : |delta| * Hkv <= heads whose top-quarter mean is within bound of 0.
    Returns the number of keys that needed the explanation."""
    nkv, nq, L = R.shape
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = rel_err(got[:, :4], ref[:, :4])
    missing = set()
    for col in (0, 1, 3):
        bad = np.nonzero(err[:, col] > rtol)[0]
        assert np.all(np.abs(got[bad, col] - ref[bad, col]) <= bound), (col, bad[:5])
        missing.update(bad.tolist())
    bad3 = np.nonzero(err[:, 2] > rtol)[0]
    ok, k = f3_flip_consistent(got[:, 2].astype(np.float32), R, bad3, rtol=rtol, near=bound)
    assert ok, ("f3", k, got[k, 2], ref[k, 2])
    missing.update(bad3.tolist())
    d5 = np.nonzero(np.abs(got[:, 4] - ref[:, 4]) > 1e-6)[0]
    if d5.size:
        amb = (np.abs(R.max(axis=0)[:, d5]) <= bound).sum(axis=0)
        assert np.all(np.rint(np.abs(got[d5, 4] - ref[d5, 4]) * nq) <= amb), ("f5", d5[:5])
        missing.update(d5.tolist())
    d6 = np.nonzero(np.abs(got[:, 5] - ref[:, 5]) > 1e-6)[0]
    if d6.size:
        q_start = max(0, L - nq)
        valid = np.clip(nq - np.maximum(d6 - q_start, 0), 1, nq)
        kf = np.maximum(np.ceil(valid * 0.25).astype(np.int64), 1)
        amb = np.zeros(d6.size, np.int64)
        for h in range(nkv):
            top = -np.sort(-R[h][:, d6], axis=0)
            means = np.array([top[:kf[i], i].mean() for i in range(d6.size)])
            amb += np.abs(means) <= bound
        assert np.all(np.rint(np.abs(got[d6, 5] - ref[d6, 5]) * nkv) <= amb), ("f6", d6[:5])
        missing.update(d6.tolist())
    assert len(missing) <= max(2, max_frac * L), len(missing)
    return len(missing)


def check_scores_explained(got_scores, ref_scores, got_feats, mlp, *, rtol=2e-3):
    """Scores within ``rtol`` relative (floored at 1e-3) of the reference's;
    a key outside it must be one whose own features, through the oracle's
    MLP, give our score (so that the difference is the features', which the
    feature checks bound).  Returns the number of such keys."""
    from oracle import core_oracle as O
    err = rel_err(got_scores, ref_scores)
    bad = np.nonzero(err > rtol)[0]
    if bad.size:
        again = O.indexer_mlp(np.asarray(got_feats)[bad], *mlp)
        np.testing.assert_allclose(np.asarray(got_scores)[bad], again, rtol=1e-5, atol=1e-6)
    return int(bad.size)
