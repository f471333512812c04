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
