"""CPU oracle for the CORE KV-compression step.  TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithm of the ``core_full``
press compression step and memory readout, one function per reference
function, each citing the reference file:line it follows (paths relative to
the reference project root).  It is the checker for the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline and
its ``--impl reference`` arm) may import it.  The product package
``core_b200`` never imports it and has no CPU fallback.

Parity pin: ``tests/test_oracle_golden.py`` checks every function here
against ``tests/golden/*.npz``, which ``tests/golden/make_golden.py``
produced by running the reference's own press code on CPU.

Numerics.  Where the reference accumulates in float32 in an order that its
libraries choose (BLAS, torch reductions), the oracle accumulates in float64
and rounds to float32 where the reference materialises a float32 tensor.
Where the reference rounds to bfloat16 (QK logits, ``fused_qk.py:83-87``;
``a_value``, ``features.py:914-915``) the oracle rounds the same way
(round-to-nearest-even).
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

try:  # exact erf for the GELU of the indexer MLP and the memory gate
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover
    _erf = np.vectorize(math.erf)

LOG_FLOOR = np.float32(math.log(1e-8))  # fused_qk.py:382


# ----------------------------------------------------------------------------
# bfloat16 helpers
# ----------------------------------------------------------------------------

def bf16_round(x) -> np.ndarray:
    """Round float32 values to bfloat16 precision (nearest-even), as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def bf16_bits(x) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (r >> np.uint32(16)).astype(np.uint16)


def bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _f32(x):
    return np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------
# QK relation features f1..f6
# ----------------------------------------------------------------------------

def _logits(qh: np.ndarray, kh: np.ndarray, round_bf16: bool) -> np.ndarray:
    """float32 dot products (BLAS), rounded to bf16 when the inputs are bf16
    (``fused_qk.py:82-87``)."""
    x = np.matmul(qh.astype(np.float32), kh.astype(np.float32).T)
    return bf16_round(x) if round_bf16 else x


def _causal_setup(seq_q: int, seq_k: int):
    q_start = max(0, seq_k - seq_q)
    key_pos = np.arange(seq_k)
    q_pos = q_start + np.arange(seq_q)
    return q_start, key_pos, q_pos, key_pos[None, :] <= q_pos[:, None]


def _lse_rows(x: np.ndarray, visible: np.ndarray) -> np.ndarray:
    """Row log-sum-exp over the visible entries, accumulated in float64."""
    xm = np.where(visible, x, -np.inf)
    m = xm.max(axis=1)
    s = np.exp((xm - m[:, None]).astype(np.float64)).sum(axis=1)
    return (m + np.log(s)).astype(np.float32)


def causal_lse(q: np.ndarray, k: np.ndarray, *, groups: int, round_bf16: bool) -> np.ndarray:
    """Causal row log-sum-exp of ``scale * round(q . k)``.

    Follows ``core/fused_qk.py:26-107`` (``_causal_row_lse_kernel``): logits
    are rounded to the input dtype before the scale (``:82-87``), query t sits
    at absolute position ``q_start + t`` with ``q_start = max(0, K - Q)``
    (``:414``), and key i is visible to query t when ``i <= q_start + t``.
    Returns (Hq, Q) float32.
    """
    nq, seq_q, d = q.shape
    _, _, _, visible = _causal_setup(seq_q, k.shape[1])
    scale = np.float32(d ** -0.5)
    out = np.empty((nq, seq_q), np.float32)
    for h in range(nq):
        out[h] = _lse_rows(_logits(q[h], k[h // groups], round_bf16) * scale, visible)
    return out


def grouped_relation(q, k, lse, *, groups: int, topk_qk: int, round_bf16: bool) -> np.ndarray:
    """GQA-reduced attention advantage R, shape (Hkv, Q, K) float32.

    ``core/fused_qk.py:110-230`` (``_grouped_relation_tile_kernel``):
    ``r = scale*logit - lse + log|C_t|`` (``:189-193``), clamped with
    ``logaddexp(r, log 1e-8)`` written as ``max + log1p(exp(-|r - f|))``
    (``:200-202``), exactly ``log1p(exp(f))`` when a query sees one key
    (``:206-210``), invisible entries at the floor (``:465-470``), the group
    sum accumulated head by head in order (``:168-213``), minus the group
    minimum for leave-one-out TopMean (``:217-218``), divided by
    ``min(topk_qk, groups)`` (``:219``, ``:496``).  When ``lse`` is None it is
    computed from the same logits (``causal_lse``).  Returns (R, lse).
    """
    nq, seq_q, d = q.shape
    nkv, seq_k, _ = k.shape
    _, key_pos, q_pos, visible = _causal_setup(seq_q, seq_k)
    scale = np.float32(d ** -0.5)
    head_topk = min(topk_qk, groups)
    cc = np.minimum(q_pos + 1, seq_k).astype(np.float32)
    log_cc = np.log(cc).astype(np.float32)
    single = (cc == 1)[:, None] & visible
    single_val = np.float32(np.log1p(np.exp(np.float64(LOG_FLOOR))))
    own_lse = lse is None
    if own_lse:
        lse = np.empty((nq, seq_q), np.float32)
    R = np.empty((nkv, seq_q, seq_k), np.float32)

    def head(h):
        acc = np.zeros((seq_q, seq_k), np.float32)
        mn = np.full((seq_q, seq_k), np.inf, np.float32) if head_topk < groups else None
        for g in range(groups):
            qh = h * groups + g
            x = _logits(q[qh], k[h], round_bf16) * scale
            if own_lse:
                lse[qh] = _lse_rows(x, visible)
            r = (x - lse[qh][:, None]) + log_cc[:, None]
            rel = np.maximum(r, LOG_FLOOR) + np.log1p(np.exp(-np.abs(r - LOG_FLOOR)))
            rel = np.where(visible, rel, LOG_FLOOR)
            rel = np.where(single, single_val, rel).astype(np.float32)
            acc += rel
            if mn is not None:
                np.minimum(mn, rel, out=mn)
        if mn is not None:
            acc -= mn
        R[h] = acc / np.float32(head_topk)

    # KV heads are independent; numpy releases the GIL inside these array ops
    with ThreadPoolExecutor(max_workers=min(nkv, os.cpu_count() or 1)) as pool:
        list(pool.map(head, range(nkv)))
    return R, lse


def _topk_mean(vals: np.ndarray, k_per: np.ndarray, k_max: int) -> np.ndarray:
    """Mean of the k_per[i] largest of vals[:, i] (sorted-descending cumsum)."""
    n = vals.shape[0]
    top = -np.sort(-np.partition(vals, n - k_max, axis=0)[n - k_max:], axis=0)
    csum = np.cumsum(top, axis=0, dtype=np.float32)
    idx = (k_per - 1)[None, :]
    return (np.take_along_axis(csum, idx, axis=0)[0] / k_per.astype(np.float32)).astype(np.float32)


def qk_features_from_relation(R: np.ndarray, *, seq_k: int, topk_qk: int,
                              n_recent_queries: int) -> np.ndarray:
    """Six per-key statistics of R (Hkv, Q, K) -> (K, 6) float32.

    ``core/fused_qk.py:505-582``: f1 max over (head, query); f2 mean of the
    top-k2 with ``k2 = clamp(valid*Hkv, 1, min(topk, Q*Hkv))``; f3 mean of the
    positive entries (``:233-292``); f4 the f2 statistic over the last
    ``n_recent`` queries; f5 fraction of queries whose max over KV heads is
    positive; f6 fraction of KV heads whose mean of the top
    ``ceil(0.25*valid)`` queries is positive.
    """
    nkv, seq_q, _ = R.shape
    q_start = max(0, seq_k - seq_q)
    key_pos = np.arange(seq_k)
    valid = np.clip(seq_q - np.maximum(key_pos - q_start, 0), 1, seq_q)
    flat = R.reshape(nkv * seq_q, seq_k)
    f1 = flat.max(axis=0)
    k2_max = min(topk_qk, seq_q * nkv)
    k2 = np.clip(valid * nkv, 1, k2_max)
    f2 = _topk_mean(flat, k2, k2_max)
    pos = flat > 0
    psum = np.where(pos, flat, 0).astype(np.float64).sum(axis=0)
    pcnt = pos.sum(axis=0)
    f3 = (psum / np.maximum(pcnt, 1)).astype(np.float32)
    n_recent = min(n_recent_queries, seq_q)
    recent = R[:, seq_q - n_recent:, :].reshape(nkv * n_recent, seq_k)
    recent_start = q_start + seq_q - n_recent
    recent_valid = np.clip(q_start + seq_q - np.maximum(key_pos, recent_start), 1, n_recent)
    k4_max = min(topk_qk, n_recent * nkv)
    k4 = np.clip(recent_valid * nkv, 1, k4_max)
    f4 = _topk_mean(recent, k4, k4_max)
    f5 = ((R.max(axis=0) > 0).sum(axis=0) / np.float32(seq_q)).astype(np.float32)
    k_frac = np.maximum(np.ceil(valid.astype(np.float32) * np.float32(0.25)).astype(np.int64), 1)
    kf_max = int(k_frac.max())
    f6 = np.zeros(seq_k, np.float32)
    for h in range(nkv):
        m = _topk_mean(R[h], k_frac, kf_max)
        f6 += (m > 0).astype(np.float32)
    f6 = (f6 / np.float32(nkv)).astype(np.float32)
    return np.stack([f1, f2, f3, f4, f5, f6], axis=-1).astype(np.float32)


def qk_features(q, k, *, groups: int, topk_qk: int = 4, n_recent_queries: int = 16,
                round_bf16: bool, lse: np.ndarray | None = None):
    """``strict_causal_qk_features`` (``core/fused_qk.py:373-587``).

    Returns (features (K, 6), lse (Hq, Q), R (Hkv, Q, K)).
    """
    q = _f32(q)
    k = _f32(k)
    R, lse = grouped_relation(q, k, lse, groups=groups, topk_qk=topk_qk, round_bf16=round_bf16)
    feats = qk_features_from_relation(R, seq_k=k.shape[1], topk_qk=topk_qk,
                                      n_recent_queries=n_recent_queries)
    return feats, lse, R


# ----------------------------------------------------------------------------
# Coverage features (o, d_proto, delta_proto, g)
# ----------------------------------------------------------------------------

def _norm(x, axis=-1):
    return np.sqrt(np.sum(x.astype(np.float64) ** 2, axis=axis, keepdims=True)).astype(np.float32)


def project_keys(k: np.ndarray, geometry: np.ndarray, eps: float = 1e-8) -> np.ndarray:
    """``LayerwiseKeyGeometryProjector.forward`` (``core/features.py:53-77``).

    Per-head L2 normalisation, head concatenation, fixed Gaussian projection
    and a final L2 normalisation.  Returns (K, P) float32.
    """
    k = _f32(k)
    nkv, n, d = k.shape
    per_head = (k / (_norm(k) + np.float32(eps))).astype(np.float32)
    kbar = per_head.transpose(1, 0, 2).reshape(n, nkv * d)
    z = (kbar.astype(np.float64) @ geometry.astype(np.float64).T).astype(np.float32)
    return (z / (_norm(z) + np.float32(eps))).astype(np.float32)


def coverage_features(k, geometry, prototypes, hadamard, *, rho: float = 0.1,
                      eps: float = 1e-8, return_parts: bool = False):
    """``COREFeatureExtractor.compute_coverage_features`` (``core/features.py:790-858``)
    with ``PrototypeBank.get_coverage_features`` (``:146-213``) and
    ``HadamardProjector.rotate`` (``:259-261``).  Returns (K, 4) float32.
    """
    z = project_keys(k, geometry, eps)
    n = z.shape[0]
    mean_z = z.astype(np.float64).mean(axis=0).astype(np.float32)
    zc = (z - mean_z[None, :]).astype(np.float32)                      # :812
    cn = _norm(zc)[:, 0]
    reliable = cn > np.float32(1e-6)                                   # :816
    zp = (zc / np.maximum(cn, np.float32(1e-6))[:, None]).astype(np.float32)
    cos = (zp.astype(np.float64) @ prototypes.astype(np.float64).T).astype(np.float32)
    m1 = cos.argmax(axis=1)                                            # :177 first max
    cos1 = cos[np.arange(n), m1]
    cos_c = cos.copy()
    cos_c[np.arange(n), m1] = np.float32(-1e9)                          # :181-183
    cos2 = cos_c.max(axis=1)
    counts = np.bincount(m1[reliable], minlength=prototypes.shape[0])  # :198-199
    o = np.log1p(counts[m1].astype(np.float32)).astype(np.float32)     # :202
    dproto = (np.float32(1.0) - cos1).astype(np.float32)
    delta = (cos1 - cos2).astype(np.float32)
    o = np.where(reliable, o, np.float32(0))                           # :207-211
    dproto = np.where(reliable, dproto, np.float32(1))
    delta = np.where(reliable, delta, np.float32(0))
    zt = (z.astype(np.float64) @ hadamard.astype(np.float64).T).astype(np.float32)  # :261
    mu = zt.astype(np.float64).mean(axis=0)
    ez2 = (zt.astype(np.float64) ** 2).mean(axis=0)
    sigma2 = np.maximum(ez2 - mu ** 2, 0.0).astype(np.float32)        # :840
    mu = mu.astype(np.float32)
    avg = np.float32(sigma2.astype(np.float64).mean())
    sig_eff = ((np.float32(1 - rho) * sigma2 + np.float32(rho) * avg) + np.float32(1e-8)).astype(np.float32)
    dev = ((zt - mu[None, :]) ** 2).astype(np.float32)
    g = np.log1p((dev.astype(np.float64) / sig_eff[None, :]).mean(axis=1)).astype(np.float32)
    feats = np.stack([o, dproto, delta, g], axis=-1).astype(np.float32)
    if return_parts:
        return feats, dict(z=z, m1=m1, counts=counts, reliable=reliable, mu=mu,
                           sigma2_eff=sig_eff, mean_z=mean_z)
    return feats


# ----------------------------------------------------------------------------
# Auxiliary features (age, sink, value energy, phase)
# ----------------------------------------------------------------------------

def auxiliary_features(v, positions, *, seq_len: int, is_prefill: bool, n_sink: int = 4,
                       token_ids=None, special_token_ids=(), round_bf16: bool):
    """``COREFeatureExtractor.compute_auxiliary_features`` (``core/features.py:861-921``).

    ``a_value`` follows the bfloat16 arithmetic of the reference when the
    inputs are bfloat16: squares, the per-head sum, the mean over heads, the
    division by d and the log1p are each rounded to bfloat16 (``:914-915``).
    """
    v = _f32(v)
    nkv, n, d = v.shape
    pos = np.asarray(positions, dtype=np.int64)
    if pos.shape != (n,) or (pos < 0).any() or (pos >= seq_len).any():
        raise ValueError("token positions must lie in [0, seq_len) and match the KV axis")
    denom = np.float32(np.log1p(np.float32(max(seq_len - 1, 1))))
    a_age = (np.log1p((seq_len - 1 - pos).astype(np.float32)) / denom).astype(np.float32)
    sink = pos < n_sink
    if token_ids is not None and len(special_token_ids):
        ids = np.asarray(token_ids).reshape(-1)[:n]
        if ids.size < n:
            ids = np.pad(ids, (0, n - ids.size), constant_values=-1)
        for sid in special_token_ids:
            sink |= ids == int(sid)
    a_sink = sink.astype(np.float32)
    if round_bf16:
        sq = bf16_round(v * v)
        s = bf16_round(sq.astype(np.float64).sum(axis=-1).astype(np.float32))
        m = bf16_round((s.astype(np.float64).sum(axis=0) / nkv).astype(np.float32))
        m = bf16_round(m / np.float32(d))
        a_value = bf16_round(np.log1p(m.astype(np.float64)).astype(np.float32))
    else:
        s = (v.astype(np.float64) ** 2).sum(axis=-1).astype(np.float32)
        m = (s.astype(np.float64).sum(axis=0) / nkv).astype(np.float32)
        a_value = np.log1p(m / np.float32(d)).astype(np.float32)
    a_phase = np.full(n, 0.0 if is_prefill else 1.0, np.float32)
    return np.stack([a_age, a_sink, a_value, a_phase], axis=-1).astype(np.float32)


# ----------------------------------------------------------------------------
# Indexer MLP
# ----------------------------------------------------------------------------

def gelu(x):
    """Exact (erf) GELU, ``torch.nn.GELU()`` default."""
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))


def indexer_mlp(x, w1, b1, w2, b2, w3, b3) -> np.ndarray:
    """``COREIndexerMLP.forward`` (``core/indexer.py:88-108``): 14->128->128->1."""
    x = _f32(x).astype(np.float64)
    h = gelu(x @ w1.astype(np.float64).T + b1).astype(np.float32).astype(np.float64)
    h = gelu(h @ w2.astype(np.float64).T + b2).astype(np.float32).astype(np.float64)
    return (h @ w3.astype(np.float64).T + b3)[:, 0].astype(np.float32)


# ----------------------------------------------------------------------------
# Selection
# ----------------------------------------------------------------------------

def n_kept_for(k_len: int, compression_ratio: float, n_sink: int) -> int:
    """``COREMemoryPress.compress`` budget (``core/kvpress_adapter.py:1002-1011``)."""
    return max(1, min(max(int(k_len * (1 - compression_ratio)), min(n_sink, k_len)), k_len))


def topb_select(scores: np.ndarray, n_kept: int, n_sink: int) -> np.ndarray:
    """Sink saturation (``core/kvpress_adapter.py:773-778``) and the pooled
    stable descending argsort (``:1017-1019``).  ``scores`` is (B, L) of the
    calibrated per-token scores (identical across KV heads).  Returns the kept
    indices (B, n_kept) in ascending order.
    """
    s = _f32(scores).copy()
    L = s.shape[-1]
    if 0 < n_sink < L:
        s[:, :n_sink] = s.max() + np.float32(1.0)
    order = np.argsort(-s, axis=-1, kind="stable")[:, :n_kept]
    return np.sort(order, axis=-1)


# ----------------------------------------------------------------------------
# Latent memory write and readout
# ----------------------------------------------------------------------------

def fold_groups(w: np.ndarray, n_kv: int, groups: int, d: int) -> np.ndarray:
    """``_gqa_folded_theta`` / ``_gqa_folded_o_proj`` (``core/kvpress_adapter.py:916-966``):
    sum the ``groups`` repeated query-head blocks of the input dimension."""
    rows = w.shape[0]
    return w.astype(np.float64).reshape(rows, n_kv, groups, d).sum(axis=2) \
        .reshape(rows, n_kv * d).astype(np.float32)


def softmax_mass(scores_cal: np.ndarray, evict: np.ndarray, tau: float = 1.0):
    """``student_distribution`` (``core/indexer.py:247-273``) and
    ``conditional_evicted_weights`` (``core/indexer.py:55-72``) with
    uniform_fraction 0, as used at ``core/kvpress_adapter.py:1054-1119``.
    Returns (p (L,), p_bar (L,), pi_E scalar)."""
    x = _f32(scores_cal).astype(np.float64) / tau
    p = np.exp(x - x.max())
    p = (p / p.sum()).astype(np.float32)
    pe = np.where(evict, p, np.float32(0)).astype(np.float32)
    pi_e = np.float32(pe.astype(np.float64).sum())
    mass = pi_e if pi_e > 0 else np.float32(1)
    return p, (pe / mass).astype(np.float32), pi_e


def memory_write(k, v, scores_cal, evict, theta, *, groups: int, M=None, b=None, Z=None,
                 gamma: float = 0.9, eta: float = 1.0, tau: float = 1.0, eps: float = 1e-8):
    """Evicted-token memory write and decayed recurrence
    (``core/kvpress_adapter.py:1041-1202``, pre_o_proj value space).

    ``k``/``v`` are (Hkv, L, d); ``theta`` is the unfolded (d_mem, Hq*d)
    projection.  Returns (M (d_mem, Hkv*d), b (d_mem,), Z scalar).
    """
    k = _f32(k)
    v = _f32(v)
    nkv, L, d = k.shape
    _, p_bar, pi_e = softmax_mass(scores_cal, evict, tau)
    theta_f = fold_groups(theta, nkv, groups, d)
    kkv = k.transpose(1, 0, 2).reshape(L, nkv * d).astype(np.float64)
    vkv = v.transpose(1, 0, 2).reshape(L, nkv * d).astype(np.float64)
    phi = (kkv @ theta_f.astype(np.float64).T).astype(np.float32).astype(np.float64)
    w = p_bar.astype(np.float64)[:, None]
    m_bar = ((phi * w).T @ vkv * eta).astype(np.float32)
    b_bar = (((phi * phi) * w).sum(axis=0) * eta).astype(np.float32)
    d_mem = theta.shape[0]
    if M is None:
        M = np.zeros((d_mem, nkv * d), np.float32)
        b = np.zeros(d_mem, np.float32)
        Z = np.float32(0)
    gz = np.float32(gamma) * np.float32(Z)
    zt = np.float32(gz + pi_e)
    den = np.float32(zt + np.float32(eps))
    M_t = ((gz * M.astype(np.float64) + pi_e * m_bar.astype(np.float64)) / den).astype(np.float32)
    b_t = ((gz * b.astype(np.float64) + pi_e * b_bar.astype(np.float64)) / den).astype(np.float32)
    return M_t, b_t, zt


def f16_round(x) -> np.ndarray:
    """Round float32 to IEEE half (round-to-nearest-even) and back."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def memory_readout(q_full, theta, gate_w1, gate_b1, gate_w2, gate_b2, M, b, o_fold,
                   attn_out, *, eps: float = 1e-8, gate_override=None,
                   out_bf16: bool = True, out_dtype: str | None = None):
    """``MemoryModule.readout`` (``core/indexer.py:165-207``) and the output
    projection of ``apply_memory_readout`` (``core/kvpress_adapter.py:1302-1352``).

    ``q_full`` is (q_len, Hq*d) post-RoPE queries (head-major columns),
    ``o_fold`` the group-folded o_proj (hidden, Hkv*d); ``attn_out`` is
    (q_len, hidden).  Returns the new attention output.  ``out_dtype``
    ("bf16", "f16" or "f32"; default from ``out_bf16``) is the attention
    output's dtype: the residual and its o_proj product are rounded to it
    before the sum (``kvpress_adapter.py:1320-1343``).
    """
    if out_dtype is None:
        out_dtype = "bf16" if out_bf16 else "f32"
    rnd = {"bf16": bf16_round, "f16": f16_round, "f32": None}[out_dtype]
    q = _f32(q_full).astype(np.float64)
    proj = (q @ theta.astype(np.float64).T).astype(np.float32).astype(np.float64)
    num = proj @ M.astype(np.float64)
    den = (proj * proj) @ b.astype(np.float64) + eps
    m = num / np.sqrt(den)[:, None]
    if gate_override is None:
        h = gelu(q @ gate_w1.astype(np.float64).T + gate_b1)
        logit = h @ gate_w2.astype(np.float64).T + gate_b2
        g = 1.0 / (1.0 + np.exp(-logit[:, 0]))
    else:
        g = np.full(q.shape[0], float(gate_override))
    res = (g[:, None] * m).astype(np.float32)
    if rnd is not None:
        res = rnd(res)
    res = (res.astype(np.float64) @ o_fold.astype(np.float64).T).astype(np.float32)
    if rnd is not None:
        return rnd(_f32(attn_out) + rnd(res))
    return (_f32(attn_out) + res).astype(np.float32)


# ----------------------------------------------------------------------------
# One layer's compression step
# ----------------------------------------------------------------------------

@dataclass
class LayerWeights:
    mlp: tuple           # (w1, b1, w2, b2, w3, b3)
    geometry: np.ndarray  # (P, Hkv*d)
    prototypes: np.ndarray
    hadamard: np.ndarray
    theta: np.ndarray    # (d_mem, Hq*d)


def compress_layer(q, k, v, weights: LayerWeights, *, compression_ratio: float,
                   is_prefill: bool, positions=None, seq_len=None, round_bf16: bool,
                   n_sink: int = 4, topk_qk: int = 4, n_recent_queries: int = 16,
                   rho: float = 0.1, memory=None, gamma: float = 0.9, eta: float = 1.0,
                   tau: float = 1.0, write_memory: bool = True):
    """``COREMemoryPress.compress`` (``core/kvpress_adapter.py:968-1210``) for
    one batch row, with the scores of ``COREScorerPress.score`` (``:690-797``,
    features assembled at ``:536``).

    Returns a dict with features, scores, keep, evict, out_k, out_v, M, b, Z.
    """
    q = _f32(q)
    k = _f32(k)
    v = _f32(v)
    nq = q.shape[0]
    nkv, L, _ = k.shape
    groups = nq // nkv
    if positions is None:
        positions = np.arange(L)
    if seq_len is None:
        seq_len = L
    qk, lse, _ = qk_features(q, k, groups=groups, topk_qk=topk_qk,
                             n_recent_queries=n_recent_queries, round_bf16=round_bf16)
    cov = coverage_features(k, weights.geometry, weights.prototypes, weights.hadamard, rho=rho)
    aux = auxiliary_features(v, positions, seq_len=seq_len, is_prefill=is_prefill,
                             n_sink=n_sink, round_bf16=round_bf16)
    feats = np.concatenate([qk, cov, aux], axis=-1)
    scores = indexer_mlp(feats, *weights.mlp)
    out = dict(features=feats, scores=scores, lse=lse)
    n_kept = n_kept_for(L, compression_ratio, n_sink)
    if n_kept >= L:
        out.update(keep=np.arange(L), evict=np.zeros(L, bool), out_k=k, out_v=v)
        if memory is not None:
            out.update(M=memory[0], b=memory[1], Z=memory[2])
        return out
    keep = topb_select(scores[None], n_kept, n_sink)[0]
    evict = np.ones(L, bool)
    evict[keep] = False
    out.update(keep=keep, evict=evict, out_k=k[:, keep], out_v=v[:, keep])
    if write_memory:
        M, b, Z = (None, None, None) if memory is None else memory
        out["M"], out["b"], out["Z"] = memory_write(
            k, v, scores, evict, weights.theta, groups=groups, M=M, b=b, Z=Z,
            gamma=gamma, eta=eta, tau=tau)
    return out


def find_target_compression_ratio(q_len: int, target_tokens: int) -> float:
    """``DecodingPress._find_target_compression_ratio``
    (``kvpress/kvpress/presses/decoding_press.py:203-245``)."""
    if q_len <= target_tokens:
        return 0.0
    ratio = 1.0 - (target_tokens / q_len)
    low, high = 0.0, 1.0
    for _ in range(20):
        n = int(q_len * (1 - ratio))
        if n == target_tokens:
            break
        if n > target_tokens:
            low = ratio
            ratio = (ratio + high) / 2
        else:
            high = ratio
            ratio = (low + ratio) / 2
    return ratio
