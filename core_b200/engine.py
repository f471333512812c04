"""One layer's CORE compression step on the CUDA library.

``LayerWeights`` holds a layer's slow weights in the device formats the
kernels take (prepared once per layer and cached by the press);
``compress_layer`` runs QK features -> coverage -> auxiliary + indexer MLP ->
Top-B -> memory write -> retained-KV gather for every batch row at once,
following ``COREMemoryPress.compress`` (core/kvpress_adapter.py:968-1210).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


def n_kept_for(k_len: int, compression_ratio: float, n_sink: int) -> int:
    """Retained budget of ``COREMemoryPress.compress`` (core/kvpress_adapter.py:1002-1011)."""
    return max(1, min(max(int(k_len * (1 - compression_ratio)), min(n_sink, k_len)), k_len))


def fold_groups(w: torch.Tensor, n_kv_heads: int, groups: int, head_dim: int) -> torch.Tensor:
    """Sum the repeated query-head blocks of the input dimension
    (``_gqa_folded_theta`` / ``_gqa_folded_o_proj``, core/kvpress_adapter.py:916-966)."""
    rows = w.shape[0]
    return (w.float().reshape(rows, n_kv_heads, groups, head_dim).sum(dim=2)
            .reshape(rows, n_kv_heads * head_dim).contiguous())


@dataclass
class LayerWeights:
    """Per-layer slow weights on the device.

    geometry_split : (3, 64, Hkv*d) bf16 terms of the fixed Gaussian projection
    prototypes     : (64, 64) f32;  hadamard : (64, 64) f32
    mlp            : packed f32 indexer MLP (see ops.pack_mlp)
    theta          : (d_mem, Hq*d) f32 memory projection (readout side)
    theta_split    : (2, d_mem, Hkv*d) bf16 terms of the group-folded projection
    gate           : (w1 (gh, Hq*d), b1 (gh), w2 (gh), b2 (1)) f32
    """

    geometry_split: torch.Tensor
    prototypes: torch.Tensor
    hadamard: torch.Tensor
    mlp: torch.Tensor
    theta: torch.Tensor | None = None
    theta_split: torch.Tensor | None = None
    gate: tuple | None = None

    @classmethod
    def prepare(cls, *, geometry, prototypes, hadamard, mlp_params, theta=None, gate=None,
                n_kv_heads: int, n_q_heads: int, head_dim: int = 128, device="cuda"):
        dev = torch.device(device)
        geometry = geometry.to(dev, torch.float32).contiguous()
        geo = ops.split_bf16(geometry, 3)
        groups = n_q_heads // n_kv_heads
        th = ths = g = None
        if theta is not None:
            th = theta.to(dev, torch.float32).contiguous()
            ths = ops.split_bf16(fold_groups(th, n_kv_heads, groups, head_dim), 2)
        if gate is not None:
            g = tuple(x.to(dev, torch.float32).reshape(-1).contiguous() if i else
                      x.to(dev, torch.float32).contiguous() for i, x in enumerate(gate))
        return cls(
            geometry_split=geo,
            prototypes=prototypes.to(dev, torch.float32).contiguous(),
            hadamard=hadamard.to(dev, torch.float32).contiguous(),
            mlp=ops.pack_mlp([t.to(dev) for t in mlp_params]),
            theta=th, theta_split=ths, gate=g)


@dataclass
class MemoryState:
    M: torch.Tensor   # (B, d_mem, Hkv*d) f32
    b: torch.Tensor   # (B, d_mem) f32
    Z: torch.Tensor   # (B,) f32

    @classmethod
    def zeros(cls, batch: int, d_mem: int, kv_width: int, device) -> "MemoryState":
        return cls(torch.zeros(batch, d_mem, kv_width, device=device),
                   torch.zeros(batch, d_mem, device=device),
                   torch.zeros(batch, device=device))


def compress_layer(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                   weights: LayerWeights, *, n_kept: int, positions: torch.Tensor,
                   original_length: int, is_prefill: bool, n_sink: int = 4, topk_qk: int = 4,
                   n_recent_queries: int = 16, shrinkage_rho: float = 0.1,
                   memory: MemoryState | None = None, gamma: float = 0.9, eta: float = 1.0,
                   student_temp: float = 1.0, special: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None, score_hook=None) -> dict:
    """Score, select, write memory and gather for one layer (all batch rows).

    q: (B, Hq, nq, 128) bf16 post-RoPE queries of the scoring window;
    keys/values: (B, Hkv, L, 128) bf16.  ``memory`` is updated in place.
    ``score_hook(scores) -> scores`` may adjust the calibrated scores before
    selection (recency bonus).  Returns dict(keys, values, keep, evict,
    scores, features).
    """
    B, hkv, L, d = keys.shape
    feats = torch.empty(B, L, 14, dtype=torch.float32, device=keys.device)
    ops.qk_features(q, keys, topk_qk=topk_qk, n_recent_queries=n_recent_queries, lse=lse,
                    features=feats)
    ops.coverage_features(keys, weights.geometry_split, weights.prototypes, weights.hadamard,
                          shrinkage_rho=shrinkage_rho, features=feats, col0=6)
    scores = ops.indexer_scores(values, positions, feats, weights.mlp,
                                original_length=original_length, is_prefill=is_prefill,
                                n_sink=n_sink, special=special)
    if score_hook is not None:
        scores = score_hook(scores)
    out = dict(scores=scores, features=feats)
    if n_kept >= L:
        out.update(keys=keys, values=values, keep=None, evict=None)
        return out
    keep, evict = ops.topb_select(scores, n_kept, n_sink)
    if memory is not None and weights.theta_split is not None and evict.shape[1] > 0:
        ops.memory_write(keys, values, scores, evict, weights.theta_split, memory.M, memory.b,
                         memory.Z, gamma=gamma, eta=eta, student_temp=student_temp)
    ok, ov = ops.compact_kv(keys, values, keep)
    out.update(keys=ok, values=ov, keep=keep, evict=evict)
    return out
