"""Torch-facing wrappers of the C ABI (one function per entry point).

Each wrapper validates shapes/dtypes/devices, allocates outputs and the
workspace with torch on the tensors' device, and calls the CUDA library on
the current torch stream.  There is no CPU path: inputs must be CUDA tensors.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import CoreDims, check

HEAD_DIM = 128


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("core_b200 operates on CUDA tensors only (no CPU path)")


_DTYPES = {torch.bfloat16: _lib.CORE_DTYPE_BF16, torch.float32: _lib.CORE_DTYPE_F32}


def _dtype_code(dtype: torch.dtype) -> int:
    """bf16 caches run on the tensor cores with the reference's bf16 roundings;
    f32 caches (the reference's fp32 path) on CUDA cores in f32."""
    if dtype not in _DTYPES:
        raise TypeError(f"core_b200 takes bfloat16 or float32 caches; got {dtype}")
    return _DTYPES[dtype]


_READOUT_DTYPES = {torch.bfloat16: _lib.CORE_DTYPE_BF16, torch.float16: _lib.CORE_DTYPE_F16,
                   torch.float32: _lib.CORE_DTYPE_F32}


def gate_value(gate_override) -> float:
    """The C-ABI gate argument: NaN selects the learned gate, a finite value
    is the constant gate (negative values included, as in the reference)."""
    if gate_override is None:
        return float("nan")
    g = float(gate_override)
    if not math.isfinite(g):
        raise ValueError(f"memory_gate_override must be finite, got {gate_override!r}")
    return g


def _dims(keys: torch.Tensor, n_q_heads: int, n_queries: int) -> CoreDims:
    b, hkv, L, d = keys.shape
    return CoreDims(b, n_q_heads, hkv, d, n_queries, L, _dtype_code(keys.dtype))


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def status(device=None) -> None:
    """Raise if a kernel recorded a device-side error (synchronises the stream)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    check(_lib.load().core_check_device_status(_stream(device)))


class sm_budget:
    """Context manager (and plain call) capping the SMs the persistent grids
    plan for, process-wide; ``sm_budget(0)`` restores all SMs."""

    def __init__(self, n_sms: int):
        self.n = int(n_sms)
        check(_lib.load().core_set_sm_budget(self.n))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        check(_lib.load().core_set_sm_budget(0))


# ---------------------------------------------------------------------------
def qk_features(q: torch.Tensor, k: torch.Tensor, *, topk_qk: int = 4,
                n_recent_queries: int = 16, lse: torch.Tensor | None = None,
                features: torch.Tensor | None = None):
    """f1..f6 of every cached key (``strict_causal_qk_features``).

    q: (B, Hq, nq, 128), k: (B, Hkv, L, 128), both bf16 (tensor-core path,
    logits rounded to bf16 like the reference's bf16 matmul) or both f32
    (CUDA-core path, unrounded f32 logits).  Returns
    (features (B, L, 6) or the given (B, L, F>=6) buffer, lse (B, Hq, nq)).
    """
    _require_cuda(q, k, lse)
    q = q.contiguous()
    k = k.contiguous()
    B, Hq, nq, d = q.shape
    dims = _dims(k, Hq, nq)
    if q.dtype != k.dtype or d != HEAD_DIM:
        raise TypeError("q must have the cache dtype and head_dim 128")
    lib = _lib.load()
    if features is None:
        features = torch.empty(B, k.shape[2], 6, dtype=torch.float32, device=k.device)
    lse_out = torch.empty(B, Hq, nq, dtype=torch.float32, device=k.device)
    ws = _workspace(lib.core_qk_features_workspace_bytes(ctypes.byref(dims)), k.device)
    lse_in = None if lse is None else lse.to(torch.float32).contiguous()
    check(lib.core_qk_features(ctypes.byref(dims), _ptr(q), _ptr(k), topk_qk, n_recent_queries,
                               _ptr(lse_in), _ptr(lse_out), _ptr(features), features.shape[-1],
                               _ptr(ws), ws.numel(), _stream(k.device)))
    return features, lse_out


_ATTN_DTYPES = {torch.bfloat16: _lib.CORE_DTYPE_BF16, torch.float16: _lib.CORE_DTYPE_F16}


def attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                      softmax_scale: float | None = None, out: torch.Tensor | None = None):
    """Causal attention with the row LSE (``flash_attn_func(..., causal=True,
    return_attn_probs=True)`` as ``_core_flash_attention_forward`` calls it).

    q: (B, Hq, Lq, 128), k, v: (B, Hkv, Lk, 128), bf16 or f16, any strides with
    the head dim contiguous (the layout an HF attention module passes).
    Returns (out (B, Lq, Hq, 128) in q's dtype, lse (B, Hq, Lq) f32).
    """
    _require_cuda(q, k, v)
    if q.dtype not in _ATTN_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("attention_prefill takes q, k, v of one dtype, bfloat16 or float16")
    B, Hq, Lq, d = q.shape
    _, Hkv, Lk, _ = k.shape
    if d != HEAD_DIM or k.shape[-1] != HEAD_DIM or v.shape != k.shape or k.shape[0] != B:
        raise ValueError("attention_prefill: head_dim 128 and matching batch / K, V shapes")

    def inner(t):
        # the head dim must be contiguous and every other stride 16-byte aligned
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    q, k, v = inner(q), inner(k), inner(v)
    dims = CoreDims(B, Hq, Hkv, HEAD_DIM, Lq, Lk, _ATTN_DTYPES[q.dtype])
    if out is None:
        out = torch.empty(B, Lq, Hq, HEAD_DIM, dtype=q.dtype, device=q.device)
    elif out.shape != (B, Lq, Hq, HEAD_DIM) or not out.is_contiguous() or out.dtype != q.dtype:
        raise ValueError("out must be a contiguous (B, Lq, Hq, 128) tensor of q's dtype")
    lse = torch.empty(B, Hq, Lq, dtype=torch.float32, device=q.device)
    scale = HEAD_DIM ** -0.5 if softmax_scale is None else float(softmax_scale)
    arrs = [(ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2)) for t in (q, k, v)]
    strides = [ctypes.cast(a, ctypes.c_void_p) for a in arrs]
    check(_lib.load().core_attention_prefill(
        ctypes.byref(dims), _ptr(q), strides[0], _ptr(k), strides[1], _ptr(v), strides[2],
        _ptr(out), _ptr(lse), scale, _stream(q.device)))
    return out, lse


def split_bf16(w: torch.Tensor, terms: int) -> torch.Tensor:
    """f32 -> (terms, *w.shape) bf16 whose sum reproduces w (hi, mid, lo)."""
    _require_cuda(w)
    w = w.to(torch.float32).contiguous()
    out = torch.empty((terms, *w.shape), dtype=torch.bfloat16, device=w.device)
    check(_lib.load().core_split_bf16(_ptr(w), w.numel(), terms, _ptr(out), _stream(w.device)))
    return out


def prepare_geometry(geometry: torch.Tensor, hadamard: torch.Tensor) -> torch.Tensor:
    """(3, 128, Hkv*d) bf16 terms of [W ; R W] for ``coverage_features``."""
    _require_cuda(geometry, hadamard)
    g = geometry.to(torch.float32).contiguous()
    r = hadamard.to(torch.float32).contiguous()
    if g.shape[0] != 64 or tuple(r.shape) != (64, 64):
        raise ValueError("geometry must be (64, Hkv*d) and hadamard (64, 64)")
    out = torch.empty(3, 128, g.shape[1], dtype=torch.bfloat16, device=g.device)
    check(_lib.load().core_prepare_geometry(_ptr(g), _ptr(r), g.shape[1], _ptr(out), _stream(g.device)))
    return out


def coverage_features(k: torch.Tensor, geometry_ext: torch.Tensor, prototypes: torch.Tensor, *,
                      shrinkage_rho: float = 0.1, features: torch.Tensor | None = None,
                      col0: int = 0):
    """o, d_proto, delta_proto, g (``compute_coverage_features``)."""
    _require_cuda(k, geometry_ext, prototypes)
    k = k.contiguous()
    B, hkv, L, d = k.shape
    dims = _dims(k, hkv, 0)
    if tuple(geometry_ext.shape) != (3, 128, hkv * d):
        raise ValueError("geometry_ext must be (3, 128, Hkv*d) (see prepare_geometry)")
    lib = _lib.load()
    if features is None:
        features = torch.empty(B, L, 4, dtype=torch.float32, device=k.device)
        col0 = 0
    ws = _workspace(lib.core_coverage_workspace_bytes(ctypes.byref(dims)), k.device)
    check(lib.core_coverage_features(
        ctypes.byref(dims), _ptr(k), _ptr(geometry_ext.contiguous()),
        _ptr(prototypes.float().contiguous()), float(shrinkage_rho), _ptr(features),
        features.shape[-1], col0, _ptr(ws), ws.numel(), _stream(k.device)))
    return features


def pack_mlp(mlp_params) -> torch.Tensor:
    """The prepared indexer MLP of ``core_prepare_indexer_mlp``: [w1 (128,14) | b1 |
    w2^T (in 128, out 128) | b2 | w3 (128) | b3] as f32 (nn.Linear weights are
    (out, in); layer 2 is stored transposed), followed on the device by layer 2's
    three-term bf16 tensor-core image."""
    w1, b1, w2, b2, w3, b3 = mlp_params
    flat = torch.cat([w1.reshape(-1), b1.reshape(-1), w2.t().reshape(-1), b2.reshape(-1),
                      w3.reshape(-1), b3.reshape(-1)]).to(torch.float32)
    _require_cuda(flat)
    lib = _lib.load()
    out = torch.zeros(lib.core_indexer_mlp_bytes() // 4, dtype=torch.float32, device=flat.device)
    out[:flat.numel()] = flat
    check(lib.core_prepare_indexer_mlp(_ptr(out), _stream(out.device)))
    return out


def indexer_scores(v: torch.Tensor, positions: torch.Tensor, features: torch.Tensor,
                   mlp_packed: torch.Tensor, *, original_length: int, is_prefill: bool,
                   n_sink: int = 4, special: torch.Tensor | None = None) -> torch.Tensor:
    """Auxiliary features into columns 10..13 of ``features`` (B, L, 14) and the
    indexer MLP scores (B, L)."""
    _require_cuda(v, positions, features, mlp_packed, special)
    v = v.contiguous()
    B, hkv, L, d = v.shape
    dims = _dims(v, hkv, 0)
    if features.shape != (B, L, 14) or not features.is_contiguous():
        raise ValueError("features must be a contiguous (B, L, 14) float32 tensor")
    pos = positions.to(torch.int64).reshape(B, L).contiguous()
    sp = None if special is None else special.to(torch.uint8).reshape(B, L).contiguous()
    scores = torch.empty(B, L, dtype=torch.float32, device=v.device)
    check(_lib.load().core_indexer_scores(
        ctypes.byref(dims), _ptr(v), _ptr(pos), _ptr(sp), int(original_length), int(is_prefill),
        int(n_sink), _ptr(features), _ptr(mlp_packed), _ptr(scores), _stream(v.device)))
    return scores


def topb_select(scores: torch.Tensor, n_kept: int, n_sink: int):
    """(keep (B, n_kept), evict (B, L - n_kept)) int32, both ascending."""
    _require_cuda(scores)
    scores = scores.to(torch.float32).contiguous()
    B, L = scores.shape
    keep = torch.empty(B, n_kept, dtype=torch.int32, device=scores.device)
    evict = torch.empty(B, max(L - n_kept, 1), dtype=torch.int32, device=scores.device)
    check(_lib.load().core_topb_select(_ptr(scores), B, L, int(n_kept), int(n_sink), _ptr(keep),
                                       _ptr(evict), _ptr(None), 0, _stream(scores.device)))
    return keep, evict[:, : L - n_kept]


def memory_write(k: torch.Tensor, v: torch.Tensor, scores_cal: torch.Tensor,
                 evict: torch.Tensor, theta_split: torch.Tensor, M: torch.Tensor,
                 b_state: torch.Tensor, Z: torch.Tensor, *, gamma: float, eta: float,
                 student_temp: float) -> None:
    """Update (M, b, Z) in place with the evicted tokens (``compress`` memory write).

    ``theta_split``: for bf16 caches the (2, d_mem, Hkv*d) bf16 terms of the
    group-folded Theta (``split_bf16(fold, 2)``); for f32 caches the folded
    (d_mem, Hkv*d) f32 Theta itself.
    """
    _require_cuda(k, v, scores_cal, evict, theta_split, M, b_state, Z)
    k = k.contiguous()
    v = v.contiguous()
    B, hkv, L, d = k.shape
    dims = _dims(k, hkv, 0)
    if v.dtype != k.dtype:
        raise TypeError("keys and values must have one dtype")
    n_evict = evict.shape[1]
    if k.dtype == torch.float32:
        if theta_split.dim() != 2 or theta_split.dtype != torch.float32:
            raise ValueError("f32 caches take the folded (d_mem, Hkv*d) f32 Theta")
        d_mem = theta_split.shape[0]
    else:
        if theta_split.dim() != 3 or theta_split.dtype != torch.bfloat16:
            raise ValueError("bf16 caches take the (2, d_mem, Hkv*d) bf16 terms of Theta")
        d_mem = theta_split.shape[1]
    for name, t, shape in (("M", M, (B, d_mem, hkv * d)), ("b", b_state, (B, d_mem)), ("Z", Z, (B,))):
        if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous float32 tensor of shape {shape}")
    lib = _lib.load()
    ws = _workspace(lib.core_memory_write_workspace_bytes(ctypes.byref(dims), n_evict, d_mem), k.device)
    check(lib.core_memory_write(
        ctypes.byref(dims), _ptr(k), _ptr(v), _ptr(scores_cal.float().contiguous()),
        _ptr(evict.to(torch.int32).contiguous()), n_evict, _ptr(theta_split.contiguous()), d_mem,
        float(gamma), float(eta), float(student_temp), _ptr(M), _ptr(b_state), _ptr(Z), _ptr(ws),
        ws.numel(), _stream(k.device)))


def compact_kv(k: torch.Tensor, v: torch.Tensor, keep: torch.Tensor):
    """Gather the kept rows: (B, Hkv, n_kept, d) keys and values (bf16, fp16
    or f32 caches: the rows are copied bit for bit)."""
    _require_cuda(k, v, keep)
    k = k.contiguous()
    v = v.contiguous()
    B, hkv, L, d = k.shape
    n_kept = keep.shape[1]
    if k.dtype == torch.float16:
        dims = CoreDims(B, hkv, hkv, d, 0, L, _lib.CORE_DTYPE_F16)
    else:
        dims = _dims(k, hkv, 0)
    ok = torch.empty(B, hkv, n_kept, d, dtype=k.dtype, device=k.device)
    ov = torch.empty_like(ok)
    check(_lib.load().core_compact_kv(ctypes.byref(dims), _ptr(k), _ptr(v),
                                      _ptr(keep.to(torch.int32).contiguous()), n_kept, _ptr(ok),
                                      _ptr(ov), _stream(k.device)))
    return ok, ov


def memory_readout(q: torch.Tensor, theta: torch.Tensor, gate, M: torch.Tensor,
                   b_state: torch.Tensor, o_fold: torch.Tensor, attn_out: torch.Tensor,
                   *, n_kv_heads: int, gate_override: float | None = None,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """attn_out (B, q_len, hidden) += o_fold(g(q) m(q)); updated in place and returned.
    attn_out's dtype (bf16, fp16 or f32) selects the arithmetic; q is cast to it.
    ``gate_override``: None for the learned gate, else any finite constant gate.

    gate = (w1 (gh, Hq*d), b1 (gh), w2 (gh), b2 (1)) f32 tensors.  ``workspace``:
    an optional uint8 device buffer of at least ``core_memory_readout_workspace_bytes``
    (allocated here when absent or too small).
    """
    _require_cuda(q, theta, M, b_state, o_fold, attn_out)
    code = _READOUT_DTYPES.get(attn_out.dtype)
    if code is None:
        raise TypeError(f"memory_readout takes bf16, fp16 or f32 outputs; got {attn_out.dtype}")
    q = q.to(attn_out.dtype).contiguous()
    B, Hq, q_len, d = q.shape
    dims = CoreDims(B, Hq, n_kv_heads, d, q_len, max(q_len, 1), code)
    d_mem = theta.shape[0]
    hidden = o_fold.shape[0]
    w1, b1, w2, b2 = gate
    gh = w1.shape[0]
    if not attn_out.is_contiguous():
        raise ValueError("attn_out must be contiguous")
    lib = _lib.load()
    need = lib.core_memory_readout_workspace_bytes(ctypes.byref(dims), q_len, d_mem, gh)
    ws = workspace if workspace is not None and workspace.numel() >= need else _workspace(need, q.device)
    go = gate_value(gate_override)
    check(lib.core_memory_readout(
        ctypes.byref(dims), q_len, _ptr(q), _ptr(theta), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
        d_mem, gh, go, _ptr(M), _ptr(b_state), _ptr(o_fold), hidden, _ptr(attn_out), _ptr(ws),
        ws.numel(), _stream(q.device)))
    return attn_out


_ROPE_DTYPES = _READOUT_DTYPES


def rope_queries(q_proj: torch.Tensor, n_q_heads: int, *, positions: torch.Tensor | None = None,
                 inv_freq: torch.Tensor | None = None, attention_scaling: float = 1.0,
                 cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Post-RoPE queries (B, Hq, T, d) from q_proj rows (B, T, Hq*d).

    Either ``positions`` (B or 1, T) int64 with the rotary ``inv_freq`` (d/2)
    and ``attention_scaling`` of a LlamaRotaryEmbedding, or the (cos, sin)
    position embeddings (B or 1, T, d) a model computed.  Roundings are those
    of transformers' apply_rotary_pos_emb in q_proj's dtype.
    """
    _require_cuda(q_proj, positions, inv_freq, cos, sin)
    if q_proj.dim() != 3 or q_proj.stride(-1) != 1:
        raise ValueError("q_proj must be (B, T, Hq*d) with unit inner stride")
    code = _ROPE_DTYPES.get(q_proj.dtype)
    if code is None:
        raise TypeError(f"rope_queries takes bf16, fp16 or f32; got {q_proj.dtype}")
    B, T, width = q_proj.shape
    if width % n_q_heads:
        raise ValueError("q_proj width must be a multiple of n_q_heads")
    d = width // n_q_heads
    if q_proj.stride(0) != T * q_proj.stride(1):
        q_proj = q_proj.contiguous()
    row_stride = q_proj.stride(1)
    if out is None:
        out = torch.empty(B, n_q_heads, T, d, dtype=q_proj.dtype, device=q_proj.device)
    pos = inv = c = s = None
    cb = 1
    if cos is not None:
        c = cos.to(q_proj.dtype).reshape(-1, T, d).contiguous()
        s = sin.to(q_proj.dtype).reshape(-1, T, d).contiguous()
        cb = c.shape[0]
        if cb not in (1, B) or s.shape != c.shape:
            raise ValueError("cos/sin must be (1 or B, T, d)")
    else:
        if positions is None or inv_freq is None:
            raise ValueError("rope_queries needs positions and inv_freq, or cos and sin")
        pos = positions.to(torch.int64).reshape(-1, T).expand(B, T).contiguous()
        inv = inv_freq.to(torch.float32).contiguous()
        if inv.numel() != d // 2:
            raise ValueError("inv_freq must hold head_dim/2 frequencies")
    check(_lib.load().core_rope_queries(B, T, n_q_heads, d, code, _ptr(q_proj), row_stride,
                                        _ptr(pos), _ptr(inv), float(attention_scaling), _ptr(c),
                                        _ptr(s), cb, _ptr(out), _stream(q_proj.device)))
    return out


# ---------------------------------------------------------------------------
# Head-sharded caches (one sequence, KV heads split across ranks).  Each call
# is one rank's part of a layer step; the cross-head sums between them are
# the caller's (core_b200.sharded runs them with NCCL).
# ---------------------------------------------------------------------------

def qk_summary_words(n_queries: int) -> int:
    return int(_lib.load().core_qk_summary_words(int(n_queries)))


def qk_head_summary(q: torch.Tensor, k: torch.Tensor, summary: torch.Tensor, *,
                    topk_qk: int = 4, n_recent_queries: int = 16) -> torch.Tensor:
    """Per-key summaries of this rank's heads into ``summary`` (rows >= L,
    core_qk_summary_words(nq)) int32; returns the rank's LSE (Hq_rank, nq)."""
    _require_cuda(q, k, summary)
    q = q.contiguous()
    k = k.contiguous()
    B, Hq, nq, d = q.shape
    if B != 1 or k.dtype != torch.bfloat16 or q.dtype != torch.bfloat16:
        raise ValueError("head-sharded summaries take one bf16 sequence")
    words = qk_summary_words(nq)
    if (summary.dim() != 2 or summary.shape[0] < k.shape[2] or summary.shape[1] != words
            or summary.dtype != torch.int32 or not summary.is_contiguous()):
        raise ValueError(f"summary must be a contiguous (>= L, {words}) int32 tensor")
    dims = _dims(k, Hq, nq)
    lib = _lib.load()
    lse = torch.empty(Hq, nq, dtype=torch.float32, device=k.device)
    ws = _workspace(lib.core_qk_features_workspace_bytes(ctypes.byref(dims)), k.device)
    check(lib.core_qk_head_summary(ctypes.byref(dims), _ptr(q), _ptr(k), int(topk_qk),
                                   int(n_recent_queries), _ptr(lse), _ptr(summary), _ptr(ws),
                                   ws.numel(), _stream(k.device)))
    return lse


def qk_merge_summaries(parts: torch.Tensor, features: torch.Tensor, *, key0: int, n_keys: int,
                       seq_len: int, n_queries: int, n_kv_heads: int, topk_qk: int = 4,
                       n_recent_queries: int = 16) -> None:
    """f1..f6 of keys key0 .. key0 + n_keys - 1 into features[:n_keys, :6] from
    the ranks' summaries ``parts`` (n_parts, rows, words)."""
    _require_cuda(parts, features)
    if parts.dim() != 3 or not parts.is_contiguous() or parts.dtype != torch.int32:
        raise ValueError("parts must be a contiguous (n_parts, rows, words) int32 tensor")
    if features.dim() != 2 or not features.is_contiguous() or features.shape[0] < n_keys:
        raise ValueError("features must be a contiguous (>= n_keys, F) float32 tensor")
    check(_lib.load().core_qk_merge_summaries(
        _ptr(parts), parts.shape[0], parts.shape[1], int(key0), int(n_keys), int(seq_len),
        int(n_queries), int(n_kv_heads), int(topk_qk), int(n_recent_queries), _ptr(features),
        features.shape[1], _stream(parts.device)))


def coverage_partial_projection(k: torch.Tensor, geometry_ext: torch.Tensor, y: torch.Tensor) -> None:
    """y[:L] = sum over this rank's heads of W_h k_h / |k_h| (raw, (L, 64) f32)."""
    _require_cuda(k, geometry_ext, y)
    k = k.contiguous()
    B, hkv, L, d = k.shape
    if B != 1:
        raise ValueError("head-sharded coverage takes one sequence")
    if tuple(geometry_ext.shape) != (3, 128, hkv * d):
        raise ValueError("geometry_ext must hold this rank's columns, (3, 128, Hkv_rank*d)")
    if y.dim() != 2 or y.shape[0] < L or y.shape[1] != 64 or not y.is_contiguous():
        raise ValueError("y must be a contiguous (>= L, 64) float32 tensor")
    dims = _dims(k, hkv, 0)
    lib = _lib.load()
    ws = _workspace(lib.core_coverage_workspace_bytes(ctypes.byref(dims)), k.device)
    check(lib.core_coverage_partial_projection(ctypes.byref(dims), _ptr(k),
                                               _ptr(geometry_ext.contiguous()), _ptr(y), _ptr(ws),
                                               ws.numel(), _stream(k.device)))


def coverage_range_totals(y: torch.Tensor, hadamard: torch.Tensor):
    """(z, zt, totals (192,) f64) for the summed projections y (n, 64) of a key range."""
    _require_cuda(y, hadamard)
    n = y.shape[0]
    y = y.contiguous()
    z = torch.empty(n, 64, dtype=torch.float32, device=y.device)
    zt = torch.empty_like(z)
    totals = torch.empty(192, dtype=torch.float64, device=y.device)
    lib = _lib.load()
    ws = _workspace(lib.core_coverage_range_workspace_bytes(n), y.device)
    check(lib.core_coverage_range_totals(_ptr(y), n, _ptr(hadamard.float().contiguous()), _ptr(z),
                                         _ptr(zt), _ptr(totals), _ptr(ws), ws.numel(),
                                         _stream(y.device)))
    return z, zt, totals


def coverage_range_assign(totals: torch.Tensor, seq_len: int, z: torch.Tensor, zt: torch.Tensor,
                          prototypes: torch.Tensor, features: torch.Tensor, *, col0: int = 6,
                          shrinkage_rho: float = 0.1):
    """Statistics of the summed totals, then d, delta and g of the range's keys
    into features[:, col0 + 1 .. col0 + 3]; returns (assign, hist (64,) int32)."""
    _require_cuda(totals, z, zt, prototypes, features)
    n = z.shape[0]
    assign = torch.empty(max(n, 1), dtype=torch.int32, device=z.device)
    hist = torch.empty(64, dtype=torch.int32, device=z.device)
    lib = _lib.load()
    ws = _workspace(lib.core_coverage_range_workspace_bytes(n), z.device)
    check(lib.core_coverage_range_assign(
        _ptr(totals.contiguous()), int(seq_len), float(shrinkage_rho), _ptr(z), _ptr(zt), n,
        _ptr(prototypes.float().contiguous()), _ptr(assign), _ptr(hist), _ptr(features),
        features.shape[-1], int(col0), _ptr(ws), ws.numel(), _stream(z.device)))
    return assign, hist


def coverage_range_occupancy(assign: torch.Tensor, hist: torch.Tensor, features: torch.Tensor,
                             n_keys: int, *, col0: int = 6) -> None:
    _require_cuda(assign, hist, features)
    check(_lib.load().core_coverage_range_occupancy(_ptr(assign), _ptr(hist.contiguous()),
                                                    int(n_keys), _ptr(features),
                                                    features.shape[-1], int(col0),
                                                    _stream(features.device)))


def value_head_sums(v: torch.Tensor, out: torch.Tensor) -> None:
    """out[h, :L] = the bf16 sum of bf16 squares of each value row of this rank's heads."""
    _require_cuda(v, out)
    v = v.contiguous()
    B, hkv, L, d = v.shape
    if out.dim() != 2 or out.shape[0] != hkv or out.shape[1] < L or not out.is_contiguous():
        raise ValueError("out must be a contiguous (Hkv_rank, >= L) float32 tensor")
    dims = _dims(v, hkv, 0)
    check(_lib.load().core_value_head_sums(ctypes.byref(dims), _ptr(v), _ptr(out), out.shape[1],
                                           _stream(v.device)))


def indexer_scores_from_sums(head_sums: torch.Tensor, key0: int, n_keys: int,
                             positions: torch.Tensor, features: torch.Tensor,
                             mlp_packed: torch.Tensor, *, original_length: int, is_prefill: bool,
                             n_sink: int = 4, special: torch.Tensor | None = None) -> torch.Tensor:
    """Scores of keys key0 .. key0 + n_keys - 1 from all heads' value sums
    head_sums (Hkv, stride); positions/special are the whole sequence's,
    features (n_keys, 14) the range's."""
    _require_cuda(head_sums, positions, features, mlp_packed, special)
    if not head_sums.is_contiguous() or head_sums.dim() != 2:
        raise ValueError("head_sums must be a contiguous (Hkv, stride) float32 tensor")
    if features.shape[0] < n_keys or features.shape[1] != 14 or not features.is_contiguous():
        raise ValueError("features must be a contiguous (>= n_keys, 14) float32 tensor")
    pos = positions.to(torch.int64).reshape(-1).contiguous()
    sp = None if special is None else special.to(torch.uint8).reshape(-1).contiguous()
    scores = torch.empty(max(n_keys, 1), dtype=torch.float32, device=features.device)
    hs_ptr = head_sums.data_ptr() + 4 * int(key0)
    pos_ptr = pos.data_ptr() + 8 * int(key0)
    sp_ptr = None if sp is None else sp.data_ptr() + int(key0)
    check(_lib.load().core_indexer_scores_from_sums(
        head_sums.shape[0], int(n_keys), ctypes.c_void_p(hs_ptr), head_sums.shape[1],
        ctypes.c_void_p(pos_ptr), ctypes.c_void_p(sp_ptr), int(original_length), int(is_prefill),
        int(n_sink), _ptr(features), _ptr(mlp_packed), _ptr(scores), _stream(features.device)))
    return scores[:n_keys]


def memory_write_gathered(k_ev: torch.Tensor, v_ev: torch.Tensor, scores_cal: torch.Tensor,
                          evict: torch.Tensor, theta_split: torch.Tensor, M: torch.Tensor,
                          b_state: torch.Tensor, Z: torch.Tensor, *, gamma: float, eta: float,
                          student_temp: float) -> None:
    """``memory_write`` with the evicted rows already gathered: k_ev, v_ev =
    (B, Hkv, n_evict, d) in evict order; scores_cal (B, L)."""
    _require_cuda(k_ev, v_ev, scores_cal, evict, theta_split, M, b_state, Z)
    k_ev = k_ev.contiguous()
    v_ev = v_ev.contiguous()
    B, hkv, n_evict, d = k_ev.shape
    L = scores_cal.shape[-1]
    if evict.shape != (B, n_evict):
        raise ValueError("evict must be (B, n_evict)")
    if k_ev.dtype != torch.bfloat16 or theta_split.dim() != 3:
        raise ValueError("gathered memory write takes bf16 rows and the (2, d_mem, Hkv*d) terms")
    d_mem = theta_split.shape[1]
    dims = CoreDims(B, hkv, hkv, d, 0, L, _lib.CORE_DTYPE_BF16)
    lib = _lib.load()
    ws = _workspace(lib.core_memory_write_workspace_bytes(ctypes.byref(dims), n_evict, d_mem),
                    k_ev.device)
    check(lib.core_memory_write_gathered(
        ctypes.byref(dims), _ptr(k_ev), _ptr(v_ev), _ptr(scores_cal.float().contiguous()),
        _ptr(evict.to(torch.int32).contiguous()), n_evict, _ptr(theta_split.contiguous()), d_mem,
        float(gamma), float(eta), float(student_temp), _ptr(M), _ptr(b_state), _ptr(Z), _ptr(ws),
        ws.numel(), _stream(k_ev.device)))
