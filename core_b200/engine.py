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


def cache_dtype(dtype: torch.dtype) -> torch.dtype:
    """Compute type of the CUDA path for caches of ``dtype``: f32 caches keep
    f32 (the reference's fp32 arithmetic), every other dtype runs as bf16."""
    return torch.float32 if dtype == torch.float32 else torch.bfloat16


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

    geometry_ext   : (3, 128, Hkv*d) bf16 terms of [W ; R W] (projection, rotation)
    prototypes     : (64, 64) f32
    mlp            : packed f32 indexer MLP (see ops.pack_mlp)
    theta          : (d_mem, Hq*d) f32 memory projection (readout side)
    theta_split    : (2, d_mem, Hkv*d) bf16 terms of the group-folded projection
                     (the memory write of bf16 caches)
    theta_fold     : (d_mem, Hkv*d) f32 group-folded projection (that of f32 caches)
    gate           : (w1 (gh, Hq*d), b1 (gh), w2 (gh), b2 (1)) f32
    """

    geometry_ext: torch.Tensor
    prototypes: torch.Tensor
    mlp: torch.Tensor
    theta: torch.Tensor | None = None
    theta_split: torch.Tensor | None = None
    gate: tuple | None = None
    theta_fold: torch.Tensor | None = None

    def write_theta(self, dtype: torch.dtype) -> torch.Tensor | None:
        """The memory-write projection in the form caches of ``dtype`` take."""
        return self.theta_fold if cache_dtype(dtype) == torch.float32 else self.theta_split

    @classmethod
    def prepare(cls, *, geometry, prototypes, hadamard, mlp_params, theta=None, gate=None,
                n_kv_heads: int, n_q_heads: int, head_dim: int = 128, device="cuda"):
        dev = torch.device(device)
        geo = ops.prepare_geometry(geometry.to(dev, torch.float32), hadamard.to(dev, torch.float32))
        groups = n_q_heads // n_kv_heads
        th = ths = thf = g = None
        if theta is not None:
            th = theta.to(dev, torch.float32).contiguous()
            thf = fold_groups(th, n_kv_heads, groups, head_dim)
            ths = ops.split_bf16(thf, 2)
        if gate is not None:
            g = tuple(x.to(dev, torch.float32).reshape(-1).contiguous() if i else
                      x.to(dev, torch.float32).contiguous() for i, x in enumerate(gate))
        return cls(
            geometry_ext=geo,
            prototypes=prototypes.to(dev, torch.float32).contiguous(),
            mlp=ops.pack_mlp([t.to(dev) for t in mlp_params]),
            theta=th, theta_split=ths, gate=g, theta_fold=thf)


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
                   lse: torch.Tensor | None = None, timing_events=None,
                   workspace: torch.Tensor | None = None) -> dict:
    """Score, select, write memory and gather for one layer (all batch rows)
    with a single call of ``core_compress_layer``.

    q: (B, Hq, nq, 128) post-RoPE queries of the scoring window;
    keys/values: (B, Hkv, L, 128).  f32 caches run the f32 path, any other
    dtype the bf16 one (q, keys and values are cast to that type).
    ``memory`` is updated in place.
    ``timing_events``: optional (start, end) torch.cuda.Event pair recorded
    around the QK relation kernel.  Returns dict(keys, values, keep, evict,
    scores, features); keep/evict are None and keys/values the inputs when
    n_kept >= L.
    """
    import ctypes

    from . import _lib
    ops._require_cuda(q, keys, values, positions)
    dt = cache_dtype(keys.dtype)
    q = q.to(dt).contiguous()
    k = keys.to(dt).contiguous()
    v = values.to(dt).contiguous()
    B, hkv, L, d = k.shape
    Hq, nq = q.shape[1], q.shape[2]
    dev = k.device
    dims = _lib.CoreDims(B, Hq, hkv, d, nq, L, ops._dtype_code(dt))
    theta_w = weights.write_theta(dt)
    write = memory is not None and theta_w is not None
    d_mem = theta_w.shape[-2] if write else 0
    feats = torch.empty(B, L, 14, dtype=torch.float32, device=dev)
    scores = torch.empty(B, L, dtype=torch.float32, device=dev)
    n_ev = max(L - n_kept, 0)
    keep = torch.empty(B, max(n_kept, 1), dtype=torch.int32, device=dev)
    evict = torch.empty(B, max(n_ev, 1), dtype=torch.int32, device=dev)
    compact = n_kept < L
    ok = torch.empty(B, hkv, n_kept, d, dtype=dt, device=dev) if compact else k
    ov = torch.empty_like(ok) if compact else v
    lib = _lib.load()
    need = lib.core_compress_layer_workspace_bytes(ctypes.byref(dims), int(n_kept), int(d_mem))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(int(need), 256), dtype=torch.uint8, device=dev)
    w = _lib.CoreLayerWeights(weights.geometry_ext.data_ptr(), weights.prototypes.data_ptr(),
                              weights.mlp.data_ptr(),
                              theta_w.data_ptr() if write else 0, int(d_mem))
    a = _lib.CoreCompressArgs(int(n_kept), int(n_sink), int(topk_qk), int(n_recent_queries),
                              float(shrinkage_rho), int(original_length), int(bool(is_prefill)),
                              float(gamma), float(eta), float(student_temp))
    pos = positions.to(torch.int64).reshape(B, L).contiguous()
    sp = None if special is None else special.to(torch.uint8).reshape(B, L).contiguous()
    lse_in = None if lse is None else lse.to(torch.float32).contiguous()
    ev0 = ev1 = None
    if timing_events is not None:
        ev0, ev1 = (ctypes.c_void_p(e.cuda_event) for e in timing_events)
    P = ops._ptr
    _lib.check(lib.core_compress_layer(
        ctypes.byref(dims), P(q), P(k), P(v), P(pos), P(sp), P(lse_in), ctypes.byref(w),
        ctypes.byref(a), P(feats), P(scores), P(keep), P(evict),
        P(memory.M if write else None), P(memory.b if write else None),
        P(memory.Z if write else None), P(ok), P(ov), P(workspace), workspace.numel(),
        ops._stream(dev), ev0, ev1))
    if not compact:
        return dict(keys=keys, values=values, keep=None, evict=None, scores=scores, features=feats)
    return dict(keys=ok, values=ov, keep=keep, evict=evict[:, :n_ev], scores=scores,
                features=feats)


def compress_layers(jobs, *, n_streams: int = 2, workspaces=None, **kwargs) -> list:
    """Compress independent layers concurrently on ``n_streams`` side streams.

    ``jobs`` is a list of dicts with the per-layer arguments of
    :func:`compress_layer` (``q``, ``keys``, ``values``, ``weights``,
    ``positions`` and optionally ``memory``, ``timing_events``, ``special``,
    ``lse``); ``kwargs`` are shared by all layers.  Layer i runs on side stream
    i mod n_streams; the side streams start after the work already queued on
    the current stream and the current stream waits for all of them before
    returning.  ``workspaces``: optional list of n_streams device buffers, one
    per side stream.  Pair it with :func:`core_b200.ops.sm_budget` so that the
    persistent grids of one layer leave SMs for the small kernels of another.
    """
    if not jobs:
        return []
    dev = jobs[0]["keys"].device
    main = torch.cuda.current_stream(dev)
    streams = _side_streams(dev, n_streams)
    fork = torch.cuda.Event()
    fork.record(main)
    for s in streams:
        s.wait_event(fork)
    out = [None] * len(jobs)
    for i, job in enumerate(jobs):
        s = streams[i % n_streams]
        for t in (job["q"], job["keys"], job["values"], job["positions"]):
            t.record_stream(s)
        with torch.cuda.stream(s):
            ws = None if workspaces is None else workspaces[i % n_streams]
            out[i] = compress_layer(**job, **kwargs, workspace=ws)
    for s in streams:
        done = torch.cuda.Event()
        done.record(s)
        main.wait_event(done)
    return out


_SIDE_STREAMS: dict = {}


def _side_streams(dev: torch.device, n: int) -> list:
    key = (dev.index, n)
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = [torch.cuda.Stream(dev) for _ in range(n)]
    return _SIDE_STREAMS[key]
