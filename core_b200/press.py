"""KVPress-compatible CORE presses running on the B200 CUDA library.

Drop-in counterparts of the reference presses (``core/kvpress_adapter.py``)
and of the KVPress hook machinery they plug into
(``kvpress/kvpress/presses/{base,scorer,decoding,prefill_decoding}_press.py``):
same class names, dataclass fields, methods, factories and hook protocol.
The compression step itself (features, scores, Top-B, memory write, gather)
and the memory readout run in the CUDA library; the classes here keep the
per-sequence host state (cache metadata, memory state, decode buffers).

Not thread-safe: one sequence per press instance, as in the reference.
"""

from __future__ import annotations

import logging
from collections import defaultdict
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Optional

import torch
from torch import nn

from . import engine, ops
from .checkpoint import FeatureGeometry, IndexerStack, MemoryStack, load_checkpoint

logger = logging.getLogger(__name__)


# ===========================================================================
# Cache metadata: original positions / token ids of the compacted slots
# (core/cache_metadata.py:6-54)
# ===========================================================================
class CacheMetadata:
    def __init__(self):
        self.reset()

    def reset(self):
        self.token_ids = None
        self.positions = {}
        self.next_position = {}

    def record(self, input_ids, position_ids=None):
        if input_ids is None:
            raise ValueError("CORE token metadata requires input_ids")
        if position_ids is None:
            start = 0 if self.token_ids is None else self.token_ids.shape[1]
            position_ids = torch.arange(start, start + input_ids.shape[1], device=input_ids.device)[None]
        position_ids = position_ids.expand(input_ids.shape[0], -1).long()
        size = int(position_ids.max()) + 1
        previous = self.token_ids
        if previous is not None:
            if previous.shape[0] != input_ids.shape[0]:
                raise ValueError("Batch changed without a sequence reset")
            size = max(size, previous.shape[1])
        ids = input_ids.new_full((input_ids.shape[0], size), -1)
        if previous is not None:
            ids[:, :previous.shape[1]] = previous.to(ids.device)
        ids.scatter_(1, position_ids, input_ids)
        self.token_ids = ids

    def align(self, layer_idx, batch_size, cache_length, device):
        previous = self.positions.get(layer_idx)
        old_length = 0 if previous is None else previous.shape[1]
        if cache_length < old_length:
            raise RuntimeError("KV metadata was not pruned with the cache; reset at new sample boundaries")
        start = self.next_position.get(layer_idx, 0)
        added = cache_length - old_length
        tail = torch.arange(start, start + added, device=device)[None].expand(batch_size, -1)
        positions = tail if previous is None else torch.cat((previous.to(device), tail), dim=1)
        self.positions[layer_idx] = positions
        self.next_position[layer_idx] = start + added
        ids = positions.new_full(positions.shape, -1)
        if self.token_ids is not None:
            journal = self.token_ids.to(device)
            if positions.numel() and int(positions.max()) >= journal.shape[1]:
                raise RuntimeError("Missing input token IDs for newly appended KV entries")
            ids = journal.gather(1, positions)
        return positions, ids, self.next_position[layer_idx]

    def retain(self, layer_idx, indices):
        self.positions[layer_idx] = self.positions[layer_idx].gather(1, indices.long()).contiguous()


def retained_budget(length, ratio, sinks=4):
    """Decode target size (core/paper_protocol.py:17-20)."""
    if not 0 <= ratio < 1 or length < 1:
        raise ValueError("Expected a nonempty sequence and 0 <= eviction ratio < 1")
    return max(min(sinks, length), int(length * (1 - ratio)))


# ===========================================================================
# KVPress hook machinery (kvpress/kvpress/presses/*.py)
# ===========================================================================
def _extract_keys_and_values(cache, layer_idx):
    layer = cache.layers[layer_idx]
    if hasattr(layer, "_quantized_keys") and getattr(layer, "keys", None) is not None \
            and layer.keys.numel() == 0:
        raise NotImplementedError("quantized KV caches are not supported by core_b200")
    return layer.keys, layer.values


def _write_back(cache, layer_idx, keys, values):
    layer = cache.layers[layer_idx]
    layer.keys = keys
    layer.values = values


@dataclass
class BasePress:
    """Hook-based press: compress the cache after each attention layer's prefill
    forward (``base_press.py:95-156``)."""

    def post_init_from_model(self, model):
        pass

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        raise NotImplementedError("compress method must be implemented in subclass")

    def forward_hook(self, module: nn.Module, input, kwargs: dict, output):
        hidden_states = kwargs["hidden_states"]
        cache = kwargs["past_key_values"]
        q_len = hidden_states.shape[1]
        if kwargs["cache_position"][-1] > q_len:
            return output
        keys, values = _extract_keys_and_values(cache, module.layer_idx)
        keys, values = self.compress(module, hidden_states, keys, values, output[1], kwargs)
        _write_back(cache, module.layer_idx, keys, values)
        return output

    @contextmanager
    def __call__(self, model):
        self.post_init_from_model(model)
        hooks = []
        try:
            lm = model.model.language_model if hasattr(model.model, "language_model") else model.model
            for layer in lm.layers:
                layer.self_attn.rotary_emb = lm.rotary_emb
                hooks.append(layer.self_attn.register_forward_hook(self.forward_hook, with_kwargs=True))

                def release_core_temporaries(module, args, output):
                    for name in ("_core_cached_query_states", "_core_cached_key_states",
                                 "_core_cached_softmax_lse"):
                        if hasattr(module, name):
                            delattr(module, name)
                hooks.append(layer.self_attn.register_forward_hook(release_core_temporaries,
                                                                   always_call=True))
            yield
        finally:
            for h in hooks:
                h.remove()


@dataclass
class ScorerPress(BasePress):
    """Score-based press (``scorer_press.py:16-106``)."""

    compression_ratio: float = 0.0

    def __post_init__(self):
        assert 0 <= self.compression_ratio < 1, "Compression ratio must be between 0 and 1"

    def score(self, module, hidden_states, keys, values, attentions, kwargs):
        raise NotImplementedError


@dataclass
class DecodingPress(BasePress):
    """Periodic decode-time compression with a hidden-state buffer (``decoding_press.py:22-248``)."""

    base_press: BasePress = None  # type: ignore[assignment]
    compression_interval: int = 512
    target_size: int = 2048
    hidden_states_buffer_size: int = 256

    def __post_init__(self):
        assert hasattr(self.base_press, "compress") and hasattr(self.base_press, "compression_ratio"), \
            "DecodingPress requires a compressible press with compression_ratio"
        self.hidden_states_buffer = defaultdict(list)
        self.layer_step_counts = defaultdict(int)
        assert self.compression_interval > 0, "compression_interval must be greater than 0"
        assert self.target_size > 0, "target_size must be greater than 0"

    def post_init_from_model(self, model):
        self.base_press.post_init_from_model(model)

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        k_len = keys.shape[2]
        target_size = self._resolve_target_size(kwargs)
        ratio = self._find_target_compression_ratio(k_len, target_size)
        original = self.base_press.compression_ratio
        self.base_press.compression_ratio = ratio
        try:
            return self.base_press.compress(module, hidden_states, keys, values, attentions, kwargs)
        finally:
            self.base_press.compression_ratio = original

    def forward_hook(self, module, input, kwargs, output):
        hidden_states = kwargs["hidden_states"]
        cache = kwargs["past_key_values"]
        q_len = hidden_states.shape[1]
        layer_idx = module.layer_idx
        if kwargs["cache_position"][-1] <= q_len:
            return output
        # Read memory written by previous compressions before this step writes.
        if hasattr(self.base_press, "apply_memory_readout"):
            output = self.base_press.apply_memory_readout(module, kwargs, output)
        self.hidden_states_buffer[layer_idx].append(hidden_states.detach().clone())
        self.layer_step_counts[layer_idx] += 1
        target_size = self._resolve_target_size(kwargs)
        if self.layer_step_counts[layer_idx] >= self.compression_interval or q_len >= target_size:
            keys, values = _extract_keys_and_values(cache, module.layer_idx)
            attentions = output[1] if len(output) > 1 and output[1] is not None else None
            buffered = torch.cat(self.hidden_states_buffer[layer_idx], dim=1)
            keys, values = self.compress(module, buffered, keys, values, attentions, kwargs)
            _write_back(cache, module.layer_idx, keys, values)
            self.layer_step_counts[layer_idx] = 0
            self.hidden_states_buffer[layer_idx] = []
        self.hidden_states_buffer[layer_idx] = (
            self.hidden_states_buffer[layer_idx][-self.hidden_states_buffer_size:]
            if self.hidden_states_buffer_size > 0 else [])
        return output

    def reset(self):
        self.hidden_states_buffer = defaultdict(list)
        self.layer_step_counts = defaultdict(int)

    @contextmanager
    def __call__(self, model):
        try:
            with super().__call__(model):
                yield
        finally:
            self.reset()

    def _find_target_compression_ratio(self, q_len: int, target_tokens: int) -> float:
        """Ratio r with int(q_len * (1 - r)) == target (``decoding_press.py:203-245``)."""
        if q_len <= target_tokens:
            return 0.0
        ratio = 1.0 - (target_tokens / q_len)
        low, high = 0.0, 1.0
        for _ in range(20):
            n_kept = int(q_len * (1 - ratio))
            if n_kept == target_tokens:
                break
            if n_kept > target_tokens:
                low = ratio
                ratio = (ratio + high) / 2
            else:
                high = ratio
                ratio = (low + ratio) / 2
        if int(q_len * (1 - ratio)) != target_tokens:
            logger.warning("Binary search failed: q_len=%d, target=%d", q_len, target_tokens)
        return ratio

    def _resolve_target_size(self, kwargs) -> int:
        return self.target_size


@dataclass
class PrefillDecodingPress(BasePress):
    """Prefill press + decoding press behind one hook (``prefill_decoding_press.py:19-113``)."""

    prefilling_press: Optional[BasePress] = None
    decoding_press: Optional[DecodingPress] = None
    query_aware_prefill: bool = False

    def post_init_from_model(self, model):
        if self.prefilling_press is not None:
            self.prefilling_press.post_init_from_model(model)
        if self.decoding_press is not None:
            self.decoding_press.post_init_from_model(model)

    def set_token_ids(self, token_ids, special_token_ids=None):
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "set_token_ids"):
            self.prefilling_press.set_token_ids(token_ids, special_token_ids)

    def set_query_boundary(self, query_start: int):
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "set_query_boundary"):
            self.prefilling_press.set_query_boundary(query_start)

    def reset_cache(self):
        seen = set()
        for press in (self.prefilling_press, getattr(self.decoding_press, "base_press", None)):
            if press is not None and id(press) not in seen and hasattr(press, "reset_cache"):
                press.reset_cache()
                seen.add(id(press))
        if self.decoding_press is not None:
            self.decoding_press.reset()

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        q_len = hidden_states.shape[1]
        if kwargs["cache_position"][-1] <= q_len and self.prefilling_press is not None:
            return self.prefilling_press.compress(module, hidden_states, keys, values, attentions, kwargs)
        if self.decoding_press is not None:
            return self.decoding_press.compress(module, hidden_states, keys, values, attentions, kwargs)
        return keys, values

    def forward_hook(self, module, input, kwargs, output):
        q_len = kwargs["hidden_states"].shape[1]
        if kwargs["cache_position"][-1] <= q_len and self.prefilling_press is not None:
            return self.prefilling_press.forward_hook(module, input, kwargs, output)
        if self.decoding_press is not None:
            return self.decoding_press.forward_hook(module, input, kwargs, output)
        return output

    @contextmanager
    def __call__(self, model):
        try:
            with super().__call__(model):
                yield
        finally:
            if self.decoding_press is not None:
                self.decoding_press.reset()


# ===========================================================================
# Post-RoPE query reconstruction (core/collector.py:135-201)
# ===========================================================================
def recompute_post_rope_queries(attn_module, hidden_states, position_ids, position_embeddings=None):
    """q = RoPE(q_proj(h)) for the given absolute positions; (B, Hq, q_len, d) or None."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    bsz, q_len, _ = hidden_states.shape
    if not hasattr(attn_module, "q_proj"):
        return None
    cfg = attn_module.config
    num_heads = getattr(attn_module, "num_heads", cfg.num_attention_heads)
    head_dim = getattr(attn_module, "head_dim", cfg.hidden_size // cfg.num_attention_heads)
    q = attn_module.q_proj(hidden_states).view(bsz, q_len, num_heads, head_dim)
    if hasattr(attn_module, "q_norm"):
        q = attn_module.q_norm(q)
    q = q.transpose(1, 2)
    if position_embeddings is not None:
        cos, sin = position_embeddings
        q, _ = apply_rotary_pos_emb(q, q, cos, sin)
    else:
        rotary_emb = getattr(attn_module, "rotary_emb", None)
        if rotary_emb is None:
            return None
        if position_ids is None:
            position_ids = torch.arange(q_len, device=q.device, dtype=torch.long)[None].expand(bsz, -1)
        try:
            cos, sin = rotary_emb(q, position_ids)
            q, _ = apply_rotary_pos_emb(q, q, cos, sin)
        except (TypeError, ValueError):
            return None
    return q.detach()


# ===========================================================================
# CORE presses (core/kvpress_adapter.py)
# ===========================================================================
@dataclass
class COREScorerPress(ScorerPress):
    """CORE scorer (``kvpress_adapter.py:130-811``): 14-D token features and the
    per-layer indexer MLP, computed by the CUDA library."""

    indexer: object = None
    feature_extractor: Optional[FeatureGeometry] = None
    student_temp: float = 1.0
    scoring_layer_idx: Optional[int] = None
    scoring_stride: int = 1
    use_indexer_stack: bool = False
    n_sink_protect: int = 0
    recency_alpha: float = 0.0
    recency_window: int = 64
    span_block_size: int = 1
    span_pool_beta: float = 5.0
    span_selection_mode: str = "tokenwise"
    coverage_fraction: float = 0.25
    query_feature_weight: float = 0.0
    lexical_overlap_weight: float = 0.0
    identifier_lexical_weight: float = 0.0
    identifier_min_match_tokens: int = 20
    identifier_context_skip: int = 64
    identifier_span_size: int = 32
    protect_query_tokens: bool = False
    query_aware_prefill: bool = False
    prefill_qk_scope: str = "all"
    capture_diagnostics: bool = False
    _token_ids: Optional[torch.Tensor] = field(default=None, init=False, repr=False)
    _query_start: Optional[int] = field(default=None, init=False, repr=False)

    def __post_init__(self):
        super().__post_init__()
        if self.feature_extractor is None:
            raise ValueError("feature_extractor must be provided")
        self._cached_kept_indices = None
        self._cached_scores = None
        self._cached_memory_scores = None
        self._latest_query_feature = None
        self._cached_original_seq_len = 0
        self.cache_metadata = CacheMetadata()
        self.diagnostic_keep_indices: dict = {}
        self.diagnostic_scores: dict = {}
        self.diagnostic_features: dict = {}
        self._weights: dict = {}

    # ---- configuration / per-sequence state ----
    def post_init_from_model(self, model):
        device = next(model.parameters()).device
        self._ensure_device(device)
        lm = model.model.language_model if hasattr(model.model, "language_model") else model.model
        n_model = len(lm.layers)
        expected = int(getattr(self.indexer, "n_layers", n_model))
        if self.use_indexer_stack and expected != n_model:
            raise ValueError(f"CORE checkpoint/model layer mismatch: checkpoint has {expected} "
                             f"indexer layers, model has {n_model}.")
        if self.scoring_layer_idx is None:
            self.scoring_layer_idx = -1 if self.scoring_stride <= 1 else 0
        if self.scoring_stride > 1 and self.scoring_layer_idx >= 0:
            self.scoring_layer_idx = self.scoring_layer_idx // self.scoring_stride * self.scoring_stride

    def _ensure_device(self, device):
        device = torch.device(device)
        if device.type != "cuda":
            return
        fe = self.feature_extractor
        if isinstance(fe, FeatureGeometry) and fe.weight.device != device:
            fe.to(device)
        if isinstance(self.indexer, IndexerStack):
            first = self.indexer.modules[0][0]
            if first.device != device:
                self.indexer.to(device)
                self._weights.clear()

    def set_token_ids(self, token_ids, special_token_ids=None):
        self._token_ids = token_ids.detach()
        self.cache_metadata.record(token_ids, torch.arange(token_ids.shape[1], device=token_ids.device)[None])
        if special_token_ids is not None and isinstance(self.feature_extractor, FeatureGeometry):
            self.feature_extractor.config.special_token_ids = tuple(int(x) for x in special_token_ids)

    def set_query_boundary(self, query_start: int):
        self._query_start = int(query_start)

    def record_input_tokens(self, input_ids, position_ids=None):
        self.cache_metadata.record(input_ids, position_ids)

    def retain_metadata(self, layer_idx, indices):
        self.cache_metadata.retain(layer_idx, indices)

    def reset_cache(self):
        self._cached_kept_indices = None
        self._cached_scores = None
        self._cached_memory_scores = None
        self._latest_query_feature = None
        self._cached_original_seq_len = 0
        self._token_ids = None
        self.cache_metadata.reset()
        self._query_start = None
        self.diagnostic_keep_indices.clear()
        self.diagnostic_scores.clear()
        self.diagnostic_features.clear()

    # ---- weights in kernel formats, prepared once per layer ----
    def layer_weights(self, layer_idx: int, device) -> engine.LayerWeights:
        key = (int(layer_idx), str(device))
        lw = self._weights.get(key)
        if lw is None:
            fe = self.feature_extractor
            cfg = fe.config
            if self.use_indexer_stack:
                mlp = self.indexer.params(layer_idx)
            else:
                mlp = self.indexer.params(0)
            lw = engine.LayerWeights.prepare(
                geometry=fe.weight[int(layer_idx)], prototypes=fe.prototypes_for(layer_idx),
                hadamard=fe.hadamard, mlp_params=mlp, n_kv_heads=int(cfg.n_kv_heads),
                n_q_heads=int(cfg.n_q_heads), head_dim=int(cfg.head_dim), device=device)
            self._weights[key] = lw
        return lw

    def _check_policy(self):
        if (int(self.span_block_size) > 1 or self.query_feature_weight != 0.0
                or self.lexical_overlap_weight != 0.0 or self.protect_query_tokens):
            raise NotImplementedError(
                "core_b200 implements the tokenwise selection policy only "
                "(span/lexical/query-feature adjustments are not supported)")
        cfg = self.feature_extractor.config
        if getattr(cfg, "qk_primary_mode", "attention_advantage") != "attention_advantage":
            raise NotImplementedError("qk_primary_mode must be 'attention_advantage'")
        if not getattr(cfg, "center_prototype_features", True):
            raise NotImplementedError("center_prototype_features=False is not supported")

    # ---- queries of the scoring window ----
    def _scoring_queries(self, module, hidden_states, keys, is_prefill, kwargs):
        """Post-RoPE queries (B, Hq, nq, d) as ``_compute_scores_from_features``
        selects them (kvpress_adapter.py:357-519), plus an optional row LSE."""
        B, _, L, _ = keys.shape
        lse = None
        if is_prefill:
            q = getattr(module, "_core_cached_query_states", None)
            if q is None:
                q = recompute_post_rope_queries(module, hidden_states, kwargs.get("position_ids"),
                                                kwargs.get("position_embeddings"))
            if q is None or q.shape[-2] == 0:
                raise RuntimeError("CORE failed to compute prefill QK relation features: no "
                                   "post-RoPE queries (set _core_cached_query_states or q_proj)")
            if q.ndim == 3:
                q = q[None]
            query_start = 0
            if self.prefill_qk_scope == "question":
                if self._query_start is None:
                    raise RuntimeError("CORE prefill_qk_scope='question' requires set_query_boundary() "
                                       "before prefill.")
                query_start = int(self._query_start)
                if not 0 <= query_start < q.shape[2]:
                    raise RuntimeError(f"Invalid CORE query boundary: query_start={query_start}, "
                                       f"seq_len={q.shape[2]}")
                q = q[:, :, query_start:]
            elif self.prefill_qk_scope != "all":
                raise ValueError(f"prefill_qk_scope must be 'all' or 'question', got {self.prefill_qk_scope!r}")
            sl = getattr(module, "_core_cached_softmax_lse", None)
            if sl is not None and sl.ndim == 3:
                sl = sl[:, :, query_start:]
                if sl.shape[-1] == q.shape[2]:
                    lse = sl
        else:
            hs = hidden_states
            pos_ids = kwargs.get("position_ids")
            pos_emb = kwargs.get("position_embeddings")
            if hs.shape[1] > 1 and kwargs.get("cache_position") is not None:
                cur = kwargs.get("position_ids")
                end = int(cur[0, -1].item()) if cur is not None else int(kwargs["cache_position"][-1].item())
                pos_ids = torch.arange(end - hs.shape[1] + 1, end + 1, device=hs.device,
                                       dtype=torch.long)[None]
                pos_emb = None
            q = getattr(module, "_core_cached_query_states", None)
            if q is None or q.shape[-2] != hs.shape[1]:
                q = recompute_post_rope_queries(module, hs, pos_ids, pos_emb)
            if q is None or q.shape[-2] == 0:
                raise RuntimeError("CORE failed to reconstruct decode QK features; refusing to "
                                   "replace the paper features with zeros")
            if q.ndim == 3:
                q = q[None]
        if q.shape[0] != B:
            q = q.expand(B, -1, -1, -1)
        return q.to(engine.cache_dtype(keys.dtype)).contiguous(), lse

    def _special_mask(self, ids):
        fe = self.feature_extractor
        sp = tuple(getattr(fe.config, "special_token_ids", ()) or ())
        if not sp or ids is None:
            return None
        t = torch.tensor(sp, device=ids.device, dtype=ids.dtype)
        return torch.isin(ids, t)

    def _scores_and_features(self, module, hidden_states, keys, values, kwargs, layer_idx):
        """Calibrated scores (B, L) and features (B, L, 14) on the CUDA path."""
        self._check_policy()
        B, hkv, L, d = keys.shape
        is_prefill = hidden_states.shape[1] >= L
        positions, ids, original_length = self.cache_metadata.align(layer_idx, B, L, keys.device)
        q, lse = self._scoring_queries(module, hidden_states, keys, is_prefill, kwargs)
        cfg = self.feature_extractor.config
        lw = self.layer_weights(layer_idx, keys.device)
        dt = engine.cache_dtype(keys.dtype)
        k = keys.to(dt).contiguous()
        v = values.to(dt).contiguous()
        feats = torch.empty(B, L, 14, dtype=torch.float32, device=keys.device)
        ops.qk_features(q, k, topk_qk=int(cfg.topk_qk), n_recent_queries=int(cfg.n_recent_queries),
                        lse=lse, features=feats)
        ops.coverage_features(k, lw.geometry_ext, lw.prototypes,
                              shrinkage_rho=float(cfg.shrinkage_rho), features=feats, col0=6)
        scores = ops.indexer_scores(v, positions, feats, lw.mlp, original_length=int(original_length),
                                    is_prefill=is_prefill, n_sink=int(cfg.n_sink),
                                    special=self._special_mask(ids))
        self._latest_query_feature = feats[:, :, 3]
        if self.capture_diagnostics:
            self.diagnostic_features[int(layer_idx)] = feats[0].detach().float().cpu()
        return scores, feats

    def _compute_scores_from_features(self, module, hidden_states, keys, values, attentions,
                                      is_prefill, kwargs=None, layer_idx=0):
        """(B, Hkv, L) calibrated scores broadcast over KV heads (kvpress_adapter.py:312-558)."""
        scores, _ = self._scores_and_features(module, hidden_states, keys, values, kwargs or {},
                                              layer_idx)
        return scores[:, None, :].expand(-1, keys.shape[1], -1).contiguous()

    def _is_scoring_layer(self, layer_idx):
        if self.scoring_stride > 1 and (self.scoring_layer_idx or 0) >= 0:
            return layer_idx is None or layer_idx % self.scoring_stride == \
                (self.scoring_layer_idx or 0) % self.scoring_stride
        return self.scoring_layer_idx in (-1, None) or layer_idx == self.scoring_layer_idx \
            or layer_idx is None

    def _recency(self, scores: torch.Tensor) -> torch.Tensor:
        seq_len = scores.shape[-1]
        if self.recency_alpha > 0.0 and seq_len > 1:
            pos = torch.arange(seq_len, device=scores.device, dtype=scores.dtype)
            bonus = self.recency_alpha * torch.exp(-(seq_len - 1 - pos) / max(1, self.recency_window))
            scores = scores + bonus.view(*([1] * (scores.ndim - 1)), -1)
        return scores

    @torch.no_grad()
    def score(self, module, hidden_states, keys, values, attentions, kwargs):
        """Selection scores (B, Hkv, L) with sinks saturated (kvpress_adapter.py:690-797)."""
        self._ensure_device(hidden_states.device)
        batch_size, num_kv_heads, seq_len, _ = keys.shape
        is_prefill = hidden_states.shape[1] >= seq_len
        layer_idx = getattr(module, "layer_idx", None)
        if seq_len != self._cached_original_seq_len:
            self._cached_kept_indices = None
            self._cached_scores = None
            self._cached_memory_scores = None
            self._cached_original_seq_len = seq_len
        if not self._is_scoring_layer(layer_idx) and self._cached_scores is not None:
            return self._cached_scores.to(device=keys.device, dtype=keys.dtype).unsqueeze(1) \
                .expand(-1, num_kv_heads, -1).contiguous()
        scores = self._compute_scores_from_features(module, hidden_states, keys, values, attentions,
                                                    is_prefill, kwargs,
                                                    layer_idx=layer_idx if layer_idx is not None else 0)
        scores = self._recency(scores)
        calibrated = scores
        n_kept = max(min(self.n_sink_protect, seq_len), int(seq_len * (1 - self.compression_ratio)))
        if 0 < self.n_sink_protect < seq_len:
            scores = scores.clone()
            scores[:, :, : self.n_sink_protect] = scores.max().detach() + 1.0
        if 0 < n_kept < seq_len:
            self._cached_scores = scores[:, 0].detach().clone()
            self._cached_memory_scores = calibrated[:, 0].detach().clone()
            if self.capture_diagnostics:
                dl = int(layer_idx if layer_idx is not None else -1)
                self.diagnostic_scores[dl] = calibrated[:, 0].detach().float().cpu()
                self._cached_kept_indices = scores[:, 0].topk(n_kept, dim=-1).indices
                self.diagnostic_keep_indices[dl] = self._cached_kept_indices.detach().cpu()
        return scores

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        """Per-token Top-B and gather (kvpress_adapter.py:299-310)."""
        if self.compression_ratio == 0:
            return keys, values
        scores = self.score(module, hidden_states, keys, values, attentions, kwargs)
        count = max(min(self.n_sink_protect, keys.shape[2]), int(keys.shape[2] * (1 - self.compression_ratio)))
        if count >= keys.shape[2]:
            self.cache_metadata.align(int(module.layer_idx), keys.shape[0], keys.shape[2], keys.device)
            return keys, values
        keep, _ = ops.topb_select(scores[:, 0].float(), count, 0)
        self.cache_metadata.align(int(module.layer_idx), keys.shape[0], keys.shape[2], keys.device)
        self.retain_metadata(int(module.layer_idx), keep)
        return ops.compact_kv(keys.contiguous(), values.contiguous(), keep)


@dataclass
class COREMemoryPress(BasePress):
    """Eviction with latent-memory writing and gated readout (kvpress_adapter.py:814-1382)."""

    base_press: COREScorerPress = None  # type: ignore[assignment]
    memory_module: Optional[MemoryStack] = None
    memory_decay: float = 0.9
    memory_write_eta: float = 1.0
    memory_uniform_fraction: float = 0.0
    enable_memory_writing: bool = True
    memory_query_space: str = "post_rope_q"
    memory_value_space: str = "pre_o_proj"
    memory_gate_override: Optional[float] = None
    query_aware_prefill: bool = False
    requires_decoding_hook: bool = field(default=True, init=False, repr=False)

    def __post_init__(self):
        assert self.base_press is not None, "base_press (COREScorerPress) is required"
        self._M: dict = {}
        self._b: dict = {}
        self._Z: dict = {}
        self._folded_theta: dict = {}
        self._folded_o_proj: dict = {}
        self._readout_weights: dict = {}

    @property
    def compression_ratio(self) -> float:
        return self.base_press.compression_ratio

    @compression_ratio.setter
    def compression_ratio(self, value: float) -> None:
        self.base_press.compression_ratio = value

    @property
    def student_temp(self) -> float:
        return self.base_press.student_temp

    def post_init_from_model(self, model):
        self.base_press.post_init_from_model(model)

    def set_token_ids(self, token_ids, special_token_ids=None):
        self.base_press.set_token_ids(token_ids, special_token_ids)

    def record_input_tokens(self, input_ids, position_ids=None):
        self.base_press.record_input_tokens(input_ids, position_ids)

    def set_query_boundary(self, query_start: int):
        self.base_press.set_query_boundary(query_start)

    def _ensure_device(self, device):
        self.base_press._ensure_device(device)
        if self.memory_module is not None and torch.device(device).type == "cuda":
            if self.memory_module.modules[0][0].device != torch.device(device):
                self.memory_module.to(device)
                self._folded_theta.clear()
                self._readout_weights.clear()

    def reset_cache(self):
        self.base_press.reset_cache()
        self._M.clear(); self._b.clear(); self._Z.clear()

    def reset_memory(self, layer_idx: Optional[int] = None):
        if layer_idx is None:
            self._M.clear(); self._b.clear(); self._Z.clear()
        else:
            self._M.pop(layer_idx, None); self._b.pop(layer_idx, None); self._Z.pop(layer_idx, None)

    def _check_spaces(self):
        if self.memory_value_space != "pre_o_proj":
            raise ValueError(f"Unknown or unsupported CORE memory_value_space={self.memory_value_space!r}")
        if self.memory_query_space != "post_rope_q":
            raise ValueError(f"Unknown or unsupported CORE memory_query_space={self.memory_query_space!r}")
        if self.memory_uniform_fraction != 0.0:
            raise NotImplementedError("memory_uniform_fraction != 0 is not supported by core_b200")

    def _theta_split(self, layer_idx, num_kv_heads, num_groups, head_dim, device, dtype):
        """Folded memory-write projection in the form caches of ``dtype`` take:
        bf16 hi/lo terms, or the f32 fold itself for f32 caches."""
        f32 = engine.cache_dtype(dtype) == torch.float32
        key = (self.memory_module.module_index(layer_idx), num_kv_heads, num_groups, str(device),
               f32)
        ts = self._folded_theta.get(key)
        if ts is None:
            theta = self.memory_module.params(layer_idx)[0].to(device)
            fold = engine.fold_groups(theta, num_kv_heads, num_groups, head_dim)
            ts = fold if f32 else ops.split_bf16(fold, 2)
            self._folded_theta[key] = ts
        return ts

    def _state(self, layer_idx, B, d_mem, kvw, device):
        M = self._M.get(layer_idx)
        if M is None or M.shape != (B, d_mem, kvw) or M.device != torch.device(device):
            self._M[layer_idx] = torch.zeros(B, d_mem, kvw, device=device)
            self._b[layer_idx] = torch.zeros(B, d_mem, device=device)
            self._Z[layer_idx] = torch.zeros(B, device=device)
        Z = self._Z.get(layer_idx)
        if Z is None or Z.shape != (B,):
            self._Z[layer_idx] = torch.zeros(B, device=device)
        return self._M[layer_idx], self._b[layer_idx], self._Z[layer_idx]

    @torch.no_grad()
    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        """Select retained tokens, write the evicted ones to memory, prune K/V
        (kvpress_adapter.py:968-1210)."""
        self._ensure_device(hidden_states.device)
        if self.compression_ratio == 0:
            return keys, values
        bp = self.base_press
        layer_idx = int(getattr(module, "layer_idx", 0))
        bsz, num_kv_heads, k_len, head_dim = keys.shape
        num_groups = bp.feature_extractor.n_q_heads // num_kv_heads
        if k_len != bp._cached_original_seq_len:
            bp._cached_scores = None
            bp._cached_memory_scores = None
            bp._cached_original_seq_len = k_len
        n_sink = int(bp.n_sink_protect)
        n_kept = engine.n_kept_for(k_len, self.compression_ratio, n_sink)
        if n_kept >= k_len:
            bp.cache_metadata.align(layer_idx, bsz, k_len, keys.device)
            return keys, values
        write = self.enable_memory_writing and self.memory_module is not None
        if write:
            self._check_spaces()
        dt = engine.cache_dtype(keys.dtype)
        k = keys.to(dt).contiguous()
        v = values.to(dt).contiguous()
        state = None
        ts = None
        if write:
            d_mem = self.memory_module.d_mem
            M, b, Z = self._state(layer_idx, bsz, d_mem, num_kv_heads * head_dim, keys.device)
            state = engine.MemoryState(M, b, Z)
            ts = self._theta_split(layer_idx, num_kv_heads, num_groups, head_dim, keys.device,
                                   keys.dtype)
        reuse = (not bp._is_scoring_layer(layer_idx)) and bp._cached_memory_scores is not None
        if reuse or bp.recency_alpha > 0.0:
            # scores first (reused across layers, or adjusted by the recency bonus)
            if reuse:
                bp.cache_metadata.align(layer_idx, bsz, k_len, keys.device)
                calibrated = bp._cached_memory_scores
            else:
                calibrated = bp._recency(bp._scores_and_features(module, hidden_states, keys,
                                                                 values, kwargs or {}, layer_idx)[0])
            keep, evict = ops.topb_select(calibrated, n_kept, n_sink)
            if write and evict.shape[1] > 0:
                ops.memory_write(k, v, calibrated, evict, ts, state.M, state.b, state.Z,
                                 gamma=self.memory_decay, eta=self.memory_write_eta,
                                 student_temp=self.student_temp)
            out_k, out_v = ops.compact_kv(k, v, keep)
        else:
            bp._check_policy()
            is_prefill = hidden_states.shape[1] >= k_len
            positions, ids, original_length = bp.cache_metadata.align(layer_idx, bsz, k_len,
                                                                       keys.device)
            q, lse = bp._scoring_queries(module, hidden_states, keys, is_prefill, kwargs or {})
            cfg = bp.feature_extractor.config
            lw = bp.layer_weights(layer_idx, keys.device)
            if dt == torch.float32:
                lw.theta_fold = ts
            else:
                lw.theta_split = ts
            out = engine.compress_layer(
                q, k, v, lw, n_kept=n_kept, positions=positions, original_length=int(original_length),
                is_prefill=is_prefill, n_sink=n_sink, topk_qk=int(cfg.topk_qk),
                n_recent_queries=int(cfg.n_recent_queries), shrinkage_rho=float(cfg.shrinkage_rho),
                memory=state, gamma=self.memory_decay, eta=self.memory_write_eta,
                student_temp=self.student_temp, special=bp._special_mask(ids), lse=lse)
            calibrated, keep, out_k, out_v = out["scores"], out["keep"], out["keys"], out["values"]
            bp._latest_query_feature = out["features"][:, :, 3]
            if bp.capture_diagnostics:
                bp.diagnostic_features[layer_idx] = out["features"][0].detach().float().cpu()
        bp._cached_memory_scores = calibrated
        sel = calibrated.clone()
        if 0 < n_sink < k_len:
            sel[:, :n_sink] = sel.max() + 1.0
        bp._cached_scores = sel
        if bp.capture_diagnostics:
            bp.diagnostic_scores[layer_idx] = calibrated.detach().float().cpu()
            bp.diagnostic_keep_indices[layer_idx] = keep.detach().long().cpu()
        bp.retain_metadata(layer_idx, keep)
        return out_k.to(keys.dtype), out_v.to(values.dtype)

    def _readout_params(self, module, layer_idx, num_kv_heads, num_groups, head_dim, device):
        key = (layer_idx, str(device))
        rp = self._readout_weights.get(key)
        if rp is None:
            th, gw1, gb1, gw2, gb2 = self.memory_module.params(layer_idx)
            o_fold = engine.fold_groups(module.o_proj.weight.to(device), num_kv_heads, num_groups,
                                        head_dim)
            rp = (th.to(device).float().contiguous(),
                  (gw1.to(device).float().contiguous(), gb1.to(device).float().contiguous(),
                   gw2.to(device).float().reshape(-1).contiguous(),
                   gb2.to(device).float().reshape(-1).contiguous()),
                  o_fold)
            self._readout_weights[key] = rp
        return rp

    @torch.no_grad()
    def apply_memory_readout(self, module, kwargs, output):
        """attention output += folded o_proj(g(q) m(q)) (kvpress_adapter.py:1212-1352)."""
        if not self.enable_memory_writing or self.memory_module is None:
            return output
        layer_idx = int(getattr(module, "layer_idx", 0))
        M = self._M.get(layer_idx)
        b = self._b.get(layer_idx)
        if M is None or b is None:
            return output
        self._check_spaces()
        hidden = kwargs["hidden_states"]
        batch_size, q_len, _ = hidden.shape
        q = getattr(module, "_core_cached_query_states", None)
        if q is None or q.ndim != 4 or q.shape[0] != batch_size or q.shape[-2] != q_len:
            q = recompute_post_rope_queries(module, hidden, kwargs.get("position_ids"),
                                            kwargs.get("position_embeddings"))
        if q is None:
            raise RuntimeError("CORE memory readout could not reconstruct post-RoPE queries; "
                               "refusing to mix hidden-state queries with post-RoPE memory keys.")
        n_q_heads = int(module.config.num_attention_heads)
        n_kv_heads = int(module.config.num_key_value_heads)
        head_dim = q.shape[-1]
        theta, gate, o_fold = self._readout_params(module, layer_idx, n_kv_heads,
                                                   n_q_heads // n_kv_heads, head_dim, hidden.device)
        attn = output[0].to(engine.cache_dtype(output[0].dtype)).contiguous().clone()
        ops.memory_readout(q, theta, gate, M, b, o_fold, attn, n_kv_heads=n_kv_heads,
                           gate_override=self.memory_gate_override)
        new_attn = attn.to(output[0].dtype)
        if isinstance(output, (list, tuple)):
            return type(output)([new_attn] + list(output[1:]))
        return new_attn

    def forward_hook(self, module, input, kwargs, output):
        q_len = kwargs["hidden_states"].shape[1]
        if kwargs["cache_position"][-1] <= q_len:
            return super().forward_hook(module, input, kwargs, output)
        return self.apply_memory_readout(module, kwargs, output)


@dataclass
class COREIndexerPress(COREScorerPress):
    """Backward-compatible press with an optional absolute budget (kvpress_adapter.py:1385-1436)."""

    budget: Optional[int] = None

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        if keys.shape[2] <= 1:
            return keys, values
        self._ensure_device(hidden_states.device)
        seq_len = keys.shape[2]
        if self.budget is not None:
            n_kept = max(1, min(self.n_sink_protect, seq_len), min(self.budget, seq_len))
        else:
            n_kept = max(1, min(self.n_sink_protect, seq_len), int(seq_len * (1 - self.compression_ratio)))
        if n_kept >= seq_len:
            return keys, values
        original = self.compression_ratio
        self.compression_ratio = 1.0 - (n_kept / seq_len)
        try:
            return super().compress(module, hidden_states, keys, values, attentions, kwargs)
        finally:
            self.compression_ratio = original


@dataclass
class COREDecodingPress(DecodingPress):
    """DecodingPress accepting the memory press (kvpress_adapter.py:92-122)."""

    hidden_states_buffer_size: Optional[int] = None

    def __post_init__(self):
        assert hasattr(self.base_press, "compress"), "CORE decoding press requires a compress-capable base press"
        self.hidden_states_buffer = defaultdict(list)
        self.layer_step_counts = defaultdict(int)
        assert self.compression_interval > 0
        assert self.target_size > 0
        if self.hidden_states_buffer_size is None:
            self.hidden_states_buffer_size = self.compression_interval
        if self.hidden_states_buffer_size < self.compression_interval:
            raise ValueError("CORE requires queries from the entire compression interval; "
                             "hidden_states_buffer_size must be >= compression_interval")


@dataclass
class COREPrefillDecodingPress(PrefillDecodingPress):
    """CORE token metadata and prefill/decode budgets (kvpress_adapter.py:56-89)."""

    query_aware_prefill: bool = False
    match_prefill_budget: bool = True

    def begin_sequence(self, context_length):
        if self.match_prefill_budget:
            self.decoding_press.target_size = retained_budget(
                context_length, self.prefilling_press.compression_ratio)

    def set_token_ids(self, token_ids, special_token_ids=None):
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "set_token_ids"):
            self.prefilling_press.set_token_ids(token_ids, special_token_ids)

    def record_input_tokens(self, input_ids, position_ids=None):
        self.prefilling_press.record_input_tokens(input_ids, position_ids)

    def set_query_boundary(self, query_start: int):
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "set_query_boundary"):
            self.prefilling_press.set_query_boundary(query_start)

    def reset_cache(self):
        if self.decoding_press is not None:
            self.decoding_press.reset()
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "reset_cache"):
            self.prefilling_press.reset_cache()


# ===========================================================================
# Factories (kvpress_adapter.py:1444-1832)
# ===========================================================================
def _check_compression_ratio(requested, cfg, checkpoint_path) -> float:
    train_cr = float(cfg.compression_ratio)
    effective = train_cr if requested is None else float(requested)
    if not 0.0 < effective < 1.0:
        raise ValueError(f"compression_ratio must lie in (0, 1), received {effective}")
    return effective


def _apply_protection_fields(press: COREScorerPress, cfg) -> None:
    press.n_sink_protect = cfg.get("n_sink_protect", 0)
    press.recency_alpha = cfg.get("recency_alpha", 0.0)
    press.recency_window = cfg.get("recency_window", 64)
    press.scoring_stride = cfg.get("scoring_stride", 1)
    press.span_block_size = cfg.get("span_block_size", 1)
    press.span_pool_beta = cfg.get("span_pool_beta", 5.0)
    press.span_selection_mode = cfg.get("span_selection_mode", "sliding_max")
    press.coverage_fraction = cfg.get("coverage_fraction", 0.25)
    press.query_feature_weight = cfg.get("query_feature_weight", 0.0)
    press.lexical_overlap_weight = cfg.get("lexical_overlap_weight", 0.0)
    press.identifier_lexical_weight = cfg.get("identifier_lexical_weight", 0.0)
    press.identifier_min_match_tokens = cfg.get("identifier_min_match_tokens", 20)
    press.identifier_context_skip = cfg.get("identifier_context_skip", 64)
    press.identifier_span_size = cfg.get("identifier_span_size", 32)
    press.protect_query_tokens = cfg.get("protect_query_tokens", False)
    press.prefill_qk_scope = cfg.get("prefill_qk_scope", "all")


def _load(checkpoint_path, device):
    parts = load_checkpoint(checkpoint_path, device=device)
    return parts["indexer"], parts["config"], parts["geometry"], parts["use_stack"], parts["memory"]


def _required_memory(memory, cfg, checkpoint_path):
    if memory is None:
        raise ValueError("CORE memory evaluation requires a joint checkpoint containing a compatible "
                         f"memory_state_dict. Checkpoint: {checkpoint_path}")
    if cfg.n_layers is not None and int(memory.n_layers) != int(cfg.n_layers):
        raise ValueError(f"CORE checkpoint memory/indexer layer mismatch: memory has "
                         f"{memory.n_layers} layers, config has {cfg.n_layers}.")
    width = cfg.n_q_heads * cfg.head_dim if cfg.n_q_heads and cfg.head_dim else cfg.hidden_size
    if width is not None and int(memory.d_model) != int(width):
        raise ValueError(f"CORE checkpoint memory query-width mismatch: memory has "
                         f"{memory.d_model}, expected H_q * d_head = {width}.")
    return memory


def load_core_scorer_press(checkpoint_path: str, device: str = "cuda:0",
                           compression_ratio: float = 0.5) -> COREScorerPress:
    indexer, cfg, fe, use_stack, _ = _load(checkpoint_path, device)
    press = COREScorerPress(indexer=indexer, feature_extractor=fe,
                            compression_ratio=_check_compression_ratio(compression_ratio, cfg, checkpoint_path),
                            student_temp=cfg.student_temp, use_indexer_stack=use_stack)
    _apply_protection_fields(press, cfg)
    return press


def load_core_indexer_press(checkpoint_path: str, device: str = "cuda:0",
                            compression_ratio: Optional[float] = None) -> COREIndexerPress:
    indexer, cfg, fe, use_stack, _ = _load(checkpoint_path, device)
    press = COREIndexerPress(indexer=indexer, feature_extractor=fe,
                             compression_ratio=_check_compression_ratio(compression_ratio, cfg, checkpoint_path),
                             budget=cfg.budget, student_temp=cfg.student_temp, use_indexer_stack=use_stack)
    _apply_protection_fields(press, cfg)
    return press


def _memory_press(base, memory, cfg):
    return COREMemoryPress(base_press=base, memory_module=memory, memory_decay=cfg.memory_decay,
                           memory_write_eta=cfg.memory_write_eta,
                           memory_uniform_fraction=cfg.memory_uniform_fraction,
                           enable_memory_writing=cfg.enable_memory_writing,
                           memory_query_space=cfg.memory_query_space,
                           memory_value_space=cfg.memory_value_space)


def load_core_memory_press(checkpoint_path: str, device: str = "cuda:0",
                           compression_ratio: Optional[float] = None) -> COREMemoryPress:
    indexer, cfg, fe, use_stack, memory = _load(checkpoint_path, device)
    base = COREScorerPress(indexer=indexer, feature_extractor=fe,
                           compression_ratio=_check_compression_ratio(compression_ratio, cfg, checkpoint_path),
                           student_temp=cfg.student_temp, use_indexer_stack=use_stack)
    _apply_protection_fields(base, cfg)
    return _memory_press(base, _required_memory(memory, cfg, checkpoint_path), cfg)


def load_core_prefill_decoding_press(checkpoint_path: str, device: str = "cuda:0",
                                     compression_ratio: Optional[float] = None,
                                     decoding_compression_interval: int = 128,
                                     decoding_target_size: Optional[int] = None,
                                     decoding_hidden_states_buffer_size: Optional[int] = None
                                     ) -> COREPrefillDecodingPress:
    indexer, cfg, fe, use_stack, memory = _load(checkpoint_path, device)
    base = COREScorerPress(indexer=indexer, feature_extractor=fe,
                           compression_ratio=_check_compression_ratio(compression_ratio, cfg, checkpoint_path),
                           student_temp=cfg.student_temp, use_indexer_stack=use_stack)
    _apply_protection_fields(base, cfg)
    shared = _memory_press(base, _required_memory(memory, cfg, checkpoint_path), cfg)
    decoding = COREDecodingPress(base_press=shared, compression_interval=decoding_compression_interval,
                                 target_size=decoding_target_size or 1,
                                 hidden_states_buffer_size=decoding_hidden_states_buffer_size)
    return COREPrefillDecodingPress(match_prefill_budget=decoding_target_size is None,
                                    prefilling_press=shared, decoding_press=decoding,
                                    query_aware_prefill=False)


PRESS_REGISTRY = {"core_full": load_core_prefill_decoding_press,
                  "core_memory": load_core_memory_press,
                  "core_indexer": load_core_indexer_press}
