"""KVPress-compatible CORE presses running on the B200 CUDA library.

The classes keep the reference's public surface -- class names, dataclass
fields, methods, factories, the ``"core_full"`` registry key and the forward
hook contract ``compress(module, hidden_states, keys, values, attentions,
kwargs) -> (keys, values)`` (kvpress/kvpress/presses/base_press.py:55-93) --
so that an evaluator which builds the reference press can build this one
instead (core/kvpress_adapter.py:56-1832 and the kvpress base presses it
extends).

What runs where:
  * the compression step of one layer (features, indexer scores, Top-B with
    sinks, memory write, retained-KV gather) is one call into the CUDA
    library (``engine.compress_layer``);
  * the memory readout of a decode step is one library call
    (``ops.memory_readout``);
  * decode-time queries are rebuilt from a device window of buffered hidden
    states by the q_proj GEMM plus the library's RoPE kernel
    (``queries.post_rope_queries``);
  * the original-position journal of the compacted cache stays on the device
    (``journal.CacheMetadata``).
The host side is a small state machine per press: which phase a forward is
in, when a decode interval is complete, which per-layer state to update.

Not thread-safe: one sequence per press instance, as in the reference.
"""

from __future__ import annotations

import logging
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Optional

import torch
from torch import nn

from . import engine, ops
from .checkpoint import FeatureGeometry, IndexerStack, MemoryStack, load_checkpoint
from .journal import CacheMetadata
from .queries import HiddenStateWindow, decode_positions, post_rope_queries

logger = logging.getLogger(__name__)

__all__ = ["BasePress", "ScorerPress", "DecodingPress", "PrefillDecodingPress", "CacheMetadata",
           "COREScorerPress", "COREMemoryPress", "COREIndexerPress", "COREDecodingPress",
           "COREPrefillDecodingPress", "retained_budget", "load_core_scorer_press",
           "load_core_indexer_press", "load_core_memory_press",
           "load_core_prefill_decoding_press", "PRESS_REGISTRY"]


def retained_budget(length: int, ratio: float, sinks: int = 4) -> int:
    """Tokens a sequence of ``length`` keeps at eviction ratio ``ratio``, never
    fewer than the sinks (core/paper_protocol.py:17-20)."""
    if length < 1 or not 0.0 <= ratio < 1.0:
        raise ValueError("retained_budget needs length >= 1 and 0 <= ratio < 1")
    return max(min(sinks, length), int(length * (1 - ratio)))


def ratio_for_kept_count(length: int, target: int) -> float:
    """An eviction ratio r with int(length * (1 - r)) == target (0 when nothing
    has to go).  The decoding press hands r to its base press, which keeps
    int(length * (1 - r)) tokens (kvpress decoding_press.py:203-245 searches
    for the same r by bisection).  The plain quotient is tried first; when
    floating point puts it one token short, the middle of the interval of
    valid ratios is exact."""
    if length <= target:
        return 0.0
    r = 1.0 - target / length
    if int(length * (1 - r)) == target:
        return r
    r = 1.0 - (target + 0.5) / length
    if int(length * (1 - r)) != target:
        logger.warning("no eviction ratio keeps exactly %d of %d tokens", target, length)
    return r


# ===========================================================================
# Hook plumbing
# ===========================================================================
def _is_quantized(cache) -> bool:
    try:
        from transformers.cache_utils import QuantizedCache
    except ImportError:  # pragma: no cover
        return False
    return isinstance(cache, QuantizedCache)


def read_cache_layer(cache, layer_idx: int):
    """(keys, values) of one cache layer, dequantized for a quantized cache
    (kvpress utils.py:98-114: the quantized part only)."""
    layer = cache.layers[layer_idx]
    if _is_quantized(cache):
        return layer._dequantize(layer._quantized_keys), layer._dequantize(layer._quantized_values)
    return layer.keys, layer.values


def write_cache_layer(cache, layer_idx: int, keys: torch.Tensor, values: torch.Tensor) -> None:
    """Store compressed keys/values back into the cache layer; a quantized
    cache re-quantizes them and empties its full-precision residual
    (kvpress base_press.py:146-155)."""
    layer = cache.layers[layer_idx]
    if _is_quantized(cache):
        layer._quantized_keys = layer._quantize(keys, axis=layer.axis_key)
        layer._quantized_values = layer._quantize(values, axis=layer.axis_value)
        layer.keys = keys.new_zeros(0)
        layer.values = values.new_zeros(0)
        layer.cumulative_length = keys.shape[2]
    else:
        layer.keys = keys
        layer.values = values


class _LastCachePosition:
    """The last entry of a forward's ``cache_position``.  Every layer of a
    model forward gets the same tensor, so its value is read from the device
    once per forward (and again only if the tensor is modified in place)."""

    def __init__(self):
        self._tensor = None
        self._version = -1
        self._value = 0

    def __call__(self, cache_position) -> int:
        if cache_position is not self._tensor or cache_position._version != self._version:
            self._value = int(cache_position[-1])
            self._tensor = cache_position
            self._version = cache_position._version
        return self._value


_LAST_POSITION = _LastCachePosition()


def _phase_is_prefill(kwargs, q_len: int) -> bool:
    """A forward is a prefill when its last cache position lies within its own
    length (kvpress base_press.py:135-138)."""
    return _LAST_POSITION(kwargs["cache_position"]) <= q_len


_TEMPORARIES = ("_core_cached_query_states", "_core_cached_key_states", "_core_cached_softmax_lse")


def _drop_temporaries(module, args, output):
    """Forget the per-forward tensors the CORE attention adapter attached to
    the module (kvpress base_press.py:198-204)."""
    for name in _TEMPORARIES:
        if hasattr(module, name):
            delattr(module, name)


def _language_model(model):
    return model.model.language_model if hasattr(model.model, "language_model") else model.model


@dataclass
class BasePress:
    """A press compresses a layer's cache from a forward hook on its attention
    module.  This base runs ``compress`` once per layer at prefill and leaves
    decode forwards alone (kvpress base_press.py:95-156)."""

    def post_init_from_model(self, model):
        pass

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        raise NotImplementedError(f"{type(self).__name__} must implement compress()")

    def _compress_cache_layer(self, module, hidden_states, kwargs, attentions) -> None:
        cache = kwargs["past_key_values"]
        keys, values = read_cache_layer(cache, module.layer_idx)
        keys, values = self.compress(module, hidden_states, keys, values, attentions, kwargs)
        write_cache_layer(cache, module.layer_idx, keys, values)

    def forward_hook(self, module: nn.Module, input, kwargs: dict, output):
        if _phase_is_prefill(kwargs, kwargs["hidden_states"].shape[1]):
            self._compress_cache_layer(module, kwargs["hidden_states"], kwargs, output[1])
        return output

    @contextmanager
    def __call__(self, model):
        """Hook every attention layer of ``model`` for the duration of the block."""
        self.post_init_from_model(model)
        handles = []
        try:
            lm = _language_model(model)
            for layer in lm.layers:
                attn = layer.self_attn
                attn.rotary_emb = lm.rotary_emb
                handles.append(attn.register_forward_hook(self.forward_hook, with_kwargs=True))
                handles.append(attn.register_forward_hook(_drop_temporaries, always_call=True))
            yield
        finally:
            for h in handles:
                h.remove()


@dataclass
class ScorerPress(BasePress):
    """A press that scores tokens and keeps the best (kvpress scorer_press.py)."""

    compression_ratio: float = 0.0

    def __post_init__(self):
        if not 0 <= self.compression_ratio < 1:
            raise ValueError("compression_ratio must lie in [0, 1)")

    def score(self, module, hidden_states, keys, values, attentions, kwargs):
        raise NotImplementedError(f"{type(self).__name__} must implement score()")


@dataclass
class DecodingPress(BasePress):
    """Recompress a layer's cache every ``compression_interval`` decode
    forwards, scoring with the hidden states buffered since the last
    compression (kvpress decoding_press.py:22-248).

    Per layer the press keeps a step counter and a ``HiddenStateWindow`` of
    the last ``hidden_states_buffer_size`` forwards.  A decode forward first
    applies the base press's memory readout (when it has one), then buffers
    its hidden states; when the interval is complete (or the forward alone
    reaches ``target_size`` tokens) the cache is compressed to
    ``target_size`` tokens with every buffered query, and the window is
    emptied.
    """

    base_press: BasePress = None  # type: ignore[assignment]
    compression_interval: int = 512
    target_size: int = 2048
    hidden_states_buffer_size: int = 256

    def __post_init__(self):
        if not (hasattr(self.base_press, "compress") and hasattr(self.base_press, "compression_ratio")):
            raise ValueError("DecodingPress needs a base press with compress() and compression_ratio")
        self._check_sizes()
        self.reset()

    def _check_sizes(self):
        if self.compression_interval <= 0:
            raise ValueError("compression_interval must be positive")
        if self.target_size <= 0:
            raise ValueError("target_size must be positive")

    def reset(self):
        """Drop the buffered hidden states and step counts of every layer."""
        self._windows: dict = {}
        self._steps: dict = {}

    # the reference's per-layer bookkeeping, readable for inspection
    @property
    def layer_step_counts(self) -> dict:
        return dict(self._steps)

    @property
    def hidden_states_buffer(self) -> dict:
        return {k: w.view() for k, w in self._windows.items() if w.n_entries}

    def _window(self, layer_idx: int) -> HiddenStateWindow:
        w = self._windows.get(layer_idx)
        if w is None:
            w = self._windows[layer_idx] = HiddenStateWindow(self.hidden_states_buffer_size)
        return w

    def post_init_from_model(self, model):
        self.base_press.post_init_from_model(model)

    def _resolve_target_size(self, kwargs) -> int:
        return self.target_size

    def _find_target_compression_ratio(self, q_len: int, target_tokens: int) -> float:
        return ratio_for_kept_count(q_len, target_tokens)

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        """Compress to ``target_size`` tokens through the base press, at the
        ratio that keeps exactly that many."""
        ratio = ratio_for_kept_count(keys.shape[2], self._resolve_target_size(kwargs))
        saved = self.base_press.compression_ratio
        self.base_press.compression_ratio = ratio
        try:
            return self.base_press.compress(module, hidden_states, keys, values, attentions, kwargs)
        finally:
            self.base_press.compression_ratio = saved

    def forward_hook(self, module: nn.Module, input, kwargs: dict, output):
        hs = kwargs["hidden_states"]
        if _phase_is_prefill(kwargs, hs.shape[1]):
            return output
        # memory written by earlier compressions is read before this step writes
        readout = getattr(self.base_press, "apply_memory_readout", None)
        if readout is not None:
            output = readout(module, kwargs, output)
        layer = module.layer_idx
        window = self._window(layer)
        window.append(hs)
        self._steps[layer] = self._steps.get(layer, 0) + 1
        due = (self._steps[layer] >= self.compression_interval
               or hs.shape[1] >= self._resolve_target_size(kwargs))
        if due:
            attn = output[1] if len(output) > 1 else None
            self._compress_cache_layer(module, window.view(), kwargs, attn)
            self._steps[layer] = 0
            window.clear()  # the cache no longer matches the buffered queries
        window.trim()
        return output

    @contextmanager
    def __call__(self, model):
        try:
            with super().__call__(model):
                yield
        finally:
            self.reset()


@dataclass
class PrefillDecodingPress(BasePress):
    """One press for both phases: prefill forwards go to ``prefilling_press``,
    decode forwards to ``decoding_press`` (kvpress prefill_decoding_press.py)."""

    prefilling_press: Optional[BasePress] = None
    decoding_press: Optional[DecodingPress] = None
    query_aware_prefill: bool = False

    def _target(self, kwargs, q_len: int):
        if self.prefilling_press is not None and _phase_is_prefill(kwargs, q_len):
            return self.prefilling_press
        return self.decoding_press

    def post_init_from_model(self, model):
        for p in (self.prefilling_press, self.decoding_press):
            if p is not None:
                p.post_init_from_model(model)

    def set_token_ids(self, token_ids, special_token_ids=None):
        fn = getattr(self.prefilling_press, "set_token_ids", None)
        if fn is not None:
            fn(token_ids, special_token_ids)

    def set_query_boundary(self, query_start: int):
        fn = getattr(self.prefilling_press, "set_query_boundary", None)
        if fn is not None:
            fn(query_start)

    def reset_cache(self):
        inner = [self.prefilling_press, getattr(self.decoding_press, "base_press", None)]
        for p in {id(p): p for p in inner if p is not None}.values():
            if hasattr(p, "reset_cache"):
                p.reset_cache()
        if self.decoding_press is not None:
            self.decoding_press.reset()

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        target = self._target(kwargs, hidden_states.shape[1])
        if target is None:
            return keys, values
        return target.compress(module, hidden_states, keys, values, attentions, kwargs)

    def forward_hook(self, module, input, kwargs, output):
        target = self._target(kwargs, kwargs["hidden_states"].shape[1])
        return output if target is None else target.forward_hook(module, input, kwargs, output)

    @contextmanager
    def __call__(self, model):
        try:
            with super().__call__(model):
                yield
        finally:
            if self.decoding_press is not None:
                self.decoding_press.reset()


# ===========================================================================
# CORE presses
# ===========================================================================
def _score_dtype(fe) -> torch.dtype:
    """Arithmetic of the features: the feature extractor's configured dtype
    (the reference casts Q, K and V to it before scoring,
    core/kvpress_adapter.py:334,420-470)."""
    name = str(getattr(getattr(fe, "config", None), "dtype", "bfloat16")).replace("torch.", "")
    if name in ("float32", "float"):
        return torch.float32
    if name in ("bfloat16",):
        return torch.bfloat16
    raise NotImplementedError(f"core_b200 scores in bfloat16 or float32, not {name}")


@dataclass
class _SelectionMemo:
    """Scores of the last scoring layer, reused by the layers that do not
    score (stride mode) and by the memory write; forgotten when the cache
    length changes (core/kvpress_adapter.py:735-797)."""

    seq_len: int = 0
    selection: Optional[torch.Tensor] = None   # (B, L), sinks saturated
    calibrated: Optional[torch.Tensor] = None  # (B, L), as the indexer produced them
    kept: Optional[torch.Tensor] = None        # (B, n_kept) top-k of selection (diagnostics)

    def follow(self, seq_len: int) -> None:
        if seq_len != self.seq_len:
            self.selection = self.calibrated = self.kept = None
            self.seq_len = seq_len


@dataclass
class COREScorerPress(ScorerPress):
    """CORE scorer (core/kvpress_adapter.py:130-811): 14-D token features and
    the per-layer indexer MLP, computed by the CUDA library."""

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
        self._memo = _SelectionMemo()
        self._latest_query_feature = None
        self.cache_metadata = CacheMetadata()
        self.diagnostic_keep_indices: dict = {}
        self.diagnostic_scores: dict = {}
        self.diagnostic_features: dict = {}
        self._weights: dict = {}

    # the reference's names for the memo's fields
    @property
    def _cached_scores(self):
        return self._memo.selection

    @_cached_scores.setter
    def _cached_scores(self, v):
        self._memo.selection = v

    @property
    def _cached_memory_scores(self):
        return self._memo.calibrated

    @_cached_memory_scores.setter
    def _cached_memory_scores(self, v):
        self._memo.calibrated = v

    @property
    def _cached_kept_indices(self):
        return self._memo.kept

    @property
    def _cached_original_seq_len(self):
        return self._memo.seq_len

    # ---- configuration and per-sequence state ----
    def post_init_from_model(self, model):
        self._ensure_device(next(model.parameters()).device)
        n_model = len(_language_model(model).layers)
        n_ckpt = int(getattr(self.indexer, "n_layers", n_model))
        if self.use_indexer_stack and n_ckpt != n_model:
            raise ValueError(f"CORE checkpoint/model layer mismatch: the checkpoint has {n_ckpt} "
                             f"indexer layers, the model {n_model}")
        want = getattr(getattr(self.feature_extractor, "config", None), "hidden_size", None)
        have = getattr(getattr(model, "config", None), "hidden_size", None)
        if want is not None and have is not None and int(want) != int(have):
            raise ValueError(f"CORE checkpoint/model hidden-size mismatch: {want} vs {have}")
        if self.scoring_layer_idx is None:
            self.scoring_layer_idx = 0 if self.scoring_stride > 1 else -1
        if self.scoring_stride > 1 and self.scoring_layer_idx >= 0:
            self.scoring_layer_idx -= self.scoring_layer_idx % self.scoring_stride

    def _ensure_device(self, device):
        device = torch.device(device)
        if device.type != "cuda":
            return
        fe = self.feature_extractor
        if isinstance(fe, FeatureGeometry) and fe.weight.device != device:
            fe.to(device)
        if isinstance(self.indexer, IndexerStack) and self.indexer.modules[0][0].device != device:
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
        self._memo = _SelectionMemo()
        self._latest_query_feature = None
        self._token_ids = None
        self._query_start = None
        self.cache_metadata.reset()
        for d in (self.diagnostic_keep_indices, self.diagnostic_scores, self.diagnostic_features):
            d.clear()

    # ---- weights in the kernels' formats, prepared once per layer ----
    def layer_weights(self, layer_idx: int, device) -> engine.LayerWeights:
        key = (int(layer_idx), str(device))
        lw = self._weights.get(key)
        if lw is None:
            fe = self.feature_extractor
            cfg = fe.config
            mlp = self.indexer.params(layer_idx if self.use_indexer_stack else 0)
            lw = engine.LayerWeights.prepare(
                geometry=fe.weight[int(layer_idx)], prototypes=fe.prototypes_for(layer_idx),
                hadamard=fe.hadamard, mlp_params=mlp, n_kv_heads=int(cfg.n_kv_heads),
                n_q_heads=int(cfg.n_q_heads), head_dim=int(cfg.head_dim), device=device)
            self._weights[key] = lw
        return lw

    def _check_policy(self):
        """Only the tokenwise policy the paper protocol requires is built
        (kvpress/evaluation/evaluate.py:743-754)."""
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

    # ---- the scoring queries ----
    def _prefill_queries(self, module, hidden_states, kwargs):
        """Post-RoPE queries of a prefill and the matching row LSE if the
        attention adapter exported one (core/kvpress_adapter.py:357-439)."""
        q = getattr(module, "_core_cached_query_states", None)
        if q is None:
            q = post_rope_queries(module, hidden_states, kwargs.get("position_ids"),
                                  kwargs.get("position_embeddings"))
        if q is None or q.shape[-2] == 0:
            raise RuntimeError("CORE failed to compute prefill QK relation features: no "
                               "post-RoPE queries (set _core_cached_query_states or q_proj)")
        if q.ndim == 3:
            q = q[None]
        first = 0
        if self.prefill_qk_scope == "question":
            if self._query_start is None:
                raise RuntimeError("CORE prefill_qk_scope='question' requires "
                                   "set_query_boundary() before prefill.")
            first = int(self._query_start)
            if not 0 <= first < q.shape[2]:
                raise RuntimeError(f"Invalid CORE query boundary: query_start={first}, "
                                   f"seq_len={q.shape[2]}")
            q = q[:, :, first:]
        elif self.prefill_qk_scope != "all":
            raise ValueError(f"prefill_qk_scope must be 'all' or 'question', got "
                             f"{self.prefill_qk_scope!r}")
        lse = getattr(module, "_core_cached_softmax_lse", None)
        if lse is not None:
            lse = lse[:, :, first:] if lse.ndim == 3 else None
            if lse is not None and lse.shape[-1] != q.shape[2]:
                lse = None
        return q, lse

    def _decode_queries(self, module, hidden_states, kwargs):
        """Queries of every buffered decode token: the adapter's own if they
        cover the buffer, else rebuilt at their absolute positions
        (core/kvpress_adapter.py:469-519)."""
        q = getattr(module, "_core_cached_query_states", None)
        t = hidden_states.shape[1]
        if q is None or q.shape[-2] != t:
            pos = emb = None
            if t > 1:
                pos = decode_positions(kwargs, t, hidden_states.device)
            if pos is None:
                pos, emb = kwargs.get("position_ids"), kwargs.get("position_embeddings")
            q = post_rope_queries(module, hidden_states, pos, emb)
        if q is None or q.shape[-2] == 0:
            raise RuntimeError("CORE failed to reconstruct decode QK features; refusing to "
                               "replace the paper features with zeros")
        return (q[None] if q.ndim == 3 else q), None

    def _scoring_queries(self, module, hidden_states, keys, is_prefill, kwargs):
        """(B, Hq, nq, d) post-RoPE queries in the scoring dtype, plus an
        optional exported row LSE."""
        pick = self._prefill_queries if is_prefill else self._decode_queries
        q, lse = pick(module, hidden_states, kwargs)
        if q.shape[0] != keys.shape[0]:
            q = q.expand(keys.shape[0], -1, -1, -1)
        return q.to(_score_dtype(self.feature_extractor)).contiguous(), lse

    def _special_mask(self, ids):
        special = tuple(getattr(self.feature_extractor.config, "special_token_ids", ()) or ())
        if not special or ids is None:
            return None
        return torch.isin(ids, torch.tensor(special, device=ids.device, dtype=ids.dtype))

    def _scores_and_features(self, module, hidden_states, keys, values, kwargs, layer_idx):
        """Calibrated scores (B, L) and features (B, L, 14) through the
        library's feature and indexer entry points."""
        self._check_policy()
        B, _, L, _ = keys.shape
        is_prefill = hidden_states.shape[1] >= L
        positions, ids, extent = self.cache_metadata.align(layer_idx, B, L, keys.device)
        q, lse = self._scoring_queries(module, hidden_states, keys, is_prefill, kwargs)
        cfg = self.feature_extractor.config
        lw = self.layer_weights(layer_idx, keys.device)
        sdt = _score_dtype(self.feature_extractor)
        k = keys.to(sdt).contiguous()
        v = values.to(sdt).contiguous()
        feats = torch.empty(B, L, 14, dtype=torch.float32, device=keys.device)
        ops.qk_features(q, k, topk_qk=int(cfg.topk_qk), n_recent_queries=int(cfg.n_recent_queries),
                        lse=lse, features=feats)
        ops.coverage_features(k, lw.geometry_ext, lw.prototypes,
                              shrinkage_rho=float(cfg.shrinkage_rho), features=feats, col0=6)
        scores = ops.indexer_scores(v, positions, feats, lw.mlp, original_length=int(extent),
                                    is_prefill=is_prefill, n_sink=int(cfg.n_sink),
                                    special=self._special_mask(ids))
        self._note_features(layer_idx, feats)
        return scores, feats

    def _note_features(self, layer_idx, feats):
        self._latest_query_feature = feats[:, :, 3]
        if self.capture_diagnostics:
            self.diagnostic_features[int(layer_idx)] = feats[0].detach().float().cpu()

    def _compute_scores_from_features(self, module, hidden_states, keys, values, attentions,
                                      is_prefill, kwargs=None, layer_idx=0):
        """(B, Hkv, L) calibrated scores, the same for every KV head
        (core/kvpress_adapter.py:312-558)."""
        scores, _ = self._scores_and_features(module, hidden_states, keys, values, kwargs or {},
                                              layer_idx)
        return scores[:, None, :].expand(-1, keys.shape[1], -1).contiguous()

    # ---- the selection policy around the indexer scores ----
    def _is_scoring_layer(self, layer_idx) -> bool:
        if layer_idx is None:
            return True
        every = self.scoring_layer_idx if self.scoring_layer_idx is not None else -1
        if self.scoring_stride > 1 and every >= 0:
            return layer_idx % self.scoring_stride == every % self.scoring_stride
        return every == -1 or layer_idx == every

    def _budget(self, seq_len: int) -> int:
        return max(min(self.n_sink_protect, seq_len), int(seq_len * (1 - self.compression_ratio)))

    def _recency(self, scores: torch.Tensor) -> torch.Tensor:
        """Add alpha * exp(-(age) / window) when the recency bonus is on."""
        n = scores.shape[-1]
        if self.recency_alpha <= 0.0 or n <= 1:
            return scores
        age = (n - 1) - torch.arange(n, device=scores.device, dtype=scores.dtype)
        bonus = self.recency_alpha * torch.exp(-age / max(1, self.recency_window))
        return scores + bonus

    def _protect_sinks(self, scores: torch.Tensor, seq_len: int) -> torch.Tensor:
        """Selection copy with the first n_sink_protect tokens lifted above
        every other score; the calibrated scores stay as they are."""
        s = self.n_sink_protect
        if not 0 < s < seq_len:
            return scores
        lifted = scores.clone()
        lifted[..., :s] = scores.max().detach() + 1.0
        return lifted

    def _remember(self, selection, calibrated, budget, layer_idx):
        self._memo.selection = selection.detach().clone()
        self._memo.calibrated = calibrated.detach().clone()
        if self.capture_diagnostics:
            dl = int(layer_idx if layer_idx is not None else -1)
            self._memo.kept = selection.topk(budget, dim=-1).indices
            self.diagnostic_scores[dl] = calibrated.detach().float().cpu()
            self.diagnostic_keep_indices[dl] = self._memo.kept.detach().cpu()

    @torch.no_grad()
    def score(self, module, hidden_states, keys, values, attentions, kwargs):
        """Selection scores (B, Hkv, L), sinks saturated (core/kvpress_adapter.py:690-797)."""
        self._ensure_device(hidden_states.device)
        B, H, L, _ = keys.shape
        layer = getattr(module, "layer_idx", None)
        self._memo.follow(L)
        if not self._is_scoring_layer(layer) and self._memo.selection is not None:
            reuse = self._memo.selection.to(device=keys.device, dtype=keys.dtype)
            return reuse[:, None, :].expand(-1, H, -1).contiguous()
        calibrated = self._recency(self._compute_scores_from_features(
            module, hidden_states, keys, values, attentions, hidden_states.shape[1] >= L, kwargs,
            layer_idx=layer if layer is not None else 0))
        selection = self._protect_sinks(calibrated, L)
        budget = self._budget(L)
        if 0 < budget < L:
            self._remember(selection[:, 0], calibrated[:, 0], budget, layer)
        return selection

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        """Keep the Top-B of the selection scores and gather them (core/kvpress_adapter.py:299-310)."""
        if self.compression_ratio == 0:
            return keys, values
        scores = self.score(module, hidden_states, keys, values, attentions, kwargs)
        layer = int(module.layer_idx)
        budget = self._budget(keys.shape[2])
        self.cache_metadata.align(layer, keys.shape[0], keys.shape[2], keys.device)
        if budget >= keys.shape[2]:
            return keys, values
        keep, _ = ops.topb_select(scores[:, 0].float(), budget, 0)
        self.retain_metadata(layer, keep)
        return ops.compact_kv(keys.contiguous(), values.contiguous(), keep)


@dataclass
class COREMemoryPress(BasePress):
    """Eviction with latent-memory writing and the gated readout
    (core/kvpress_adapter.py:814-1382).  The memory state of layer l is
    ``_M[l]`` (B, d_mem, Hkv*d), ``_b[l]`` (B, d_mem), ``_Z[l]`` (B,)."""

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
        if self.base_press is None:
            raise ValueError("COREMemoryPress needs a COREScorerPress as base_press")
        self._M: dict = {}
        self._b: dict = {}
        self._Z: dict = {}
        self._write_theta: dict = {}   # folded memory projection per (module, layout)
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
        mm = self.memory_module
        if mm is not None and torch.device(device).type == "cuda" \
                and mm.modules[0][0].device != torch.device(device):
            mm.to(device)
            self._write_theta.clear()
            self._readout_weights.clear()

    def reset_cache(self):
        self.base_press.reset_cache()
        self.reset_memory()

    def reset_memory(self, layer_idx: Optional[int] = None):
        for state in (self._M, self._b, self._Z):
            if layer_idx is None:
                state.clear()
            else:
                state.pop(layer_idx, None)

    def _check_spaces(self):
        if self.memory_value_space != "pre_o_proj":
            raise ValueError(f"Unknown or unsupported CORE memory_value_space={self.memory_value_space!r}")
        if self.memory_query_space != "post_rope_q":
            raise ValueError(f"Unknown or unsupported CORE memory_query_space={self.memory_query_space!r}")
        if self.memory_uniform_fraction != 0.0:
            raise NotImplementedError("memory_uniform_fraction != 0 is not supported by core_b200")

    def _theta_for(self, layer_idx, n_kv, groups, head_dim, device, f32: bool):
        """The group-folded memory projection (core/kvpress_adapter.py:916-940):
        its f32 fold for the f32 kernels, its two bf16 terms for the tensor-core ones."""
        key = (self.memory_module.module_index(layer_idx), n_kv, groups, str(device), f32)
        t = self._write_theta.get(key)
        if t is None:
            fold = engine.fold_groups(self.memory_module.params(layer_idx)[0].to(device), n_kv,
                                      groups, head_dim)
            t = self._write_theta[key] = fold if f32 else ops.split_bf16(fold, 2)
        return t

    def _memory_state(self, layer_idx, B, d_mem, width, device) -> engine.MemoryState:
        M = self._M.get(layer_idx)
        if M is None or M.shape != (B, d_mem, width) or M.device != torch.device(device):
            self._M[layer_idx] = torch.zeros(B, d_mem, width, device=device)
            self._b[layer_idx] = torch.zeros(B, d_mem, device=device)
        if self._Z.get(layer_idx) is None or self._Z[layer_idx].shape != (B,):
            self._Z[layer_idx] = torch.zeros(B, device=device)
        return engine.MemoryState(self._M[layer_idx], self._b[layer_idx], self._Z[layer_idx])

    @torch.no_grad()
    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        """Select the retained tokens, fold the evicted ones into the layer's
        memory state, return the retained K/V (core/kvpress_adapter.py:968-1210)."""
        self._ensure_device(hidden_states.device)
        if self.compression_ratio == 0:
            return keys, values
        sp = self.base_press
        layer = int(getattr(module, "layer_idx", 0))
        B, n_kv, L, head_dim = keys.shape
        sp._memo.follow(L)
        n_sink = int(sp.n_sink_protect)
        n_kept = engine.n_kept_for(L, self.compression_ratio, n_sink)
        if n_kept >= L:
            sp.cache_metadata.align(layer, B, L, keys.device)
            return keys, values
        write = self.enable_memory_writing and self.memory_module is not None
        if write:
            self._check_spaces()
        sdt = _score_dtype(sp.feature_extractor)
        # the memory write and the gather see the cache's own values; the
        # features see them in the scoring dtype
        mdt = torch.float32 if keys.dtype != torch.bfloat16 else torch.bfloat16
        fused = keys.dtype == sdt and mdt == sdt
        state = theta = None
        if write:
            state = self._memory_state(layer, B, self.memory_module.d_mem, n_kv * head_dim,
                                       keys.device)
            theta = self._theta_for(layer, n_kv, sp.feature_extractor.n_q_heads // n_kv,
                                    head_dim, keys.device, f32=mdt == torch.float32)
        reuse = (not sp._is_scoring_layer(layer)) and sp._memo.calibrated is not None
        if reuse or sp.recency_alpha > 0.0 or not fused:
            calibrated, keep, evict = self._select_outside(module, hidden_states, keys, values,
                                                           kwargs, layer, n_kept, reuse)
            if write and evict.shape[1] > 0:
                ops.memory_write(keys.to(mdt).contiguous(), values.to(mdt).contiguous(),
                                 calibrated, evict, theta, state.M, state.b, state.Z,
                                 gamma=self.memory_decay, eta=self.memory_write_eta,
                                 student_temp=self.student_temp)
            out_k, out_v = ops.compact_kv(keys.contiguous(), values.contiguous(), keep)
        else:
            calibrated, keep, out_k, out_v = self._select_fused(
                module, hidden_states, keys, values, kwargs, layer, n_kept, n_sink, state, theta)
        self._remember_layer(layer, calibrated, keep, L)
        return out_k, out_v

    def _select_fused(self, module, hidden_states, keys, values, kwargs, layer, n_kept, n_sink,
                      state, theta):
        """The whole layer step in one library call (features, scores, Top-B,
        memory write, gather) on caches already in the scoring dtype."""
        sp = self.base_press
        sp._check_policy()
        B, _, L, _ = keys.shape
        is_prefill = hidden_states.shape[1] >= L
        positions, ids, extent = sp.cache_metadata.align(layer, B, L, keys.device)
        q, lse = sp._scoring_queries(module, hidden_states, keys, is_prefill, kwargs or {})
        cfg = sp.feature_extractor.config
        lw = sp.layer_weights(layer, keys.device)
        if theta is not None:
            if keys.dtype == torch.float32:
                lw.theta_fold = theta
            else:
                lw.theta_split = theta
        out = engine.compress_layer(
            q, keys, values, lw, n_kept=n_kept, positions=positions, original_length=int(extent),
            is_prefill=is_prefill, n_sink=n_sink, topk_qk=int(cfg.topk_qk),
            n_recent_queries=int(cfg.n_recent_queries), shrinkage_rho=float(cfg.shrinkage_rho),
            memory=state, gamma=self.memory_decay, eta=self.memory_write_eta,
            student_temp=self.student_temp, special=sp._special_mask(ids), lse=lse)
        sp._note_features(layer, out["features"])
        return out["scores"], out["keep"], out["keys"], out["values"]

    def _select_outside(self, module, hidden_states, keys, values, kwargs, layer, n_kept, reuse):
        """Scores (reused from the scoring layer, or computed in the scoring
        dtype and adjusted by the recency bonus) and the Top-B split."""
        sp = self.base_press
        if reuse:
            sp.cache_metadata.align(layer, keys.shape[0], keys.shape[2], keys.device)
            calibrated = sp._memo.calibrated
        else:
            calibrated = sp._recency(sp._scores_and_features(module, hidden_states, keys, values,
                                                             kwargs or {}, layer)[0])
        keep, evict = ops.topb_select(calibrated, n_kept, int(sp.n_sink_protect))
        return calibrated, keep, evict

    def _remember_layer(self, layer, calibrated, keep, L):
        sp = self.base_press
        sp._memo.seq_len = L
        sp._memo.calibrated = calibrated
        sp._memo.selection = sp._protect_sinks(calibrated, L)
        if sp.capture_diagnostics:
            sp.diagnostic_scores[layer] = calibrated.detach().float().cpu()
            sp.diagnostic_keep_indices[layer] = keep.detach().long().cpu()
        sp.retain_metadata(layer, keep)

    # ---- decode-step readout ----
    def _readout_params(self, module, layer_idx, n_kv, groups, head_dim, device):
        key = (layer_idx, str(device))
        rp = self._readout_weights.get(key)
        if rp is None:
            th, gw1, gb1, gw2, gb2 = self.memory_module.params(layer_idx)
            f32 = lambda t: t.to(device).float().contiguous()  # noqa: E731
            rp = (f32(th), (f32(gw1), f32(gb1), f32(gw2).reshape(-1), f32(gb2).reshape(-1)),
                  engine.fold_groups(module.o_proj.weight.to(device), n_kv, groups, head_dim))
            self._readout_weights[key] = rp
        return rp

    def _readout_queries(self, module, kwargs):
        hidden = kwargs["hidden_states"]
        q = getattr(module, "_core_cached_query_states", None)
        if q is not None and q.ndim == 4 and q.shape[0] == hidden.shape[0] \
                and q.shape[-2] == hidden.shape[1]:
            return q
        return post_rope_queries(module, hidden, kwargs.get("position_ids"),
                                 kwargs.get("position_embeddings"))

    @torch.no_grad()
    def apply_memory_readout(self, module, kwargs, output):
        """attention output += folded o_proj(g(q) m(q)) for this layer's memory
        (core/kvpress_adapter.py:1212-1352)."""
        if not self.enable_memory_writing or self.memory_module is None:
            return output
        layer = int(getattr(module, "layer_idx", 0))
        if self._M.get(layer) is None or self._b.get(layer) is None:
            return output
        self._check_spaces()
        q = self._readout_queries(module, kwargs)
        if q is None:
            raise RuntimeError("CORE memory readout could not reconstruct post-RoPE queries; "
                               "refusing to mix hidden-state queries with post-RoPE memory keys.")
        n_q = int(module.config.num_attention_heads)
        n_kv = int(module.config.num_key_value_heads)
        theta, gate, o_fold = self._readout_params(module, layer, n_kv, n_q // n_kv, q.shape[-1],
                                                   q.device)
        attn = output[0] if isinstance(output, (list, tuple)) else output
        out = attn.contiguous().clone()
        ops.memory_readout(q, theta, gate, self._M[layer], self._b[layer], o_fold, out,
                           n_kv_heads=n_kv, gate_override=self.memory_gate_override)
        if isinstance(output, (list, tuple)):
            return type(output)([out, *output[1:]])
        return out

    def forward_hook(self, module, input, kwargs, output):
        """Prefill: compress (the base hook); decode: add the memory readout."""
        if _phase_is_prefill(kwargs, kwargs["hidden_states"].shape[1]):
            return super().forward_hook(module, input, kwargs, output)
        return self.apply_memory_readout(module, kwargs, output)


@dataclass
class COREIndexerPress(COREScorerPress):
    """Scorer press with an optional absolute budget (core/kvpress_adapter.py:1385-1436)."""

    budget: Optional[int] = None

    def compress(self, module, hidden_states, keys, values, attentions, kwargs):
        L = keys.shape[2]
        if L <= 1:
            return keys, values
        self._ensure_device(hidden_states.device)
        want = self.budget if self.budget is not None else int(L * (1 - self.compression_ratio))
        n_kept = max(1, min(self.n_sink_protect, L), min(want, L))
        if n_kept >= L:
            return keys, values
        saved = self.compression_ratio
        self.compression_ratio = 1.0 - n_kept / L
        try:
            return super().compress(module, hidden_states, keys, values, attentions, kwargs)
        finally:
            self.compression_ratio = saved


@dataclass
class COREDecodingPress(DecodingPress):
    """Decoding press over the CORE memory press (core/kvpress_adapter.py:92-122):
    the buffer defaults to, and may not be shorter than, one compression
    interval, since every query of the interval scores the recompression."""

    hidden_states_buffer_size: Optional[int] = None

    def __post_init__(self):
        if not hasattr(self.base_press, "compress"):
            raise ValueError("CORE decoding press requires a compress-capable base press")
        self._check_sizes()
        if self.hidden_states_buffer_size is None:
            self.hidden_states_buffer_size = self.compression_interval
        if self.hidden_states_buffer_size < self.compression_interval:
            raise ValueError("CORE requires queries from the entire compression interval; "
                             "hidden_states_buffer_size must be >= compression_interval")
        self.reset()


@dataclass
class COREPrefillDecodingPress(PrefillDecodingPress):
    """CORE token metadata and matched prefill/decode budgets
    (core/kvpress_adapter.py:56-89)."""

    query_aware_prefill: bool = False
    match_prefill_budget: bool = True

    def begin_sequence(self, context_length):
        """Decode recompressions return the cache to the prefill's budget."""
        if self.match_prefill_budget:
            self.decoding_press.target_size = retained_budget(
                context_length, self.prefilling_press.compression_ratio)

    def record_input_tokens(self, input_ids, position_ids=None):
        self.prefilling_press.record_input_tokens(input_ids, position_ids)

    def reset_cache(self):
        if self.decoding_press is not None:
            self.decoding_press.reset()
        if self.prefilling_press is not None and hasattr(self.prefilling_press, "reset_cache"):
            self.prefilling_press.reset_cache()


# ===========================================================================
# Factories (core/kvpress_adapter.py:1444-1832)
# ===========================================================================
def _effective_ratio(requested, cfg) -> float:
    r = float(cfg.compression_ratio) if requested is None else float(requested)
    if not 0.0 < r < 1.0:
        raise ValueError(f"compression_ratio must lie in (0, 1), received {r}")
    return r


# checkpoint config key -> (press field, default when absent)
_POLICY_FIELDS = {
    "n_sink_protect": 0, "recency_alpha": 0.0, "recency_window": 64, "scoring_stride": 1,
    "span_block_size": 1, "span_pool_beta": 5.0, "span_selection_mode": "sliding_max",
    "coverage_fraction": 0.25, "query_feature_weight": 0.0, "lexical_overlap_weight": 0.0,
    "identifier_lexical_weight": 0.0, "identifier_min_match_tokens": 20,
    "identifier_context_skip": 64, "identifier_span_size": 32, "protect_query_tokens": False,
    "prefill_qk_scope": "all",
}


def _apply_policy(press: COREScorerPress, cfg) -> None:
    for name, default in _POLICY_FIELDS.items():
        setattr(press, name, cfg.get(name, default))


def _scorer(cls, checkpoint_path, device, compression_ratio, **extra):
    parts = load_checkpoint(checkpoint_path, device=device)
    cfg = parts["config"]
    press = cls(indexer=parts["indexer"], feature_extractor=parts["geometry"],
                compression_ratio=_effective_ratio(compression_ratio, cfg),
                student_temp=cfg.student_temp, use_indexer_stack=parts["use_stack"],
                **{k: v(cfg) for k, v in extra.items()})
    _apply_policy(press, cfg)
    return press, parts


def _memory_of(parts, checkpoint_path):
    memory, cfg = parts["memory"], parts["config"]
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


def _with_memory(base, memory, cfg) -> COREMemoryPress:
    return COREMemoryPress(base_press=base, memory_module=memory, memory_decay=cfg.memory_decay,
                           memory_write_eta=cfg.memory_write_eta,
                           memory_uniform_fraction=cfg.memory_uniform_fraction,
                           enable_memory_writing=cfg.enable_memory_writing,
                           memory_query_space=cfg.memory_query_space,
                           memory_value_space=cfg.memory_value_space)


def load_core_scorer_press(checkpoint_path: str, device: str = "cuda:0",
                           compression_ratio: float = 0.5) -> COREScorerPress:
    return _scorer(COREScorerPress, checkpoint_path, device, compression_ratio)[0]


def load_core_indexer_press(checkpoint_path: str, device: str = "cuda:0",
                            compression_ratio: Optional[float] = None) -> COREIndexerPress:
    return _scorer(COREIndexerPress, checkpoint_path, device, compression_ratio,
                   budget=lambda cfg: cfg.budget)[0]


def load_core_memory_press(checkpoint_path: str, device: str = "cuda:0",
                           compression_ratio: Optional[float] = None) -> COREMemoryPress:
    base, parts = _scorer(COREScorerPress, checkpoint_path, device, compression_ratio)
    return _with_memory(base, _memory_of(parts, checkpoint_path), parts["config"])


def load_core_prefill_decoding_press(checkpoint_path: str, device: str = "cuda:0",
                                     compression_ratio: Optional[float] = None,
                                     decoding_compression_interval: int = 128,
                                     decoding_target_size: Optional[int] = None,
                                     decoding_hidden_states_buffer_size: Optional[int] = None
                                     ) -> COREPrefillDecodingPress:
    """The ``core_full`` press: one memory press shared by the prefill and the
    decoding press, decode recompression back to the prefill budget unless a
    target size is given."""
    base, parts = _scorer(COREScorerPress, checkpoint_path, device, compression_ratio)
    shared = _with_memory(base, _memory_of(parts, checkpoint_path), parts["config"])
    decoding = COREDecodingPress(base_press=shared, compression_interval=decoding_compression_interval,
                                 target_size=decoding_target_size or 1,
                                 hidden_states_buffer_size=decoding_hidden_states_buffer_size)
    return COREPrefillDecodingPress(prefilling_press=shared, decoding_press=decoding,
                                    match_prefill_budget=decoding_target_size is None,
                                    query_aware_prefill=False)


PRESS_REGISTRY = {"core_full": load_core_prefill_decoding_press,
                  "core_memory": load_core_memory_press,
                  "core_indexer": load_core_indexer_press}
