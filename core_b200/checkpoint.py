"""Reader and writer of the CORE checkpoint format (``core_indexer.pt``).

The format is the reference's (``core/train.py:2982-3047``): a ``torch.save``
dict with ``state_dict`` (indexer stack: ``layers.<i>.net.{0,2,4}.{weight,bias}``),
``n_layers``, ``input_dim``, ``hidden_dim``, ``indexer_compact_stride``,
``config`` (the COREConfig fields), ``is_stack``, optional
``feature_extractor_state_dict`` (``format_version`` 3, ``hadamard_rotation``,
``geometry_state_dict.weight`` (L, P, Hkv*d), ``prototype_bank_state_dict``),
``memory_state_dict`` (``layers.<i>.theta.weight``, ``layers.<i>.gate.{0,2}``)
and ``memory_dims``.  It is read here without importing the reference.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

import numpy as np
import torch

# Fields the press reads from the checkpoint config, with COREConfig defaults
# (core/config.py:24-309).
CONFIG_DEFAULTS = dict(
    n_layers=None, n_kv_heads=None, n_q_heads=None, head_dim=None, hidden_size=None,
    compression_ratio=0.5, budget=None, n_prototypes=64, center_prototype_features=True,
    proto_dim=64, key_geometry_mode="head_concat_layer_gaussian", key_geometry_eps=1e-8,
    shrinkage_rho=0.1, n_sink=4, topk_qk=4, qk_query_block_size=128,
    qk_primary_mode="attention_advantage", prefill_qk_scope="all", n_recent_queries=16,
    special_token_ids=(), indexer_hidden_dim=128, student_temp=1.0,
    enable_memory_writing=True, memory_decay=0.9, memory_dim=512, memory_gate_hidden=64,
    memory_share_across_layers=False, memory_projection_groups=1, memory_write_eta=1.0,
    memory_uniform_fraction=0.0, memory_query_space="post_rope_q",
    memory_value_space="pre_o_proj", n_sink_protect=4, recency_alpha=0.0, recency_window=64,
    span_block_size=1, span_selection_mode="tokenwise", coverage_fraction=0.25,
    span_pool_beta=5.0, query_feature_weight=0.0, lexical_overlap_weight=0.0,
    identifier_lexical_weight=0.0, identifier_min_match_tokens=20, identifier_context_skip=64,
    identifier_span_size=32, protect_query_tokens=False, scoring_stride=1, seed=42,
    geometry_seed=42, dtype="bfloat16",
)

INTERFACE = {
    "memory_query_space": "post_rope_q",
    "memory_value_space": "pre_o_proj",
    "key_geometry_mode": "head_concat_layer_gaussian",
}


def validate_checkpoint_interface(config: dict) -> None:
    """``validate_checkpoint_interface`` (core/config.py:312-324)."""
    for name, expected in INTERFACE.items():
        if config.get(name) != expected:
            raise ValueError(
                f"Checkpoint interface mismatch: {name}={config.get(name)!r}; "
                f"the current method requires {expected!r}")


class Config(dict):
    """COREConfig values as attributes; unknown keys are kept, missing ones default."""

    def __init__(self, d: dict | None = None):
        super().__init__(CONFIG_DEFAULTS)
        if d:
            self.update(d)

    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e

    def __setattr__(self, k, v):
        self[k] = v


@dataclass
class IndexerStack:
    """Per-layer indexer MLPs 14 -> 128 -> 128 -> 1 (core/indexer.py:521-578)."""

    n_layers: int
    compact_stride: int
    modules: list  # [(w1, b1, w2, b2, w3, b3)]
    input_dim: int = 14
    hidden_dim: int = 128

    def module_index(self, layer_idx: int) -> int:
        layer_idx = max(0, min(int(layer_idx), self.n_layers - 1))
        return layer_idx // self.compact_stride

    def params(self, layer_idx: int):
        return self.modules[self.module_index(layer_idx)]

    def to(self, device):
        self.modules = [tuple(t.to(device) for t in m) for m in self.modules]
        return self

    def eval(self):
        return self

    def parameters(self):
        for m in self.modules:
            yield from m


@dataclass
class MemoryStack:
    """Per-layer memory projection and gate (core/indexer.py:591-669)."""

    n_layers: int
    d_model: int
    d_mem: int
    gate_hidden: int
    share_across_layers: bool
    modules: list  # [(theta (d_mem, d_model), gw1, gb1, gw2 (gh,), gb2 (1,))]

    def module_index(self, layer_idx: int) -> int:
        if self.share_across_layers:
            return 0
        return max(0, min(int(layer_idx), self.n_layers - 1))

    def params(self, layer_idx: int):
        return self.modules[self.module_index(layer_idx)]

    def to(self, device):
        self.modules = [tuple(t.to(device) for t in m) for m in self.modules]
        return self


@dataclass
class FeatureGeometry:
    """Fixed coverage geometry: per-layer Gaussian projection, prototypes, Hadamard rotation."""

    weight: torch.Tensor       # (n_layers, P, Hkv*d)
    prototypes: torch.Tensor   # (M, P) or (n_layers, M, P)
    hadamard: torch.Tensor     # (P, P)
    config: Config = field(default_factory=Config)

    @property
    def n_q_heads(self):
        return int(self.config.n_q_heads)

    @property
    def n_kv_heads(self):
        return int(self.config.n_kv_heads)

    def prototypes_for(self, layer_idx: int) -> torch.Tensor:
        if self.prototypes.ndim == 3:
            return self.prototypes[int(layer_idx)]
        return self.prototypes

    def to(self, device):
        self.weight = self.weight.to(device)
        self.prototypes = self.prototypes.to(device)
        self.hadamard = self.hadamard.to(device)
        return self


# ---- fixed geometry constructions (used when a checkpoint omits them) ----

def gaussian_geometry(n_layers: int, n_kv_heads: int, head_dim: int, proto_dim: int,
                      seed: int) -> torch.Tensor:
    """``LayerwiseKeyGeometryProjector`` weights (core/features.py:29-50)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return torch.randn(n_layers, proto_dim, n_kv_heads * head_dim, generator=g,
                       dtype=torch.float32) / np.sqrt(proto_dim)


def unit_prototypes(n_prototypes: int, dim: int, seed: int) -> torch.Tensor:
    """``PrototypeBank`` default bank (core/features.py:95-100)."""
    raw = np.random.RandomState(seed).randn(n_prototypes, dim).astype(np.float32)
    return torch.from_numpy(raw / np.maximum(np.linalg.norm(raw, axis=1, keepdims=True), 1e-8))


def hadamard_rotation(dim: int, seed: int) -> torch.Tensor:
    """``HadamardProjector`` R = H D / sqrt(d) (core/features.py:224-236)."""
    signs = np.random.RandomState(seed).choice([-1.0, 1.0], size=dim).astype(np.float32)
    n = 1
    while n < dim:
        n *= 2
    H = np.array([[1.0]])
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    Ht = torch.tensor(H, dtype=torch.float32)[:dim, :dim]
    return (1.0 / np.sqrt(dim)) * Ht @ torch.diag(torch.from_numpy(signs))


def _normalize_rows(t: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.normalize(t.float(), dim=-1, eps=1e-8)


def _stack_modules(state: dict, prefix_re: str) -> dict:
    out: dict[int, dict] = {}
    pat = re.compile(prefix_re)
    for k, v in state.items():
        m = pat.match(k)
        if m:
            out.setdefault(int(m.group(1)), {})[m.group(2)] = v
    return out


def _dense_theta(w: torch.Tensor) -> torch.Tensor:
    """Grouped (block-diagonal) projection as a dense matrix (core/indexer.py:48-52)."""
    if w.ndim == 2:
        return w
    return torch.block_diag(*[w[g] for g in range(w.shape[0])])


def load_checkpoint(path: str, device="cpu") -> dict:
    """Parse a ``core_indexer.pt`` file into the press's containers.

    Returns dict(config, indexer, geometry, memory (or None), use_stack).
    """
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    raw_config = dict(ckpt["config"])
    validate_checkpoint_interface(raw_config)
    cfg = Config(raw_config)
    # ---- indexer (core/train.py:3247-3282) ----
    is_stack = bool(ckpt.get("is_stack", False))
    sd = ckpt["state_dict"]
    if is_stack:
        mods = _stack_modules(sd, r"layers\.(\d+)\.net\.(.+)$")
        n_layers = int(ckpt["n_layers"])
        stride = int(ckpt.get("indexer_compact_stride", 1))
        modules = [tuple(mods[i][n].float() for n in ("0.weight", "0.bias", "2.weight", "2.bias",
                                                       "4.weight", "4.bias"))
                   for i in sorted(mods)]
    else:
        n_layers = max(1, int(ckpt.get("n_layers", 1)))
        stride = 1
        single = tuple(sd[f"net.{n}"].float() for n in ("0.weight", "0.bias", "2.weight",
                                                          "2.bias", "4.weight", "4.bias"))
        modules = [single] * n_layers
    indexer = IndexerStack(n_layers=n_layers, compact_stride=max(1, stride), modules=modules,
                           input_dim=int(ckpt.get("input_dim", 14)),
                           hidden_dim=int(ckpt.get("hidden_dim", 128)))
    # ---- feature geometry (core/kvpress_adapter.py:1444-1456, features.py:357-372) ----
    L = int(cfg.n_layers)
    fe = ckpt.get("feature_extractor_state_dict")
    weight = prototypes = hadamard = None
    if fe is not None and "geometry_state_dict" in fe:
        weight = fe["geometry_state_dict"]["weight"].float()
        if "hadamard_rotation" in fe:
            hadamard = fe["hadamard_rotation"].float()
        if "prototype_bank_state_dict" in fe:
            prototypes = _normalize_rows(fe["prototype_bank_state_dict"]["prototypes"])
    elif fe is not None:
        weight = fe["weight"].float()
    if weight is None:
        weight = gaussian_geometry(L, int(cfg.n_kv_heads), int(cfg.head_dim), int(cfg.proto_dim),
                                   int(cfg.geometry_seed))
    if prototypes is None:
        prototypes = unit_prototypes(int(cfg.n_prototypes), int(cfg.proto_dim), int(cfg.geometry_seed))
    if hadamard is None:
        hadamard = hadamard_rotation(int(cfg.proto_dim), int(cfg.geometry_seed))
    geometry = FeatureGeometry(weight=weight, prototypes=prototypes, hadamard=hadamard, config=cfg)
    # ---- memory stack (core/train.py:3285-3327) ----
    memory = None
    if "memory_state_dict" in ckpt:
        dims = ckpt["memory_dims"]
        msd = ckpt["memory_state_dict"]
        mn = max(1, int(dims.get("n_layers", 1)))
        gh = int(dims.get("gate_hidden", 128))
        share = bool(dims.get("share_across_layers", False))
        if dims.get("is_stack", False):
            mods = _stack_modules(msd, r"layers\.(\d+)\.(.+)$")
            per = [mods[i] for i in sorted(mods)]
        else:
            per = [msd] * (1 if share else mn)
        mmods = []
        for m in per:
            mmods.append((_dense_theta(m["theta.weight"].float()), m["gate.0.weight"].float(),
                          m["gate.0.bias"].float(), m["gate.2.weight"].float().reshape(-1),
                          m["gate.2.bias"].float().reshape(-1)))
        memory = MemoryStack(n_layers=mn, d_model=int(dims["d_model"]), d_mem=int(dims["d_mem"]),
                             gate_hidden=gh, share_across_layers=share, modules=mmods)
    out = dict(config=cfg, indexer=indexer.to(device), geometry=geometry.to(device),
               memory=memory.to(device) if memory is not None else None, use_stack=is_stack)
    return out


def save_checkpoint(path: str, *, config: dict, indexer: IndexerStack, geometry: FeatureGeometry,
                    memory: MemoryStack | None = None) -> None:
    """Write a checkpoint in the reference layout (core/train.py:3004-3046)."""
    sd = {}
    for i, (w1, b1, w2, b2, w3, b3) in enumerate(indexer.modules):
        for n, t in zip(("0.weight", "0.bias", "2.weight", "2.bias", "4.weight", "4.bias"),
                        (w1, b1, w2, b2, w3, b3)):
            sd[f"layers.{i}.net.{n}"] = t.detach().cpu().float()
    ckpt = {
        "state_dict": sd, "n_layers": indexer.n_layers, "input_dim": indexer.input_dim,
        "hidden_dim": indexer.hidden_dim, "indexer_compact_stride": indexer.compact_stride,
        "config": dict(config), "history": [], "metrics": {}, "is_stack": True,
        "feature_extractor_state_dict": {
            "format_version": 3,
            "hadamard_rotation": geometry.hadamard.detach().cpu().float(),
            "geometry_state_dict": {"weight": geometry.weight.detach().cpu().float()},
            "prototype_bank_state_dict": {"prototypes": geometry.prototypes.detach().cpu().float()},
        },
    }
    if memory is not None:
        msd = {}
        for i, (th, gw1, gb1, gw2, gb2) in enumerate(memory.modules):
            msd[f"layers.{i}.theta.weight"] = th.detach().cpu().float()
            msd[f"layers.{i}.gate.0.weight"] = gw1.detach().cpu().float()
            msd[f"layers.{i}.gate.0.bias"] = gb1.detach().cpu().float()
            msd[f"layers.{i}.gate.2.weight"] = gw2.detach().cpu().float().reshape(1, -1)
            msd[f"layers.{i}.gate.2.bias"] = gb2.detach().cpu().float().reshape(1)
        ckpt["memory_state_dict"] = msd
        ckpt["memory_dims"] = {"d_model": memory.d_model, "d_mem": memory.d_mem,
                               "gate_hidden": memory.gate_hidden, "projection_groups": 1,
                               "share_across_layers": memory.share_across_layers,
                               "n_layers": memory.n_layers, "is_stack": True}
        ckpt["memory_history"] = []
    torch.save(ckpt, path)


def random_checkpoint_parts(*, seed: int, n_layers: int, n_kv_heads: int, n_q_heads: int,
                            head_dim: int = 128, d_mem: int = 512, gate_hidden: int = 64,
                            hidden_size: int | None = None, geometry_seed: int = 42,
                            **config_overrides):
    """Random-init indexer and memory stacks with nn.Linear's initialisation
    (kaiming-uniform weights, uniform(+-1/sqrt(fan_in)) biases), the fixed
    geometry constructions, and a matching config."""
    torch.manual_seed(int(seed))

    def linear(out_f, in_f):
        lin = torch.nn.Linear(in_f, out_f)
        return lin.weight.detach().clone(), lin.bias.detach().clone()

    mods = []
    for _ in range(n_layers):
        w1, b1 = linear(128, 14)
        w2, b2 = linear(128, 128)
        w3, b3 = linear(1, 128)
        mods.append((w1, b1, w2, b2, w3, b3))
    d_model = n_q_heads * head_dim
    mmods = []
    for _ in range(n_layers):
        th, _ = linear(d_mem, d_model)
        gw1, gb1 = linear(gate_hidden, d_model)
        gw2, gb2 = linear(1, gate_hidden)
        mmods.append((th, gw1, gb1, gw2.reshape(-1), gb2.reshape(-1)))
    cfg = Config(dict(n_layers=n_layers, n_kv_heads=n_kv_heads, n_q_heads=n_q_heads,
                      head_dim=head_dim, hidden_size=hidden_size or d_model, memory_dim=d_mem,
                      memory_gate_hidden=gate_hidden, geometry_seed=geometry_seed,
                      compression_ratio=0.75))
    cfg.update(config_overrides)
    geometry = FeatureGeometry(
        weight=gaussian_geometry(n_layers, n_kv_heads, head_dim, 64, geometry_seed),
        prototypes=unit_prototypes(64, 64, geometry_seed),
        hadamard=hadamard_rotation(64, geometry_seed), config=cfg)
    indexer = IndexerStack(n_layers=n_layers, compact_stride=1, modules=mods)
    memory = MemoryStack(n_layers=n_layers, d_model=d_model, d_mem=d_mem, gate_hidden=gate_hidden,
                         share_across_layers=False, modules=mmods)
    return dict(config=cfg, indexer=indexer, geometry=geometry, memory=memory)


__all__ = ["Config", "IndexerStack", "MemoryStack", "FeatureGeometry", "load_checkpoint",
           "save_checkpoint", "random_checkpoint_parts", "validate_checkpoint_interface",
           "gaussian_geometry", "unit_prototypes", "hadamard_rotation"]
