"""Head-sharded layer step for one long sequence (KV heads split across GPUs).

The reference compresses a layer in one process holding all KV heads
(``COREMemoryPress.compress``, core/kvpress_adapter.py:968-1210).  Here rank
r of N holds KV heads [r*Hkv/N, (r+1)*Hkv/N) (and their query heads) and the
step is split at its cross-head reductions:

1. QK relation features over the rank's heads, reduced to a per-key summary
   (``ops.qk_head_summary``); an all-to-all brings every rank the summaries
   of its key range [r*Lc, (r+1)*Lc), Lc = ceil(L/N), and
   ``ops.qk_merge_summaries`` finishes f1..f6 there.
2. Coverage: each rank projects its heads (``coverage_partial_projection``);
   a reduce-scatter sums the projections by key range; the range's column
   sums and assignment histogram are summed across ranks (two all-reduces).
3. Auxiliary features: per-head value sums are all-gathered.
4. Each rank scores its key range; an all-gather gives every rank all
   scores, and every rank runs the same Top-B (identical inputs, identical
   keep sets, no further exchange).
5. Memory write: the layer's memory state lives on rank ``layer % N``,
   which gathers the K/V rows of all heads (the whole caches when most rows
   are evicted, else the evicted rows only) and runs the write.
6. Each rank gathers its own heads' retained K/V.

Collectives go through an :class:`Exchange`.  :class:`DistExchange` runs
them with ``torch.distributed`` (NCCL on GPUs, gloo on CPU) for the one rank
of this process; :class:`LocalExchange` computes every rank in one process,
so the split arithmetic can be checked on one GPU against the unsharded
step.  The step functions take the list of ranks the exchange handles and
lists of per-rank tensors.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import engine, ops

__all__ = ["HeadShard", "Exchange", "DistExchange", "LocalExchange", "ShardWeights",
           "compress_layer_sharded"]


@dataclass(frozen=True)
class HeadShard:
    """Rank ``rank`` of ``world``: its KV heads and its key range."""

    rank: int
    world: int
    n_kv_heads: int
    seq_len: int

    def __post_init__(self):
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError("bad rank / world size")
        if self.n_kv_heads % self.world != 0:
            raise ValueError(f"{self.n_kv_heads} KV heads do not split over {self.world} ranks")

    @property
    def heads_per_rank(self) -> int:
        return self.n_kv_heads // self.world

    @property
    def h0(self) -> int:
        return self.rank * self.heads_per_rank

    @property
    def h1(self) -> int:
        return self.h0 + self.heads_per_rank

    @property
    def chunk(self) -> int:
        """Keys per range (the last range may be shorter or empty)."""
        return math.ceil(self.seq_len / self.world)

    @property
    def k0(self) -> int:
        return min(self.rank * self.chunk, self.seq_len)

    @property
    def k1(self) -> int:
        return min(self.k0 + self.chunk, self.seq_len)

    @property
    def n_keys(self) -> int:
        return self.k1 - self.k0

    @property
    def padded(self) -> int:
        """Rows of the buffers exchanged by key range (world * chunk)."""
        return self.world * self.chunk

    @staticmethod
    def owner(layer_idx: int, world: int) -> int:
        """Rank holding the memory state of layer ``layer_idx``."""
        return int(layer_idx) % world


class Exchange:
    """Collectives over the ranks, for the ranks this process computes.

    Every method takes and returns lists indexed like ``self.ranks``."""

    world: int
    ranks: list

    def all_to_all(self, xs):
        """xs[i]: (world * chunk, ...) split by destination -> (world, chunk, ...) by source."""
        raise NotImplementedError

    def reduce_scatter_sum(self, xs):
        """xs[i]: (world * chunk, ...) -> the sum over ranks of chunk rank (chunk, ...)."""
        raise NotImplementedError

    def all_reduce_sum(self, xs):
        raise NotImplementedError

    def all_gather(self, xs):
        """xs[i]: (n, ...) -> (world * n, ...) in rank order."""
        raise NotImplementedError

    def gather_to(self, owner: int, xs):
        """xs[i]: (n, ...) -> on the owner (world * n, ...) in rank order, elsewhere None."""
        raise NotImplementedError

    def gather_to_async(self, owner: int, xs):
        """gather_to without ordering later work on the current stream after it:
        returns (outputs, wait); wait() orders the current stream after the gather."""
        out = self.gather_to(owner, xs)
        return out, (lambda: None)


class LocalExchange(Exchange):
    """All ``world`` ranks in this process (sums in rank order)."""

    def __init__(self, world: int):
        self.world = int(world)
        self.ranks = list(range(self.world))

    def all_to_all(self, xs):
        n = xs[0].shape[0] // self.world
        return [torch.stack([xs[p][r * n:(r + 1) * n] for p in range(self.world)])
                for r in range(self.world)]

    def reduce_scatter_sum(self, xs):
        n = xs[0].shape[0] // self.world
        out = []
        for r in range(self.world):
            acc = xs[0][r * n:(r + 1) * n].clone()
            for p in range(1, self.world):
                acc += xs[p][r * n:(r + 1) * n]
            out.append(acc)
        return out

    def all_reduce_sum(self, xs):
        acc = xs[0].clone()
        for p in range(1, self.world):
            acc += xs[p]
        return [acc.clone() for _ in range(self.world)]

    def all_gather(self, xs):
        cat = torch.cat(list(xs))
        return [cat for _ in range(self.world)]

    def gather_to(self, owner: int, xs):
        cat = torch.cat(list(xs))
        return [cat if r == owner else None for r in range(self.world)]


class DistExchange(Exchange):
    """The one rank of this process, over a ``torch.distributed`` group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.ranks = [dist.get_rank(group)]
        self._gloo = dist.get_backend(group) == "gloo"

    def all_to_all(self, xs):
        (x,) = xs
        out = torch.empty_like(x)
        self._dist.all_to_all_single(out, x.contiguous(), group=self.group)
        return [out.view(self.world, x.shape[0] // self.world, *x.shape[1:])]

    def reduce_scatter_sum(self, xs):
        (x,) = xs
        n = x.shape[0] // self.world
        if self._gloo:  # gloo has no reduce-scatter: all-reduce, keep this rank's chunk
            y = x.clone()
            self._dist.all_reduce(y, group=self.group)
            r = self.ranks[0]
            return [y[r * n:(r + 1) * n].contiguous()]
        out = torch.empty((n, *x.shape[1:]), dtype=x.dtype, device=x.device)
        self._dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return [out]

    def all_reduce_sum(self, xs):
        (x,) = xs
        y = x.clone()
        self._dist.all_reduce(y, group=self.group)
        return [y]

    def all_gather(self, xs):
        (x,) = xs
        x = x.contiguous()
        if self._gloo:
            parts = [torch.empty_like(x) for _ in range(self.world)]
            self._dist.all_gather(parts, x, group=self.group)
            return [torch.cat(parts)]
        out = torch.empty((self.world * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
        self._dist.all_gather_into_tensor(out, x, group=self.group)
        return [out]

    def gather_to(self, owner: int, xs):
        out, wait = self.gather_to_async(owner, xs)
        wait()
        return out

    def gather_to_async(self, owner: int, xs):
        (x,) = xs
        x = x.contiguous()
        me = self.ranks[0]
        if me == owner:  # the ranks' parts land in one buffer, in rank order
            buf = torch.empty((self.world * x.shape[0], *x.shape[1:]), dtype=x.dtype,
                              device=x.device)
            parts = list(buf.chunk(self.world))
        else:
            buf, parts = None, None
        work = self._dist.gather(x, gather_list=parts, dst=owner, group=self.group, async_op=True)
        return [buf], work.wait


@dataclass
class ShardWeights:
    """One rank's view of a layer's weights: its own geometry columns, the
    rest shared."""

    geometry_ext: torch.Tensor   # (3, 128, Hkv_rank*d) bf16 terms of [W ; R W] for the rank's heads
    hadamard: torch.Tensor       # (64, 64) f32
    prototypes: torch.Tensor     # (64, 64) f32
    mlp: torch.Tensor            # packed indexer MLP
    theta_split: torch.Tensor | None  # (2, d_mem, Hkv*d) bf16: used on the layer's owner

    @classmethod
    def prepare(cls, shard: HeadShard, *, geometry, prototypes, hadamard, mlp_params,
                theta=None, n_q_heads: int, head_dim: int = 128, device="cuda"):
        dev = torch.device(device)
        cols = slice(shard.h0 * head_dim, shard.h1 * head_dim)
        g = geometry.to(dev, torch.float32)[:, cols].contiguous()
        had = hadamard.to(dev, torch.float32).contiguous()
        ts = None
        if theta is not None:
            groups = n_q_heads // shard.n_kv_heads
            fold = engine.fold_groups(theta.to(dev, torch.float32), shard.n_kv_heads, groups,
                                      head_dim)
            ts = ops.split_bf16(fold, 2)
        return cls(geometry_ext=ops.prepare_geometry(g, had), hadamard=had,
                   prototypes=prototypes.to(dev, torch.float32).contiguous(),
                   mlp=ops.pack_mlp([t.to(dev) for t in mlp_params]), theta_split=ts)


def compress_layer_sharded(ex: Exchange, shards, inputs, weights, *, layer_idx: int,
                           n_kept: int, positions: torch.Tensor, original_length: int,
                           is_prefill: bool, n_sink: int = 4, topk_qk: int = 4,
                           n_recent_queries: int = 16, shrinkage_rho: float = 0.1,
                           write_memory: bool = True,
                           memory: engine.MemoryState | None = None, gamma: float = 0.9,
                           eta: float = 1.0, student_temp: float = 1.0,
                           special: torch.Tensor | None = None,
                           keep_features: bool = False, qk_events=None,
                           bulk: Exchange | None = None) -> list:
    """One layer of one sequence on head-sharded caches.

    ``shards``, ``inputs`` and ``weights`` are lists indexed like
    ``ex.ranks``: inputs[i] = dict(q (1, Hq_rank, nq, d), keys, values
    (1, Hkv_rank, L, d)) bf16.  ``memory`` is the layer's state on its owner
    rank (ignored elsewhere).  Returns per rank a dict with the rank's retained
    ``keys``/``values``, ``keep``/``evict`` (1, n) int32 (the same on every
    rank), ``scores`` (1, L) and, with ``keep_features``, the rank's range of
    features (n_keys, 14).

    ``write_memory`` must be the same on every rank: it decides whether the
    ranks take part in gathering K/V rows to the owner, which then writes
    ``memory`` with its ``theta_split``.  ``bulk``: an exchange over a second
    communicator for that gather, so that it overlaps the rest of the layer
    (default: ``ex``).  ``qk_events``: optional (start, end) CUDA events
    recorded around the QK summaries (LSE, relation, the rank's merge).

    Issue order: every exchange is issued as soon as its inputs are queued,
    and the exchanges that depend only on the first compute stage go back to
    back, so that the ranks' small kernels do not wait on one another more
    often than the reductions require.
    """
    R = range(len(ex.ranks))
    bulk = bulk or ex
    L = shards[0].seq_len
    nq = inputs[0]["q"].shape[2]
    hkv = shards[0].n_kv_heads
    words = ops.qk_summary_words(nq)
    dev = inputs[0]["keys"].device
    pos = positions.to(torch.int64).reshape(-1).contiguous()
    sp = None if special is None else special.reshape(-1).contiguous()
    compact = n_kept < L
    n_ev = L - n_kept
    write = compact and write_memory
    # Memory write inputs: when most of the cache is evicted the ranks send
    # their whole K/V (no copy on the sender, the owner gathers the rows);
    # otherwise the evicted rows only, after Top-B.
    whole = 4 * n_ev >= 3 * L
    owner = HeadShard.owner(layer_idx, ex.world)
    if write and whole:
        kv_all, kv_wait = [], []
        for t in ("keys", "values"):
            out, wait = bulk.gather_to_async(owner, [inputs[i][t][0] for i in R])
            kv_all.append(out)
            kv_wait.append(wait)

    # stage A: the rank's own heads over all keys
    summ, ys, hs = [], [], []
    for i in R:
        sh = shards[i]
        s_ = torch.empty(sh.padded, words, dtype=torch.int32, device=dev)
        if qk_events is not None:
            qk_events[0].record()
        ops.qk_head_summary(inputs[i]["q"], inputs[i]["keys"], s_, topk_qk=topk_qk,
                            n_recent_queries=n_recent_queries)
        if qk_events is not None:
            qk_events[1].record()
        y = torch.empty(sh.padded, 64, dtype=torch.float32, device=dev)
        ops.coverage_partial_projection(inputs[i]["keys"], weights[i].geometry_ext, y)
        h = torch.empty(sh.heads_per_rank, sh.padded, dtype=torch.float32, device=dev)
        ops.value_head_sums(inputs[i]["values"], h)
        summ.append(s_)
        ys.append(y)
        hs.append(h)
    parts = ex.all_to_all(summ)
    y_range = ex.reduce_scatter_sum(ys)
    hs = ex.all_gather(hs)

    # stage B: the rank's key range
    feats, zs, totals = [], [], []
    for i in R:
        sh = shards[i]
        f = torch.empty(max(sh.chunk, 1), 14, dtype=torch.float32, device=dev)
        ops.qk_merge_summaries(parts[i].contiguous(), f, key0=sh.k0, n_keys=sh.n_keys, seq_len=L,
                               n_queries=nq, n_kv_heads=hkv, topk_qk=topk_qk,
                               n_recent_queries=n_recent_queries)
        z, zt, tot = ops.coverage_range_totals(y_range[i][:sh.n_keys], weights[i].hadamard)
        feats.append(f)
        zs.append((z, zt))
        totals.append(tot)
    totals = ex.all_reduce_sum(totals)
    assigns, hists = [], []
    for i in R:
        z, zt = zs[i]
        a, h = ops.coverage_range_assign(totals[i], L, z, zt, weights[i].prototypes, feats[i],
                                         col0=6, shrinkage_rho=shrinkage_rho)
        assigns.append(a)
        hists.append(h)
    hists = ex.all_reduce_sum(hists)
    sc = []
    for i in R:
        sh = shards[i]
        ops.coverage_range_occupancy(assigns[i], hists[i], feats[i], sh.n_keys, col0=6)
        s_ = torch.empty(sh.chunk, dtype=torch.float32, device=dev)
        if sh.n_keys > 0:
            s_[:sh.n_keys] = ops.indexer_scores_from_sums(
                hs[i], sh.k0, sh.n_keys, pos, feats[i], weights[i].mlp,
                original_length=original_length, is_prefill=is_prefill, n_sink=n_sink,
                special=sp)
        sc.append(s_)
    # every rank gets all scores and runs the same Top-B (identical keep sets)
    scores = [x[:L][None] for x in ex.all_gather(sc)]
    keeps = [ops.topb_select(scores[i], n_kept, n_sink) if compact else (None, None) for i in R]

    # memory write on the layer's owner
    if write:
        if whole:
            k_all, v_all = kv_all
        else:
            k_send, v_send = [], []
            for i in R:
                ke, ve = ops.compact_kv(inputs[i]["keys"], inputs[i]["values"], keeps[i][1])
                k_send.append(ke[0])
                v_send.append(ve[0])
            k_all, wk = bulk.gather_to_async(owner, k_send)
            v_all, wv = bulk.gather_to_async(owner, v_send)
            kv_wait = [wk, wv]
        for w in kv_wait:
            w()
        for i in R:
            if ex.ranks[i] == owner:
                if memory is None or weights[i].theta_split is None:
                    raise ValueError("the owner of the layer needs its memory state and theta_split")
                fn = ops.memory_write if whole else ops.memory_write_gathered
                fn(k_all[i][None], v_all[i][None], scores[i], keeps[i][1], weights[i].theta_split,
                   memory.M, memory.b, memory.Z, gamma=gamma, eta=eta, student_temp=student_temp)

    # the rank's own retained K/V
    out = []
    for i in R:
        keep, evict = keeps[i]
        if compact:
            ok, ov = ops.compact_kv(inputs[i]["keys"], inputs[i]["values"], keep)
        else:
            ok, ov = inputs[i]["keys"], inputs[i]["values"]
        d = dict(keys=ok, values=ov, keep=keep, evict=evict, scores=scores[i])
        if keep_features:
            d["features"] = feats[i][:shards[i].n_keys]
        out.append(d)
    return out
