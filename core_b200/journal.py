"""Device-resident token journal of a compressed cache.

Counterpart of ``CacheMetadata`` (core/cache_metadata.py:6-54): for every
layer it knows which original token position (and token id) sits in each
slot of the compacted KV cache, so that the auxiliary features (token age,
sink flag, special-token flag; core/features.py:861-921) see original
positions after any number of evictions.

Design: the token ids live in one device buffer that grows by doubling, and
each layer's slot positions are a device tensor; the host keeps only integer
extents.  Appending cache slots, looking up their ids and dropping evicted
slots are device operations with no host synchronisation.  The single
remaining host read is in :meth:`CacheMetadata.record` when the caller passes
explicit device ``position_ids`` (their largest value sizes the journal),
once per model forward.
"""

from __future__ import annotations

import torch


class CacheMetadata:
    """Original positions and token ids behind the compacted cache slots.

    ``positions[layer]`` : (B, L) int64 device tensor, slot -> original position
    ``next_position[layer]``: next original position a new slot of that layer gets
    ``token_ids``        : (B, extent) int64, original position -> token id (-1: unknown)
    """

    def __init__(self):
        self.reset()

    def reset(self) -> None:
        """Forget the sequence (call at every sample boundary)."""
        self._ids: torch.Tensor | None = None  # (B, capacity) int64, -1 where unknown
        self._extent = 0                       # positions [0, extent) are journaled
        self.positions: dict = {}
        self.next_position: dict = {}

    @property
    def token_ids(self) -> torch.Tensor | None:
        return None if self._ids is None else self._ids[:, : self._extent]

    # ---- token ids, once per model forward ----
    def _reserve(self, batch: int, extent: int, like: torch.Tensor) -> None:
        if self._ids is None:
            cap = max(256, extent)
            self._ids = torch.full((batch, cap), -1, dtype=torch.long, device=like.device)
            return
        if self._ids.shape[0] != batch:
            raise ValueError("the batch size changed inside one sequence; call reset() between "
                             "sequences")
        if extent > self._ids.shape[1]:
            cap = max(extent, 2 * self._ids.shape[1])
            grown = torch.full((batch, cap), -1, dtype=torch.long, device=self._ids.device)
            grown[:, : self._extent].copy_(self._ids[:, : self._extent])
            self._ids = grown

    def record(self, input_ids: torch.Tensor, position_ids: torch.Tensor | None = None) -> None:
        """Journal the ids of tokens entering the model at ``position_ids``
        (default: right after the journaled extent)."""
        if input_ids is None:
            raise ValueError("CORE token metadata requires the input token ids")
        batch, n = input_ids.shape
        ids = input_ids.long()
        if position_ids is None:
            start = self._extent
            self._reserve(batch, start + n, ids)
            self._ids[:, start:start + n].copy_(ids)
            self._extent = start + n
            return
        pos = position_ids.long().expand(batch, -1)
        top = int(pos.max()) + 1 if pos.numel() else 0  # the one host read
        extent = max(top, self._extent)
        self._reserve(batch, extent, ids)
        self._ids.scatter_(1, pos.to(self._ids.device), ids.to(self._ids.device))
        self._extent = extent

    # ---- per layer ----
    def align(self, layer_idx: int, batch_size: int, cache_length: int, device):
        """Extend layer ``layer_idx``'s slot map to ``cache_length`` slots (new
        slots take the next original positions) and return
        ``(positions (B, L) int64, token ids (B, L) int64, next_position)``."""
        held = self.positions.get(layer_idx)
        have = 0 if held is None else held.shape[1]
        if cache_length < have:
            raise RuntimeError(f"the cache of layer {layer_idx} holds {cache_length} slots but "
                               f"the journal {have}: it was pruned without the journal; call "
                               "reset_cache() at sequence boundaries")
        first = self.next_position.get(layer_idx, 0)
        grow = cache_length - have
        if grow or held is None:
            new = torch.arange(first, first + grow, device=device, dtype=torch.long)
            new = new[None].expand(batch_size, grow)
            held = new if held is None else torch.cat((held.to(device), new), dim=1)
            self.positions[layer_idx] = held
        self.next_position[layer_idx] = first + grow
        if self._ids is None:
            ids = torch.full_like(held, -1)
        else:
            # every slot's position is below next_position, so this bound is sufficient
            if held.numel() and first + grow > self._extent:
                raise RuntimeError(f"token ids of positions up to {first + grow - 1} were never "
                                   f"recorded (journal covers {self._extent})")
            ids = self._ids.to(device).gather(1, held)
        return held, ids, first + grow

    def retain(self, layer_idx: int, indices: torch.Tensor) -> None:
        """Keep the slots ``indices`` (B, n_kept) of layer ``layer_idx``, in that order."""
        self.positions[layer_idx] = self.positions[layer_idx].gather(1, indices.long()).contiguous()
