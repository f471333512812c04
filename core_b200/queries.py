"""Decode-time query buffer and post-RoPE query reconstruction.

``HiddenStateWindow`` replaces the per-layer Python list of cloned hidden
states that the decoding press concatenates at every compression
(kvpress/kvpress/presses/decoding_press.py:144,168,183-187): the hidden
states are copied into one preallocated device buffer per layer, and a
compression reads the retained entries as a contiguous view, with no
``torch.cat`` and no host synchronisation.

``post_rope_queries`` rebuilds the post-RoPE queries of buffered hidden states
(core/collector.py:135-201): the q_proj GEMM is a library call, the rotary
embedding and the transpose to the QK kernels' (B, Hq, T, d) layout are one
kernel of the CUDA library (``core_rope_queries``).
"""

from __future__ import annotations

from collections import deque

import torch

from . import ops

# rotary types whose inverse frequencies never change after construction: the
# kernel recomputes cos / sin from inv_freq itself
_STATIC_ROPE = ("default", "linear", "llama3", "yarn")


class HiddenStateWindow:
    """The last ``max_entries`` hidden-state entries (one per forward call)
    of one layer, kept in a device buffer.

    Entries may hold several tokens (a multi-token forward); retention counts
    entries, as the reference's list slicing does.  ``view()`` returns the
    retained tokens, oldest first, as a (B, T, H) view of the buffer.
    """

    def __init__(self, max_entries: int):
        self.max_entries = int(max_entries)
        self._buf: torch.Tensor | None = None
        self._lens: deque = deque()   # tokens per retained entry, oldest first
        self._end = 0                 # buffer column after the newest token

    @property
    def n_entries(self) -> int:
        return len(self._lens)

    @property
    def n_tokens(self) -> int:
        return sum(self._lens)

    def _room(self, hs: torch.Tensor) -> None:
        b, n, h = hs.shape
        keep = self.n_tokens
        buf = self._buf
        fits = (buf is not None and buf.shape[0] == b and buf.shape[2] == h
                and buf.dtype == hs.dtype and buf.device == hs.device)
        if fits and self._end + n <= buf.shape[1]:
            return
        start = self._end - keep
        need = keep + n
        if fits and need <= buf.shape[1] // 2:
            # slide the retained tokens to the front (through a copy: the ranges may overlap)
            if keep:
                buf[:, :keep].copy_(buf[:, start:self._end].clone())
            self._end = keep
            return
        cap = max(2 * need, 2 * max(1, self.max_entries) * n, 64)
        grown = torch.empty(b, cap, h, dtype=hs.dtype, device=hs.device)
        if keep and fits:
            grown[:, :keep].copy_(buf[:, start:self._end])
        elif keep:  # the shape or dtype changed: drop what no longer fits
            self._lens.clear()
            keep = 0
        self._buf = grown
        self._end = keep

    def append(self, hidden_states: torch.Tensor) -> None:
        hs = hidden_states.detach()
        self._room(hs)
        n = hs.shape[1]
        self._buf[:, self._end:self._end + n].copy_(hs)
        self._end += n
        self._lens.append(n)

    def view(self) -> torch.Tensor:
        t = self.n_tokens
        return self._buf[:, self._end - t:self._end]

    def clear(self) -> None:
        self._lens.clear()

    def trim(self) -> None:
        """Drop the oldest entries beyond ``max_entries`` (all of them when
        ``max_entries`` is not positive)."""
        keep = self.max_entries if self.max_entries > 0 else 0
        while len(self._lens) > keep:
            self._lens.popleft()


def decode_positions(kwargs: dict, n_tokens: int, device) -> torch.Tensor | None:
    """Absolute positions (1, T) of the T buffered decode queries, ending at the
    current token (core/kvpress_adapter.py:479-502): the last explicit
    ``position_ids`` of batch row 0, else the last ``cache_position``.
    Computed on the device (no host read)."""
    cur = kwargs.get("position_ids")
    if cur is not None:
        end = cur[0, -1]
    elif kwargs.get("cache_position") is not None:
        end = kwargs["cache_position"][-1]
    else:
        return None
    steps = torch.arange(n_tokens, device=device, dtype=torch.long)
    return (end.to(device=device, dtype=torch.long) - (n_tokens - 1) + steps)[None]


def _rotary(attn_module):
    return getattr(attn_module, "rotary_emb", None)


def post_rope_queries(attn_module, hidden_states: torch.Tensor, position_ids=None,
                      position_embeddings=None) -> torch.Tensor | None:
    """q = RoPE(q_proj(h)) as (B, Hq, T, d), or None when the module has no
    q_proj or no rotary embedding to use (core/collector.py:135-201).

    ``position_embeddings`` (cos, sin) are used as given; otherwise the
    module's rotary embedding at ``position_ids`` (default 0..T-1).  The
    rotation runs in the library's RoPE kernel: CUDA tensors only.
    """
    if not hasattr(attn_module, "q_proj"):
        return None
    bsz, t, _ = hidden_states.shape
    cfg = attn_module.config
    n_heads = getattr(attn_module, "num_heads", cfg.num_attention_heads)
    head_dim = getattr(attn_module, "head_dim", cfg.hidden_size // cfg.num_attention_heads)
    proj = attn_module.q_proj(hidden_states)
    if hasattr(attn_module, "q_norm"):
        proj = attn_module.q_norm(proj.view(bsz, t, n_heads, head_dim)).reshape(bsz, t, -1)
    if position_embeddings is not None:
        cos, sin = position_embeddings
        return ops.rope_queries(proj, n_heads, cos=cos, sin=sin).detach()
    rot = _rotary(attn_module)
    if rot is None:
        return None
    if position_ids is None:
        position_ids = torch.arange(t, device=proj.device, dtype=torch.long)[None]
    if getattr(rot, "rope_type", "default") in _STATIC_ROPE and hasattr(rot, "inv_freq"):
        return ops.rope_queries(proj, n_heads, positions=position_ids.to(proj.device),
                                inv_freq=rot.inv_freq,
                                attention_scaling=float(getattr(rot, "attention_scaling", 1.0))
                                ).detach()
    try:  # rotary types that update their frequencies per call: let the module compute cos/sin
        cos, sin = rot(proj, position_ids)
    except (TypeError, ValueError):
        return None
    return ops.rope_queries(proj, n_heads, cos=cos, sin=sin).detach()

