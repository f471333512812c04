"""Seeded synthetic Llama-shaped inputs for the compression step.

Queries and keys are N(0, 1)/sqrt(d) with four outlier channels per KV head
(shared by the head's query group) scaled by 8; values are N(0, 1).  The
outlier channel indices come from the seed.  These stand in for the RULER /
LongBench caches the reference evaluates on; only their shapes (context
length, query buffer, head geometry) are borrowed.
"""

from __future__ import annotations

import torch


def outlier_channels(seed: int, n_kv_heads: int, head_dim: int = 128) -> torch.Tensor:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) + 7919)
    return torch.stack([torch.randperm(head_dim, generator=g)[:4] for _ in range(n_kv_heads)])


def gaussian_outliers(shape, outliers: torch.Tensor, groups: int, *, generator, device,
                      dtype=torch.bfloat16, scale: float = 8.0) -> torch.Tensor:
    """(B, H, N, d) with H = outliers.shape[0] * groups."""
    B, H, N, d = shape
    x = torch.randn(shape, generator=generator, device=device, dtype=torch.float32) / d ** 0.5
    mult = torch.ones(H, d, device=device)
    idx = outliers.to(device).repeat_interleave(groups, dim=0)
    mult.scatter_(1, idx, scale)
    x.mul_(mult[None, :, None, :])
    return x.to(dtype)


def make_layer_inputs(*, seed: int, batch: int, n_kv_heads: int, n_q_heads: int, seq_len: int,
                      n_queries: int, head_dim: int = 128, device="cuda",
                      dtype=torch.bfloat16):
    """Returns (q (B, Hq, nq, d), k (B, Hkv, L, d), v (B, Hkv, L, d))."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    out = outlier_channels(seed, n_kv_heads, head_dim)
    groups = n_q_heads // n_kv_heads
    k = gaussian_outliers((batch, n_kv_heads, seq_len, head_dim), out, 1, generator=g,
                          device=device, dtype=dtype)
    q = gaussian_outliers((batch, n_q_heads, n_queries, head_dim), out, groups, generator=g,
                          device=device, dtype=dtype)
    v = torch.randn((batch, n_kv_heads, seq_len, head_dim), generator=g, device=device,
                    dtype=torch.float32).to(dtype)
    return q, k, v


def make_layer_weights(*, seed: int, n_kv_heads: int, n_q_heads: int, head_dim: int = 128,
                       d_mem: int = 512, gate_hidden: int = 64, hidden: int = 128,
                       proto_dim: int = 64, n_prototypes: int = 64):
    """Random-init slow weights of one layer (CPU float32 tensors), with the
    same initialisers as torch.nn.Linear and the reference's fixed geometry
    constructions (Gaussian projection / sqrt(P), unit prototypes, random-sign
    Hadamard rotation)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))

    def linear(out_f, in_f):
        bound = 1.0 / in_f ** 0.5
        w = (torch.rand(out_f, in_f, generator=g) * 2 - 1) * bound
        b = (torch.rand(out_f, generator=g) * 2 - 1) * bound
        return w, b

    w1, b1 = linear(128, 14)
    w2, b2 = linear(128, 128)
    w3, b3 = linear(1, 128)
    d_model = n_q_heads * head_dim
    theta, _ = linear(d_mem, d_model)
    gw1, gb1 = linear(gate_hidden, d_model)
    gw2, gb2 = linear(1, gate_hidden)
    o_proj, _ = linear(hidden, d_model)
    geometry = torch.randn(proto_dim, n_kv_heads * head_dim, generator=g) / proto_dim ** 0.5
    protos = torch.randn(n_prototypes, proto_dim, generator=g)
    protos = protos / protos.norm(dim=1, keepdim=True).clamp_min(1e-8)
    signs = torch.where(torch.rand(proto_dim, generator=g) < 0.5, -1.0, 1.0)
    H = torch.ones(1, 1)
    while H.shape[0] < proto_dim:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    hadamard = (H[:proto_dim, :proto_dim] * signs[None, :]) / proto_dim ** 0.5
    return dict(mlp=(w1, b1, w2, b2, w3, b3), theta=theta, gate=(gw1, gb1, gw2, gb2),
                o_proj=o_proj, geometry=geometry, prototypes=protos, hadamard=hadamard)
