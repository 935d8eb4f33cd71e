"""Seeded synthetic prompt K/V and decode queries with RefineKV's benchmark shapes.

The reference measures on real prompts (LongBench/RULER/HELMET) through real
Llama/Qwen weights; neither is available here, so these generators stand in
with the shapes and value distributions of the benchmark configuration:

* keys: per (kv head, channel) scale ``s_c ~ LogNormal(0, 0.5)``, entries
  ``N(0, s_c^2)``, rotated with rotate-half RoPE (theta 500000) at positions
  ``0..N-1``;
* values: ``N(0, 1)``;
* six planted random blocks per layer; every query row is
  ``0.7 * mean(keys of the planted blocks) + 0.3 * N(0, 1)``, which makes the
  selection non-trivial;
* every decode step appends one fresh ``N(0, 1)`` K/V token, the key rotated
  at position ``N + step``.

Everything is drawn from an explicit ``torch.Generator`` so a (seed, layer)
pair always gives the same tensors on the same device type.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

ROPE_THETA = 500000.0
PLANTED_BLOCKS = 6


def rope_tables(positions: torch.Tensor, dim: int, theta: float = ROPE_THETA):
    """cos/sin tables (len(positions), dim) for rotate-half RoPE, in FP32."""
    inv = theta ** (-torch.arange(0, dim, 2, device=positions.device, dtype=torch.float32) / dim)
    ang = positions.to(torch.float32)[:, None] * inv[None, :]
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float = ROPE_THETA):
    """Rotate-half RoPE over the last dim of (..., tokens, dim) FP32 ``x``."""
    cos, sin = rope_tables(positions, x.shape[-1], theta)
    half = x.shape[-1] // 2
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rotated * sin


@dataclass
class LayerInputs:
    keys: torch.Tensor          # (kv_heads, tokens, dim)
    values: torch.Tensor        # (kv_heads, tokens, dim)
    planted: torch.Tensor       # (PLANTED_BLOCKS,) int64 block ids
    planted_mean: torch.Tensor  # (kv_heads, dim) FP32 mean key of the planted blocks


def make_layer(seed: int, layer: int, kv_heads: int, tokens: int, dim: int, block_size: int,
               dtype=torch.bfloat16, device="cpu", chunk_tokens: int = 1 << 16) -> LayerInputs:
    """Prompt K/V for one layer; generated in token chunks to bound FP32 temporaries."""
    gen = torch.Generator(device=device).manual_seed(seed * 1_000_003 + layer)
    scale = torch.empty(kv_heads, dim, device=device).log_normal_(0.0, 0.5, generator=gen)
    keys = torch.empty(kv_heads, tokens, dim, device=device, dtype=dtype)
    values = torch.empty(kv_heads, tokens, dim, device=device, dtype=dtype)
    for start in range(0, tokens, chunk_tokens):
        stop = min(tokens, start + chunk_tokens)
        raw = torch.randn(kv_heads, stop - start, dim, device=device, generator=gen)
        pos = torch.arange(start, stop, device=device)
        keys[:, start:stop] = apply_rope(raw * scale[:, None, :], pos).to(dtype)
        values[:, start:stop] = torch.randn(
            kv_heads, stop - start, dim, device=device, generator=gen).to(dtype)
    blocks = -(-tokens // block_size)
    planted = torch.randperm(blocks, generator=gen, device=device)[:PLANTED_BLOCKS]
    rows = []
    for b in planted.tolist():
        rows.append(keys[:, b * block_size: min(tokens, (b + 1) * block_size)].float())
    planted_mean = torch.cat(rows, dim=1).mean(1)
    return LayerInputs(keys, values, planted, planted_mean)


def make_queries(seed: int, layer: int, step: int, planted_mean: torch.Tensor, group: int,
                 count: int = 1, dtype=torch.bfloat16) -> torch.Tensor:
    """(count, kv_heads, group, 1, dim) queries near the planted blocks' mean key."""
    heads, dim = planted_mean.shape
    gen = torch.Generator(device=planted_mean.device).manual_seed(
        (seed * 1_000_003 + layer) * 7919 + 104_729 + step)
    noise = torch.randn(count, heads, group, 1, dim, device=planted_mean.device, generator=gen)
    q = 0.7 * planted_mean[None, :, None, None, :] + 0.3 * noise
    return q.to(dtype)


def make_decode_token(seed: int, layer: int, step: int, kv_heads: int, dim: int, position: int,
                      dtype=torch.bfloat16, device="cpu"):
    """One fresh (kv_heads, 1, dim) K/V token for decode step ``step`` at ``position``."""
    gen = torch.Generator(device=device).manual_seed(
        (seed * 1_000_003 + layer) * 104_729 + 7919 + step)
    k = torch.randn(kv_heads, 1, dim, device=device, generator=gen)
    v = torch.randn(kv_heads, 1, dim, device=device, generator=gen)
    pos = torch.tensor([position], device=device)
    return apply_rope(k, pos).to(dtype), v.to(dtype)
