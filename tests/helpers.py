"""Shared helpers for the test suite (inputs, digests); imports only torch."""

import hashlib

import torch


def reference_inputs(length, dim, seed=42, device="cpu"):
    """Seed-42 bf16 draw of the reference tests (tests/test_attention.py:10-16)."""
    gen = torch.Generator(device=device).manual_seed(seed)

    def normal(shape):
        return torch.randn(shape, device=device, generator=gen, dtype=torch.bfloat16)

    return normal((2, 4, 1, dim)), normal((2, length, dim)), normal((2, length, dim))


def checksum(t: torch.Tensor) -> list:
    f = t.detach().float().reshape(-1).cpu()
    idx = torch.linspace(0, f.numel() - 1, steps=min(64, f.numel())).long()
    return [float(f.double().sum()), float(f.double().abs().sum())] + f[idx].tolist()


def sha256(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.uint8) if t.dtype != torch.bool else t.to(torch.uint8)
    return hashlib.sha256(raw.numpy().tobytes()).hexdigest()


def bf16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 units-in-the-last-place between two bf16 tensors (same sign domain)."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    # map sign-magnitude to a monotone integer line
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return (ia - ib).abs()
