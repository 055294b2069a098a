"""Seeded synthetic inputs shared by the golden generator, the tests and bench.py.

Every cache is i.i.d. N(0, 1) in the requested dtype drawn from
``torch.Generator().manual_seed(seed)`` on the CPU, and block ids come from
``torch.randperm(N, generator=...)``, as the benchmark configurations specify.
The recipes are frozen: golden digests in ``tests/golden/`` depend on them.
"""
from __future__ import annotations

import hashlib

import torch


def seeded_cache(shape, seed: int, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator().manual_seed(int(seed))
    return torch.randn(tuple(shape), generator=g, dtype=dtype)


def seeded_perm(n: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(int(seed))
    return torch.randperm(int(n), generator=g).tolist()


def config1_inputs():
    """benchmark config 1: two [2, 28, 64, 256, 8, 128] bf16 caches (seeds 0 and 1),
    8 source ids from randperm(64, seed 0), 8 destination ids from randperm(64, seed 1)."""
    shape = (2, 28, 64, 256, 8, 128)
    src = seeded_cache(shape, 0)
    dst = seeded_cache(shape, 1)
    src_ids = seeded_perm(64, 0)[:8]
    dst_ids = seeded_perm(64, 1)[:8]
    return src, dst, src_ids, dst_ids


def sha256_of(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    return hashlib.sha256(t.view(torch.uint8).reshape(-1).numpy()).hexdigest()


def slot_mapping(num_tokens: int, num_slots: int, seed: int, skip_fraction: float = 0.1) -> torch.Tensor:
    """Distinct random slots with about `skip_fraction` of entries set to -1 (padding)."""
    g = torch.Generator().manual_seed(int(seed))
    slots = torch.randperm(int(num_slots), generator=g)[:num_tokens].to(torch.int64)
    skip = torch.rand(num_tokens, generator=g) < skip_fraction
    slots[skip] = -1
    return slots
