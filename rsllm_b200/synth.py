"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations: bf16 KV rows drawn from N(0, 1) with a seeded 1% of
elements scaled by 20 (outliers), physical page orders from seeded random
permutations, and f32 indexer scores from N(0, 1).

Generation runs on the CPU with torch's seeded generator, so the same seed
gives the same bytes on every machine; large inputs can be made on the GPU
(``device="cuda"``), which is deterministic for a given GPU and seed.
"""
from __future__ import annotations

import torch

ROW_DIM = 576


def kv_rows(n: int, seed: int, device: str | torch.device = "cpu", outlier_frac: float = 0.01,
            outlier_scale: float = 20.0) -> torch.Tensor:
    """bf16 [n, 576]: N(0,1) with ``outlier_frac`` of elements x ``outlier_scale``."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((n, ROW_DIM), generator=g, device=dev, dtype=torch.float32)
    mask = torch.rand((n, ROW_DIM), generator=g, device=dev) < outlier_frac
    x = torch.where(mask, x * outlier_scale, x)
    return x.to(torch.bfloat16)


def permutation(n: int, seed: int) -> torch.Tensor:
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randperm(n, generator=g).to(torch.int32)


def scores(n_q: int, n_keys: int, seed: int, device: str | torch.device = "cpu") -> torch.Tensor:
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn((n_q, n_keys), generator=g, device=dev, dtype=torch.float32)


def uniform_ints(n: int, lo: int, hi: int, seed: int) -> torch.Tensor:
    """int32 [n] uniform in [lo, hi]."""
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g, dtype=torch.int64).to(torch.int32)
