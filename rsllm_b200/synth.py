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


def decode_slots(n_seq: int, n_steps: int, seed: int, len_range: tuple[int, int] = (1024, 32768)):
    """The slot mappings of ``n_steps`` decode steps of the benchmark's
    config 2: ``n_seq`` sequences with current lengths uniform in
    ``len_range`` (seed ``seed``) each append one token per step; the pages the
    run touches (each sequence's current page and every page it crosses into)
    get physical ids from a seeded permutation (seed ``seed + 1``).
    Returns ``(slots int32 [n_steps, n_seq], n_pages, lens int64 [n_seq])``."""
    import numpy as np

    lens = uniform_ints(n_seq, *len_range, seed=seed).numpy().astype(np.int64)
    first = lens // 64
    need = (lens + n_steps - 1) // 64 - first + 1
    off = np.concatenate([[0], np.cumsum(need)])
    n_pages = int(off[-1])
    phys = permutation(n_pages, seed=seed + 1).numpy().astype(np.int64)
    pos = lens[None, :] + np.arange(n_steps)[:, None]
    page = phys[off[:-1][None, :] + pos // 64 - first[None, :]]
    return (page * 64 + pos % 64).astype(np.int32), n_pages, lens
