"""Seeded synthetic graphs and CIGN workloads with the shapes of the
benchmark configurations (the reference's datasets are not available; none
of their records are reproduced).

* ``erdos_renyi(n, avg_degree, seed)``           -- cfg1 (N=2,000, degree 8)
* ``powerlaw_graph(n, num_edges, exponent, ...)``  -- cfg2/3 (N=24,492,
  186,100 directed edges, exponent 2.5, min degree 1): Chung-Lu sampling with
  expected degrees drawn from a discrete power law (a configuration-model
  stand-in), self-loops and duplicate directed pairs removed, topped up to
  exactly `num_edges` edges.
* ``rmat_graph(scale, num_edges, a, b, c, ...)``   -- cfg4/5 (RMAT a=.57,
  b=.19, c=.19), node ids truncated to `n`.

All generators return a PyG-style int64 edge_index [2, E] (source, target)
on the CPU; ``build_workload`` turns one into the tensors a CIGN training
step consumes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch


def erdos_renyi(n: int, avg_degree: float, seed: int = 0) -> torch.Tensor:
    g = np.random.default_rng(seed)
    m = int(round(n * avg_degree / 2))
    seen = set()
    src, dst = [], []
    while len(src) < m:
        u = g.integers(0, n, size=2 * (m - len(src)) + 16)
        v = g.integers(0, n, size=u.size)
        for a, b in zip(u.tolist(), v.tolist()):
            if a == b:
                continue
            k = (min(a, b), max(a, b))
            if k in seen:
                continue
            seen.add(k)
            src.append(k[0])
            dst.append(k[1])
            if len(src) == m:
                break
    return torch.tensor([src, dst], dtype=torch.int64)


def _unique_pairs(src: np.ndarray, dst: np.ndarray, n: int):
    keep = src != dst
    src, dst = src[keep], dst[keep]
    key = src.astype(np.int64) * n + dst
    _, first = np.unique(key, return_index=True)
    first.sort()
    return src[first], dst[first]


def powerlaw_graph(n: int, num_edges: int, exponent: float = 2.5, min_degree: int = 1,
                   seed: int = 0) -> torch.Tensor:
    g = np.random.default_rng(seed)
    u = g.random(n)
    deg = np.floor(min_degree * np.power(1.0 - u, -1.0 / (exponent - 1.0)))
    deg = np.clip(deg, min_degree, n - 1)
    p = deg / deg.sum()
    src = np.empty(0, np.int64)
    dst = np.empty(0, np.int64)
    while src.size < num_edges:
        need = int((num_edges - src.size) * 1.2) + 64
        s = g.choice(n, size=need, p=p)
        d = g.choice(n, size=need, p=p)
        src, dst = _unique_pairs(np.concatenate([src, s]), np.concatenate([dst, d]), n)
    return torch.from_numpy(np.stack([src[:num_edges], dst[:num_edges]]).astype(np.int64))


def rmat_graph(n: int, num_edges: int, a: float = 0.57, b: float = 0.19, c: float = 0.19,
               seed: int = 0, device=None) -> torch.Tensor:
    """R-MAT edges over [0, 2^scale) with scale = ceil(log2 n); ids >= n are
    dropped (truncation), self-loops and duplicates removed, topped up to
    exactly num_edges.  With a CUDA `device` the same recursion draws from
    torch's generator on that device (a different, equally seeded stream;
    seconds instead of minutes for the 61.9M-edge cfg4 graph); the result is
    returned on the CPU either way."""
    if device is not None and torch.device(device).type == "cuda":
        return _rmat_graph_device(n, num_edges, a, b, c, seed, torch.device(device))
    scale = int(np.ceil(np.log2(max(n, 2))))
    g = np.random.default_rng(seed)
    probs = np.array([a, b, c, 1.0 - a - b - c])
    src = np.empty(0, np.int64)
    dst = np.empty(0, np.int64)
    while src.size < num_edges:
        need = int((num_edges - src.size) * 1.3) + 1024
        s = np.zeros(need, np.int64)
        d = np.zeros(need, np.int64)
        for _ in range(scale):
            q = g.choice(4, size=need, p=probs)
            s = (s << 1) | (q >> 1)
            d = (d << 1) | (q & 1)
        ok = (s < n) & (d < n)
        src, dst = _unique_pairs(np.concatenate([src, s[ok]]), np.concatenate([dst, d[ok]]), n)
    return torch.from_numpy(np.stack([src[:num_edges], dst[:num_edges]]).astype(np.int64))


def _rmat_graph_device(n, num_edges, a, b, c, seed, device) -> torch.Tensor:
    scale = int(np.ceil(np.log2(max(n, 2))))
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    keys = torch.empty(0, dtype=torch.int64, device=device)
    order = torch.empty(0, dtype=torch.int64, device=device)  # draw index: keeps first occurrences
    drawn = 0
    while keys.numel() < num_edges:
        need = int((num_edges - keys.numel()) * 1.3) + 1024
        s = torch.zeros(need, dtype=torch.int64, device=device)
        d = torch.zeros(need, dtype=torch.int64, device=device)
        for _ in range(scale):
            r = torch.rand(need, generator=g, device=device)
            q = (r >= a).long() + (r >= a + b).long() + (r >= a + b + c).long()
            s = (s << 1) | (q >> 1)
            d = (d << 1) | (q & 1)
        ok = (s < n) & (d < n) & (s != d)
        k_new = s[ok] * n + d[ok]
        o_new = torch.arange(drawn, drawn + need, device=device)[ok]
        drawn += need
        allk = torch.cat([keys, k_new])
        allo = torch.cat([order, o_new])
        uk, inv = torch.unique(allk, return_inverse=True)
        first = torch.full((uk.numel(),), torch.iinfo(torch.int64).max, dtype=torch.int64,
                           device=device).scatter_reduce(0, inv, allo, reduce="amin")
        sel = torch.argsort(first)
        keys, order = uk[sel], first[sel]
    keys = keys[:num_edges].cpu()
    return torch.stack([keys // n, keys % n])


def random_ratio_split(num_nodes: int, train_ratio: float, val_ratio: float, test_ratio: float,
                       split_seed: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Node masks by one seeded permutation (generic_engine/train_cign.py:1386-1423)."""
    if abs(train_ratio + val_ratio + test_ratio - 1.0) > 1e-6:
        raise ValueError("Ratios must sum to 1.0")
    gen = torch.Generator()
    gen.manual_seed(int(split_seed))
    perm = torch.randperm(num_nodes, generator=gen)
    n_train = int(num_nodes * train_ratio)
    n_val = int(num_nodes * val_ratio)
    masks = [torch.zeros(num_nodes, dtype=torch.bool) for _ in range(3)]
    masks[0][perm[:n_train]] = True
    masks[1][perm[n_train:n_train + n_val]] = True
    masks[2][perm[n_train + n_val:]] = True
    return masks[0], masks[1], masks[2]


@dataclass
class WorkloadConfig:
    name: str
    num_nodes: int
    num_edges: int
    generator: str  # "er" | "powerlaw" | "rmat"
    in_dim: int
    num_classes: int
    hidden_dim: int
    hops: Tuple[int, ...]
    heads: int
    layers: int
    dropout: float
    gat_dropout: float
    seed: int = 0
    avg_degree: float = 8.0


# The benchmark configurations that a single GPU runs (cfg2 is the headline
# training step; cfg1 the CPU-runnable case; cfg4 the large RMAT graph).
CONFIGS = {
    "cfg1": WorkloadConfig("cfg1_er2000", 2000, 8000, "er", 64, 5, 64, (1, 2), 4, 2, 0.5, 0.5,
                           seed=0, avg_degree=8.0),
    "cfg2": WorkloadConfig("cfg2_powerlaw24492", 24492, 186100, "powerlaw", 300, 5, 512, (1, 2, 3),
                           4, 2, 0.5, 0.5, seed=42),
    "cfg4": WorkloadConfig("cfg4_rmat2450000", 2450000, 61900000, "rmat", 100, 47, 512, (1, 2), 4, 1,
                           0.5, 0.5, seed=7),
    # the stress configuration: 10M-node RMAT, average degree 32, features
    # [N, 128] stored as bf16, D = 512 (32 channels x 16 blades), K = 3,
    # 8 heads; one block (its depth is not specified), 47 classes as cfg4
    "cfg5": WorkloadConfig("cfg5_rmat10000000", 10_000_000, 320_000_000, "rmat", 128, 47, 512,
                           (1, 2, 3), 8, 1, 0.5, 0.5, seed=11),
}


def make_edges(cfg: WorkloadConfig, device=None) -> torch.Tensor:
    if cfg.generator == "er":
        return erdos_renyi(cfg.num_nodes, cfg.avg_degree, cfg.seed)
    if cfg.generator == "powerlaw":
        return powerlaw_graph(cfg.num_nodes, cfg.num_edges, 2.5, 1, cfg.seed)
    if cfg.generator == "rmat":
        return rmat_graph(cfg.num_nodes, cfg.num_edges, seed=cfg.seed, device=device)
    raise ValueError(cfg.generator)


def make_features(cfg: WorkloadConfig, seed: Optional[int] = None):
    """x ~ N(0,1) [N, in_dim] fp32, labels uniform over classes, 50/25/25 split."""
    gen = torch.Generator()
    gen.manual_seed(cfg.seed if seed is None else seed)
    x = torch.randn(cfg.num_nodes, cfg.in_dim, generator=gen)
    y = torch.randint(0, cfg.num_classes, (cfg.num_nodes,), generator=gen)
    train, val, test = random_ratio_split(cfg.num_nodes, 0.5, 0.25, 0.25, 42)
    return x, y, train, val, test
