"""Counter-based dropout streams of the reference, restated in numpy uint64.

TEST INFRASTRUCTURE (see oracle/__init__.py).

* splitmix64 finaliser: collapsed_gat_ext/collapsed_gat_cuda.cu:27-32 and
  fused_block_ops.py:15 (identical constants).
* GAT attention mask: collapsed_gat_cuda.cu:34-47 -- keep[idx] =
  ((r >> 32) + 0.5f) * 2^-32 > p  (float arithmetic), idx = e*H + h.
* Block-op mask: fused_block_ops.py:15 dropout_keep -- keep =
  (r >> 11) * 2^-53 >= p  (double arithmetic), idx = n*D + d; p <= 0 keeps all.
* Seeds: collapsed_gat.py:204-211 and fused_block_ops.py:46-50.
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
IDX_MUL = np.uint64(0xD2B74407B1CE6E93)
MASK63 = (1 << 63) - 1


def splitmix64(x) -> np.ndarray:
    """The splitmix64 finaliser (collapsed_gat_cuda.cu:27-32), elementwise on uint64."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + GOLDEN
        x = (x ^ (x >> np.uint64(30))) * M1
        x = (x ^ (x >> np.uint64(27))) * M2
        return x ^ (x >> np.uint64(31))


def _hash(seed: int, count: int) -> np.ndarray:
    idx = np.arange(int(count), dtype=np.uint64)
    with np.errstate(over="ignore"):
        return splitmix64(np.uint64(int(seed) & ((1 << 64) - 1)) ^ (idx * IDX_MUL))


def gat_keep_mask(seed: int, count: int, p: float) -> np.ndarray:
    """bool [count]: the attention keep-mask (collapsed_gat_cuda.cu:34-47);
    p <= 0 keeps everything."""
    if float(p) <= 0.0:
        return np.ones(int(count), dtype=bool)
    hi = (_hash(seed, count) >> np.uint64(32)).astype(np.uint32)
    u = (hi.astype(np.float32) + np.float32(0.5)) * np.float32(2.3283064365386963e-10)
    return u > np.float32(p)


def block_keep_mask(seed: int, count: int, p: float) -> np.ndarray:
    """bool [count]: the block-op keep-mask (dropout_keep of
    fused_block_ops.py:15)."""
    if float(p) <= 0.0:
        return np.ones(int(count), dtype=bool)
    r = _hash(seed, count) >> np.uint64(11)
    u = r.astype(np.float64) * (1.0 / 9007199254740992.0)
    return u >= np.float64(np.float32(p))


def gat_seed(initial_seed: int, call_id: int) -> int:
    """Seed of GAT call number call_id (0-based) (collapsed_gat.py:204-211)."""
    base = int(initial_seed) & MASK63
    return (base + 0x9E3779B97F4A7C15 * (call_id + 1)) & MASK63


def block_seed(initial_seed: int, call: int, tag: int) -> int:
    """Seed of block-op call number `call` (1-based) with tag 1 (dropout-LN) or
    2 (gamma residual) (fused_block_ops.py:46-50)."""
    base = int(initial_seed) & MASK63
    return (base + 0x9E3779B97F4A7C15 * call + 0xD2B74407B1CE6E93 * int(tag)) & MASK63
