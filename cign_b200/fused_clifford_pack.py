"""Clifford pack, "old" interaction (drop-in for the reference's
fused_clifford_pack, fused_clifford_pack.py:1-244).

``fused_clifford_pack(H_norm, C_norm, propagated, alpha)`` returns
``cat_k alpha_k [W_k, D_k]`` of shape [N, 2KD] with ``T_H, T_C = P_k[:, :D],
P_k[:, D:]``, ``W_k = H*T_C - T_H*C`` and ``D_k = SiLU(H*T_C)``; alpha is
None (all ones), [N,K] or [N,K,1].  Any K runs the same native kernel (the
reference has a K=3 specialisation plus an inline generic-K build); the
``ensure_*`` loaders are kept for callers that preload extensions.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib
from ._pack import PackFunction, run_pack

_EXT = None


def _extension_name() -> str:
    return "cign_sm100_clifford_pack"


def ensure_special_fused_clifford_pack_loaded(verbose: bool = False):
    global _EXT
    if _EXT is None:
        if not torch.cuda.is_available():
            raise RuntimeError("A3 fused Clifford pack requires CUDA.")
        _EXT = _lib.load_library()
    return _EXT


def ensure_generic_fused_clifford_pack_loaded(verbose: bool = False):
    return ensure_special_fused_clifford_pack_loaded(verbose)


def ensure_fused_clifford_pack_loaded(verbose: bool = False, hop_count: int = 3):
    return ensure_special_fused_clifford_pack_loaded(verbose)


FusedCliffordPack3Function = PackFunction
GenericFusedCliffordPackFunction = PackFunction


def fused_clifford_pack(
    H_norm: torch.Tensor,
    C_norm: torch.Tensor,
    propagated: Sequence[torch.Tensor],
    alpha: torch.Tensor | None,
) -> torch.Tensor:
    ensure_special_fused_clifford_pack_loaded()
    return run_pack(H_norm, C_norm, propagated, alpha, interaction=0, outer=0, weighting=0)
