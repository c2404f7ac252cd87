"""CIGN generic-K pack: "new" interaction, no outer nonlinearity, "old"
weighting (drop-in for the reference's generic_engine/
fused_clifford_cign_generic.py:1-190).

``fused_clifford_pack(H_norm, C_norm, propagated, alpha)`` returns
``cat_k alpha_k [W_k, D_k]`` [N, 2KD] with ``D_k = SiLU((H*T_C + C*T_H)/2)``
and ``W_k = (H*T_C - C*T_H)/2``.  The reference stacks the K propagated
tensors into [N,K,2D] first (:189) and accumulates grad_H/grad_C/grad_alpha
with atomics; here the kernel reads the K tensors in place and the backward
is atomic-free.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib
from ._pack import PackFunction, run_pack

_EXT = None


def ensure_generic_fused_clifford_pack_loaded(verbose: bool = False):
    global _EXT
    if _EXT is None:
        if not torch.cuda.is_available():
            raise RuntimeError("Generic Clifford pack requires CUDA")
        _EXT = _lib.load_library()
    return _EXT


GenericFusedCliffordPackFunction = PackFunction


def fused_clifford_pack(
    H_norm: torch.Tensor,
    C_norm: torch.Tensor,
    propagated: Sequence[torch.Tensor],
    alpha: torch.Tensor | None,
) -> torch.Tensor:
    ensure_generic_fused_clifford_pack_loaded()
    return run_pack(H_norm, C_norm, propagated, alpha, interaction=1, outer=0, weighting=0)
