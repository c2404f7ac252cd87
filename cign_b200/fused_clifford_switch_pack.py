"""CIGN switch pack, K=3 (drop-in for the reference's
generic_engine/fused_clifford_switch_pack.py:1-183).

``fused_clifford_switch_pack(H_norm, C_norm, propagated, alpha,
interaction_mode, alpha_weighting_mode)`` with modes "old"/"new":

* interaction "old": D = SiLU(B_HR), W = B_HR - B_RH;
  "new": D = SiLU((B_HR + B_RH)/2), W = tanh((B_HR - B_RH)/2);
  B_HR = H*T_C, B_RH = C*T_H.
* weighting "old": cat_k alpha_k [W_k, D_k] -> [N, 6D];
  "new": [sum_k alpha_k D_k, sum_k alpha_k W_k] -> [N, 2D].

Exactly three hops, as in the reference (ValueError otherwise).
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib
from ._pack import PackFunction, run_pack

_EXT = None
OUTER = 1  # tanh on the antisymmetric part of the "new" interaction


def _extension_name() -> str:
    return "cign_sm100_switch_pack"


def ensure_fused_clifford_switch_pack_loaded(verbose: bool = False):
    global _EXT
    if _EXT is None:
        if not torch.cuda.is_available():
            raise RuntimeError("CIGN switch fused Clifford pack requires CUDA.")
        _EXT = _lib.load_library()
    return _EXT


def _mode_to_int(name: str, kind: str) -> int:
    value = str(name).strip().lower()
    if value == "old":
        return 0
    if value == "new":
        return 1
    raise ValueError(f"{kind} must be old/new, got {name!r}")


FusedCliffordSwitchPackFunction = PackFunction


def fused_clifford_switch_pack(
    H_norm: torch.Tensor,
    C_norm: torch.Tensor,
    propagated: Sequence[torch.Tensor],
    alpha: torch.Tensor | None,
    interaction_mode: str,
    alpha_weighting_mode: str,
) -> torch.Tensor:
    if len(propagated) != 3:
        raise ValueError(
            "CIGN switch fused pack v1 is specialized for exactly 3 hops; "
            f"got {len(propagated)}."
        )
    if H_norm.dim() != 2 or C_norm.shape != H_norm.shape:
        raise ValueError("H_norm/C_norm must both be [N,D]")
    interaction = _mode_to_int(interaction_mode, "interaction_mode")
    weighting = _mode_to_int(alpha_weighting_mode, "alpha_weighting_mode")
    ensure_fused_clifford_switch_pack_loaded()
    return run_pack(H_norm, C_norm, propagated, alpha, interaction=interaction, outer=OUTER,
                    weighting=weighting)
