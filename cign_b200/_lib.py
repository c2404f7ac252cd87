"""ctypes binding of libcign_sm100.so (declared in include/cign_sm100.h).

The library is built in-tree by ``python -m cign_b200.build`` (or
``__graft_entry__.build()``).  There is no CPU fallback: every op of this
package calls into this library and raises if it cannot be loaded.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libcign_sm100.so"

CIGN_OK = 0
ERR_NAMES = {
    1: "invalid argument",
    2: "null pointer",
    3: "alignment",
    4: "kernel launch failed",
    5: "device wait timed out",
    6: "unsupported shape",
    7: "CUDA runtime error",
}

_LOCK = threading.Lock()
_LIB = None
_LOAD_ERROR = None


class CsrF32(ctypes.Structure):
    """Mirror of ``cign_csr_f32``."""

    _fields_ = [
        ("rows", c_int64),
        ("cols", c_int64),
        ("nnz", c_int64),
        ("crow", c_void_p),
        ("col", c_void_p),
        ("val", c_void_p),
    ]


class SpmmPlanInfo(ctypes.Structure):
    """Mirror of ``cign_spmm_plan_info``."""

    _fields_ = [
        ("rows", c_int64),
        ("nnz", c_int64),
        ("heavy_rows", c_int64),
        ("heavy_rows_t", c_int64),
        ("segments", c_int64),
        ("segments_t", c_int64),
        ("max_degree", c_int32),
        ("max_degree_t", c_int32),
        ("segment_length", c_int32),
        ("transpose_is_forward", c_int32),
    ]


_P = c_void_p  # any device pointer / opaque handle
_PP = POINTER(c_void_p)  # host array of device pointers

# name -> (restype, argtypes)
SIGNATURES = {
    "cign_version": (c_int, []),
    "cign_last_error": (c_char_p, []),
    "cign_kernel_launches": (c_uint64, []),
    "cign_spmm_plan_create": (c_int, [POINTER(CsrF32), POINTER(CsrF32), POINTER(c_void_p)]),
    "cign_spmm_plan_destroy": (c_int, [_P]),
    "cign_spmm_plan_get_info": (c_int, [_P, POINTER(SpmmPlanInfo)]),
    "cign_spmm_workspace_bytes": (c_size_t, [_P, c_int64]),
    "cign_spmm": (c_int, [_P, c_int, _P, c_int64, _P, _P, _P, c_size_t, _P]),
    "cign_multihop_workspace_bytes": (c_size_t, [_P, c_int, c_int64]),
    "cign_multihop_fwd": (c_int, [_P, c_int, _P, c_int64, _PP, _P, c_size_t, _P]),
    "cign_multihop_fwd_split": (c_int, [_P, c_int, _P, _P, c_int64, _PP, _P, c_size_t, _P]),
    "cign_multihop_bwd": (c_int, [_P, c_int, _PP, c_int64, _P, _P, c_size_t, _P]),
    "cign_spmm_bf16": (c_int, [_P, c_int, _P, c_int64, _P, c_int, _P, c_size_t, _P]),
    "cign_multihop_fwd_bf16": (c_int, [_P, c_int, _P, c_int64, _PP, _P, c_size_t, _P]),
    "cign_gat_agg_fwd_bf16": (c_int, [_P, c_int32, c_int64, _P, _P, _P, c_float, c_float, c_uint64,
                                      _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_plan_create": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, POINTER(c_void_p)]),
    "cign_gat_plan_create_rect": (c_int, [c_int64, c_int64, c_int64, _P, _P, _P, _P, _P,
                                          POINTER(c_void_p)]),
    "cign_gat_plan_destroy": (c_int, [_P]),
    "cign_gat_plan_get_info": (c_int, [_P, POINTER(c_int64)]),
    "cign_gat_fwd_workspace_bytes": (c_size_t, [_P, c_int32, c_int32]),
    "cign_gat_fwd": (c_int, [_P, c_int32, c_int32, _P, _P, _P, _P, c_float, c_float, c_uint64, _P,
                             _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_bwd_workspace_bytes": (c_size_t, [_P, c_int32, c_int32]),
    "cign_gat_bwd": (c_int, [_P, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P, c_float, c_float,
                             c_uint64, _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_dropout_mask": (c_int, [c_int64, c_int32, c_float, c_uint64, _P, _P, _P]),
    "cign_device_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "cign_device_free": (c_int, [_P]),
    "cign_ipc_handle": (c_int, [_P, _P]),
    "cign_ipc_open": (c_int, [_P, POINTER(c_void_p)]),
    "cign_ipc_close": (c_int, [_P]),
    "cign_silu_mix_fwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P]),
    "cign_silu_mix_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_silu_mix_bwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_halo_push": (c_int, [c_int32, _P, c_int64, _P, _P, _P, c_int64, _P, _P]),
    "cign_halo_push_copy": (c_int, [c_int32, _P, c_int64, _P, _P, _P, c_int64, _P, c_int32,
                                    _P]),
    "cign_colsum_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_colsum_f32": (c_int, [c_int64, c_int64, _P, _P, _P, c_size_t, _P]),
    "cign_seed_table_step": (c_int, [c_uint64, c_int32, _P, _P, c_int32, c_int32, _P, _P]),
    "cign_hop_gate_fwd": (c_int, [c_int64, c_int64, c_int32, c_int32, _P, _P, _P, _P, _P, _P]),
    "cign_hop_gate_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int32]),
    "cign_hop_gate_bwd": (c_int, [c_int64, c_int64, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P,
                                  _P, _P, c_int32, _P, _P, c_int64, _P, c_size_t, _P]),
    "cign_gat_agg_workspace_bytes": (c_size_t, [_P, c_int32, c_int64, c_int64]),
    "cign_gat_agg_fwd": (c_int, [_P, c_int32, c_int64, _P, _P, _P, c_float, c_float, c_uint64, _P,
                                 _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_agg_bwd": (c_int, [_P, c_int32, c_int64, c_int64, _P, _P, _P, _P, _P, _P, _P,
                                 c_float, c_float, c_uint64, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_agg_fwd_w": (c_int, [_P, c_int32, c_int64, _P, _P, _P, c_float, c_float, c_uint64,
                                   _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_gat_agg_bwd_w": (c_int, [_P, c_int32, c_int64, c_int64, _P, _P, _P, _P, _P, _P, _P,
                                   _P, c_float, c_float, c_uint64, _P, _P, _P, _P, _P, c_size_t,
                                   _P]),
    "cign_attn_logits_fwd": (c_int, [c_int64, c_int32, c_int32, _P, _P, _P, _P, _P, _P]),
    "cign_attn_logits_bwd_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32]),
    "cign_attn_logits_bwd": (c_int, [c_int64, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P, _P,
                                     c_int32, _P, c_size_t, _P]),
    "cign_row_dots_fwd": (c_int, [c_int64, c_int64, c_int32, _P, _P, _P, _P]),
    "cign_row_dots_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int32]),
    "cign_row_dots_bwd": (c_int, [c_int64, c_int64, c_int32, _P, _P, _P, _P, c_int32, _P, _P,
                                  c_size_t, _P]),
    "cign_head_mean_bias_silu_fwd": (c_int, [c_int64, c_int32, c_int32, _P, _P, _P, _P, _P]),
    "cign_head_mean_bias_silu_bwd_workspace_bytes": (c_size_t, [c_int64, c_int32]),
    "cign_head_mean_bias_silu_bwd": (c_int, [c_int64, c_int32, c_int32, _P, _P, _P, _P, _P,
                                             c_size_t, _P]),
    "cign_pack_fwd": (c_int, [c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, _P, _P, _PP,
                              c_int64, _P, _P, _P]),
    "cign_jk_ln_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_jk_ln_fwd": (c_int, [c_int64, c_int32, c_int64, _PP, _P, _P, c_float, _P, _P, _P, _P]),
    "cign_jk_ln_bwd": (c_int, [c_int64, c_int32, c_int64, _P, _PP, _P, _P, _P, _PP, _P, _P, _P,
                               c_size_t, _P]),
    "cign_pack_proj_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int64]),
    "cign_pack_proj_gemm_tf32": (c_int, [c_int64, c_int64, c_int32, c_int64, _P, _P, _PP, c_int64,
                                         _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_pack_proj_status": (c_int, [_P, c_int64, c_int32, c_int64, _P]),
    "cign_gate_pack_fwd": (c_int, [c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                                   _P, _P, _PP, c_int64, _P, _P, _P, _P, _P]),
    "cign_pack_bwd": (c_int, [c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, _P, _P, _P,
                              _PP, c_int64, _P, _P, _P, _PP, c_int64, c_int32, _P, _P]),
    "cign_dropout_ln_fwd": (c_int, [c_int64, c_int64, _P, _P, _P, c_float, c_float, c_uint64, _P,
                                    _P, _P, _P, _P]),
    "cign_ln_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_dropout_ln_bwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, c_float, c_uint64, _P, _P,
                                    _P, _P, _P, c_size_t, _P]),
    "cign_dropout_ln_bwd_add": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, c_float, c_uint64,
                                        _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "cign_dropout_ln_bwd_static": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, c_float, c_uint64,
                                           _P, _P, _P, _P]),
    "cign_silu_add_ln_fwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, c_float, _P, _P, _P, _P,
                                     _P]),
    "cign_silu_add_ln_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_silu_add_ln_bwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, _P, c_int32, _P, _P,
                                     _P, _P, _P, _P, c_size_t, _P]),
    "cign_add_ln_fwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, c_float, _P, _P, _P, _P]),
    "cign_add_ln_bwd": (c_int, [c_int64, c_int64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                c_size_t, _P]),
    "cign_gamma_residual_fwd": (c_int, [c_int64, c_int64, _P, _P, _P, c_float, c_uint64, _P, _P, _P]),
    "cign_gamma_residual_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "cign_gamma_residual_bwd": (c_int, [c_int64, c_int64, _P, _P, _P, c_float, c_uint64, _P, _P, _P,
                                        _P, c_size_t, _P]),
    "cign_block_dropout_mask": (c_int, [c_int64, c_float, c_uint64, _P, _P, _P]),
}


def load_library(path: Path | str | None = None):
    """Load (once) and return the ctypes handle; raises if the .so is absent."""
    global _LIB, _LOAD_ERROR
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if _LOAD_ERROR is not None:
            raise RuntimeError("libcign_sm100.so previously failed to load") from _LOAD_ERROR
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            err = FileNotFoundError(
                f"{p} not found; build it with `python -m cign_b200.build` "
                "(there is no CPU fallback)"
            )
            _LOAD_ERROR = err
            raise err
        try:
            handle = ctypes.CDLL(str(p))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
        except Exception as exc:  # pragma: no cover - depends on the box
            _LOAD_ERROR = exc
            raise
        _LIB = handle
        return _LIB


def last_error() -> str:
    msg = load_library().cign_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(rc: int, what: str) -> None:
    if rc != CIGN_OK:
        kind = ERR_NAMES.get(rc, f"error {rc}")
        raise RuntimeError(f"{what} failed ({kind}): {last_error()}")


def require_cuda(what: str) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(f"{what} requires CUDA.")


def seed_args(seed) -> tuple:
    """(value, device pointer) of a dropout seed for the ABI's
    `uint64_t seed, const uint64_t* seed_ptr` pair: a Python int is passed by
    value; a one-element int64 CUDA tensor (a slot of a device seed table) is
    passed by address and read by the kernel when it runs."""
    if isinstance(seed, torch.Tensor):
        return 0, c_void_p(seed.data_ptr())
    return int(seed) & ((1 << 64) - 1), None


def ptr(t: torch.Tensor | None) -> c_void_p:
    return c_void_p(0 if t is None else t.data_ptr())


def ptr_array(ts) -> "ctypes.Array":
    arr = (c_void_p * len(ts))()
    for i, t in enumerate(ts):
        arr[i] = 0 if t is None else t.data_ptr()
    return arr


def stream_of(t: torch.Tensor) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def stream_on(device) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(torch.device(device)).cuda_stream)


def workspace(nbytes: int, device) -> torch.Tensor:
    """Caller-owned scratch (16-byte aligned by the caching allocator)."""
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


class DeviceGuard:
    """Makes `device` current for the duration of a call (no-op if it is)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = torch.device(device).index
        self.prev = None

    def __enter__(self):
        if self.idx is not None:
            cur = torch.cuda.current_device()
            if cur != self.idx:
                self.prev = cur
                torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False
