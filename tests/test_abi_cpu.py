"""The C-ABI library loads and exports every symbol include/cign_sm100.h
declares; argument validation rejects bad input before touching the GPU.
CPU only (no compute calls)."""
import ctypes
import re
from pathlib import Path

import pytest

from cign_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "cign_sm100.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^CIGN_API\s+[\w\s\*]+?\b(cign_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers every declared symbol
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_version_and_error_text():
    lib = _lib.load_library()
    assert lib.cign_version() >= 1
    assert lib.cign_kernel_launches() == 0  # nothing launched without a GPU
    out = ctypes.c_void_p()
    rc = lib.cign_spmm_plan_create(None, None, ctypes.byref(out))
    assert rc == 2  # CIGN_ERR_NULL_POINTER
    assert "csr is NULL" in _lib.last_error()


def test_invalid_arguments_rejected_before_launch():
    lib = _lib.load_library()
    # unknown pack modes / hop counts
    assert lib.cign_pack_fwd(4, 8, 0, 1, 0, 0, None, None, None, 16, None, None, None) == 6
    assert lib.cign_pack_fwd(4, 8, 2, 7, 0, 0, None, None, None, 16, None, None, None) == 1
    # dropout probability out of range
    assert lib.cign_dropout_ln_fwd(4, 8, None, None, None, 1.5, 1e-5, 0, None, None, None,
                                   None, None) == 1
    # D above the register-resident limit
    assert lib.cign_add_ln_fwd(4, 4096, None, None, None, None, 1e-5, None, None, None,
                               None) == 6
    # GAT heads above the supported range
    assert lib.cign_gat_fwd(ctypes.c_void_p(1), 65, 8, None, None, None, None, 0.2, 0.0, 0, None,
                            None, None, None, None, None, 0, None) == 6
    assert "heads" in _lib.last_error()
    # pack + proj GEMM: D not a multiple of 32, Dout above the 512 TMEM columns,
    # more hops than the kernel's pointer table
    ws = ctypes.c_void_p(16)
    assert lib.cign_pack_proj_gemm_tf32(128, 48, 2, 64, None, None, None, 96, None, None, None,
                                        None, None, ws, 1 << 20, None) == 6
    assert "multiple of 32" in _lib.last_error()
    assert lib.cign_pack_proj_gemm_tf32(128, 64, 2, 1024, None, None, None, 128, None, None,
                                        None, None, None, ws, 1 << 30, None) == 6
    assert lib.cign_pack_proj_gemm_tf32(128, 64, 9, 64, None, None, None, 128, None, None, None,
                                        None, None, ws, 1 << 30, None) == 6
    assert lib.cign_pack_proj_workspace_bytes(512, 3, 512) >= 512 * 3072 * 4
    # JK LayerNorm: row wider than 2048 floats, too many segments
    assert lib.cign_jk_ln_fwd(4, 3, 1024, None, None, None, 1e-5, None, None, None, None) == 6
    assert lib.cign_jk_ln_fwd(4, 9, 64, None, None, None, 1e-5, None, None, None, None) == 6
    assert lib.cign_jk_ln_workspace_bytes(1000, 1536) == 2 * 16 * 1536 * 4


def test_python_api_requires_cuda_without_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    from cign_b200 import collapsed_gat, fused_block_ops, multihop_csr_pipeline
    with pytest.raises(RuntimeError):
        multihop_csr_pipeline.ensure_multihop_csr_loaded()
    with pytest.raises(RuntimeError):
        collapsed_gat.ensure_collapsed_gat_loaded()
    with pytest.raises(TypeError):
        fused_block_ops.fused_add_layernorm(torch.zeros(2, 4), torch.zeros(2, 4), torch.ones(4),
                                            torch.zeros(4), 1e-5)


def test_python_api_raises_the_reference_exception_types():
    """Bad inputs raise what the reference raises, before any launch:
    multihop_csr_pipeline.py:38-48, 94-101, 171; collapsed_gat.py:184-187;
    fused_gat_sideops.py:96; fused_clifford_pack.py:29;
    fused_block_ops.py:102-104."""
    import torch
    from cign_b200 import collapsed_gat, fused_block_ops, fused_clifford_pack, fused_gat_sideops
    from cign_b200 import multihop_csr_pipeline as mh
    if torch.cuda.is_available():
        pytest.skip("CUDA present: the device checks would pass")
    csr = torch.eye(4).to_sparse_csr()

    class Base:  # a prepared FixedCSRGraphOperator as the reference expects it
        shape, nnz = (4, 4), 4

    Base.csr = Base.csr_t = csr
    with pytest.raises(TypeError):
        mh._csr_parts_int32(torch.eye(4))
    with pytest.raises(RuntimeError):
        mh._csr_parts_int32(csr)
    with pytest.raises(ValueError):
        mh.MultiHopCSR3GraphOperator(Base(), dense_cols=0)
    with pytest.raises(ValueError):
        mh.MultiHopCSR3GraphOperator(Base(), dense_cols=8, algorithm=5)
    with pytest.raises(TypeError):
        mh.MultiHopCSR3GraphOperator(object(), dense_cols=8)
    with pytest.raises(ValueError):
        mh.prepare_multihop_csr_operator(Base(), 8, powers=())
    x = torch.zeros(4, 2, 3)
    with pytest.raises(TypeError):
        collapsed_gat.collapsed_gat_mean_bias_silu(torch.zeros(4, 2), torch.zeros(4, 2), None,
                                                   None, None, 0.2, x, torch.zeros(3), 0.0)
    with pytest.raises(TypeError):
        fused_gat_sideops.fused_attention_logits(x, torch.zeros(1, 2, 3), torch.zeros(1, 2, 3))
    with pytest.raises(RuntimeError):
        fused_clifford_pack.fused_clifford_pack(torch.zeros(4, 8), torch.zeros(4, 8),
                                                [torch.zeros(4, 16)] * 3, None)
    with pytest.raises(TypeError):
        fused_block_ops.fused_dropout_layernorm(torch.zeros(4, 8), torch.ones(8), torch.zeros(8),
                                                0.1, 1e-5)
