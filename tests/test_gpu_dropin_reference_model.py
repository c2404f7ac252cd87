"""The drop-in boundary, end to end: the REFERENCE's own CIGN model
(generic_engine/model_cign.py, unchanged) running on this repository's op
modules.

The reference module is byte-compiled from its source by oracle/build_ref.py
into oracle/_ref/py/model_cign.bytecode (git-ignored; it travels with the working
tree to the GPU box, the reference tree does not).  Its imports
(model_cign.py:27-44) are satisfied exactly as a user switching to this
library would satisfy them:

  * the op modules it imports by name -- multihop_csr_pipeline, collapsed_gat,
    fused_gat_sideops, fused_block_ops, fused_clifford_pack,
    fused_clifford_switch_pack, fused_clifford_cign_pack,
    fused_clifford_cign_generic -- are the cign_b200 modules, aliased in
    sys.modules;
  * torch_geometric (absent here) is the test stub of tests/golden/make_golden.py,
    with to_graph_format bound to this library's CSR/CSC/perm builder;
  * chunked_dgnn_gat (the dgNN work-around, out of scope) is an inert stub.

GraphCliffordNet is then built with every fused switch on (collapsed GAT,
side ops, Clifford pack, block ops) in the production modes and compared with
tests/golden/model_cases.npz (the same model run by the reference on the CPU
with every fused switch off) at the reference's thresholds
(validate_cign_acceleration.py:53-57).
"""
import importlib.machinery
import importlib.util
import sys
import types
from pathlib import Path

import pytest
import torch

import cign_b200
from cign_b200 import (collapsed_gat, fused_block_ops, fused_clifford_cign_generic,
                       fused_clifford_cign_pack, fused_clifford_pack, fused_clifford_switch_pack,
                       fused_gat_sideops, multihop_csr_pipeline)
from cign_b200.graph_operator import prepare_fixed_csr_operator, to_graph_format
from tests.golden.make_golden import _StubGATConv

pytestmark = pytest.mark.gpu

ROOT = Path(cign_b200.__file__).resolve().parents[1]
REF_PYC = ROOT / "oracle" / "_ref" / "py" / "model_cign.bytecode"

ALIASES = {
    "multihop_csr_pipeline": multihop_csr_pipeline,
    "collapsed_gat": collapsed_gat,
    "fused_gat_sideops": fused_gat_sideops,
    "fused_block_ops": fused_block_ops,
    "fused_clifford_pack": fused_clifford_pack,
    "fused_clifford_switch_pack": fused_clifford_switch_pack,
    "fused_clifford_cign_pack": fused_clifford_cign_pack,
    "fused_clifford_cign_generic": fused_clifford_cign_generic,
}


class _StubFusedGATConv(_StubGATConv):
    """PyG FusedGATConv stand-in: GATConv's parameters plus to_graph_format."""

    @staticmethod
    def to_graph_format(edge_index, size=None):
        n = int(size[0]) if size is not None else int(edge_index.max()) + 1
        return to_graph_format(edge_index, n)


def _install(monkeypatch):
    tg = types.ModuleType("torch_geometric")
    tgnn = types.ModuleType("torch_geometric.nn")
    tgnn.GATConv = _StubGATConv
    tgnn.FusedGATConv = _StubFusedGATConv
    tg.nn = tgnn
    chunked = types.ModuleType("chunked_dgnn_gat")

    class ChunkedDgNNGraph:  # never instantiated on the collapsed path
        pass

    def _unused(*args, **kwargs):
        raise RuntimeError("chunked dgNN path is out of scope")

    chunked.ChunkedDgNNGraph = ChunkedDgNNGraph
    chunked.prepare_chunked_dgnn_graph = _unused
    chunked.run_chunked_dgnn_op = _unused
    for name, mod in {"torch_geometric": tg, "torch_geometric.nn": tgnn,
                      "chunked_dgnn_gat": chunked, **ALIASES}.items():
        monkeypatch.setitem(sys.modules, name, mod)
    for key, val in (("CIGN_ALPHA_SCORE_MODE", "new"), ("CIGN_INTERACTION_MODE", "new"),
                     ("CIGN_ALPHA_WEIGHTING_MODE", "old"), ("CIGN_OUTER_NONLINEARITY", "none")):
        monkeypatch.setenv(key, val)
    loader = importlib.machinery.SourcelessFileLoader("reference_model_cign", str(REF_PYC))
    spec = importlib.util.spec_from_loader("reference_model_cign", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


@pytest.fixture
def ref_model_cign(monkeypatch):
    if not REF_PYC.exists():
        pytest.skip("the reference model is not built (oracle/build_ref.py needs the reference tree)")
    return _install(monkeypatch)


def test_reference_model_on_these_modules(cuda, golden, ref_model_cign):
    z = golden("model_cases.npz")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for case in z["cases"]:
            tag, gname, hops = str(case).split("|")
            hops = [int(h) for h in hops.split(",")]
            n = int(z[f"{tag}_n"])
            op_coo = torch.sparse_coo_tensor(torch.from_numpy(z[f"{tag}_op_idx"]),
                                             torch.from_numpy(z[f"{tag}_op_val"]), (n, n)).to(cuda)
            base = prepare_fixed_csr_operator(op_coo)
            op = multihop_csr_pipeline.prepare_multihop_csr_operator(base, dense_cols=48,
                                                                     powers=hops)
            model = ref_model_cign.build_model(
                in_dim=8, hidden_dim=24, out_dim=3, num_layers=2, dropout=0.0, gat_dropout=0.0,
                gat_heads=2, hop_scales=hops, use_fused_gat=True, use_fused_gat_sideops=True,
                use_collapsed_fused_gat=True, use_fused_clifford_pack=True,
                use_fused_block_ops=True).to(cuda)
            assert isinstance(model.blocks[0].context_gat,
                              ref_model_cign.CompatibleCollapsedFusedGATConv)
            state = {k[len(tag) + 3:]: torch.from_numpy(z[k]) for k in z.keys()
                     if k.startswith(f"{tag}_p_")}
            model.load_state_dict(state, strict=True)
            edge = torch.from_numpy(z[f"{tag}_edge"]).to(cuda)
            model.prepare_fused_gat_graph(edge, n)
            y = model(torch.from_numpy(z[f"{tag}_x"]).to(cuda), edge, op)
            torch.testing.assert_close(y.cpu(), torch.from_numpy(z[f"{tag}_y"]), rtol=2e-4,
                                       atol=2e-5, msg=str(case))
            (y * torch.from_numpy(z[f"{tag}_go"]).to(cuda)).sum().backward()
            checked = 0
            for name, p in model.named_parameters():
                key = f"{tag}_gp_{name}"
                if key in z:
                    torch.testing.assert_close(p.grad.cpu(), torch.from_numpy(z[key]), rtol=5e-4,
                                               atol=5e-5, msg=f"{case} {name}")
                    checked += 1
            assert checked >= 20, (case, checked)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
