"""Full CIGN model (the caller of every hot-path op) on the GPU against the
reference model's own outputs and parameter gradients (golden, produced by
generic_engine/model_cign.py with every fused switch off), at the
reference's thresholds (validate_cign_acceleration.py:53-57)."""
import pytest
import torch

from cign_b200.graph_operator import prepare_fixed_csr_operator, to_graph_format
from cign_b200.model_cign import build_model
from cign_b200.multihop_csr_pipeline import prepare_multihop_csr_operator

pytestmark = pytest.mark.gpu


def test_model_matches_reference(cuda, golden):
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
            op = prepare_multihop_csr_operator(base, dense_cols=48, powers=hops)
            edge = torch.from_numpy(z[f"{tag}_edge"])
            (rp, c), (r, cp), perm = to_graph_format(edge.flip(0), n)
            model = build_model(in_dim=8, hidden_dim=24, out_dim=3, num_layers=2, dropout=0.0,
                                gat_dropout=0.0, gat_heads=2, hop_scales=hops).to(cuda)
            state = {k[len(tag) + 3:]: torch.from_numpy(z[k]) for k in z.keys()
                     if k.startswith(f"{tag}_p_")}
            model.load_state_dict(state, strict=True)
            model.prepare_fused_gat_graph(((rp.to(cuda), c.to(cuda)), (r.to(cuda), cp.to(cuda)),
                                           perm.to(cuda)))
            y = model(torch.from_numpy(z[f"{tag}_x"]).to(cuda), op)
            torch.testing.assert_close(y.cpu(), torch.from_numpy(z[f"{tag}_y"]), rtol=2e-4,
                                       atol=2e-5, msg=str(case))
            (y * torch.from_numpy(z[f"{tag}_go"]).to(cuda)).sum().backward()
            for name, p in model.named_parameters():
                key = f"{tag}_gp_{name}"
                if key in z:
                    torch.testing.assert_close(p.grad.cpu(), torch.from_numpy(z[key]), rtol=5e-4,
                                               atol=5e-5, msg=f"{case} {name}")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
