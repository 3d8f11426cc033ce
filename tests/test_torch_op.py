"""torch.ops.tcaspmm.spmm: the GCN / SAGE aggregation op over the C-ABI path."""
import numpy as np
import pytest
import torch

import oracle
import spmm_b200 as T
from spmm_b200 import torch_op


def _graph(scale=11, edges=20000, kind="gcn", seed=3):
    A = T.gen_rmat(scale, edges, kind=kind, seed=seed)
    return A, torch.from_numpy(A.row_ptr), torch.from_numpy(A.col), torch.from_numpy(A.values())


def test_op_is_registered_and_rejects_cpu_inputs():
    A, crow, col, val = _graph()
    assert hasattr(torch.ops.tcaspmm, "spmm") and hasattr(torch.ops.tcaspmm, "spmm_t")
    with pytest.raises(Exception):
        torch.ops.tcaspmm.spmm(crow, col, val, torch.zeros(A.ncol, 4))


def test_transposed_host_csr_is_the_transpose():
    A, crow, col, val = _graph()
    At = torch_op._host_csr(crow, col, val, A.ncol, transposed=True)
    At.validate()
    np.testing.assert_array_equal(At.to_scipy().toarray(), A.to_scipy().T.toarray())


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
def test_forward_and_backward_match_the_oracle(dt):
    A, crow, col, val = _graph()
    X = torch.randn(A.ncol, 64, generator=torch.Generator().manual_seed(1)).to(dt).cuda().requires_grad_(True)
    Y = torch.ops.tcaspmm.spmm(crow, col, val, X)
    vals = val.to(dt).float().numpy()
    ref = oracle.spmm_f64(A.row_ptr, A.col, vals, X.detach().float().cpu().numpy())
    tol = 1e-5 if dt == torch.float32 else 5e-3
    assert oracle.rel_l2(Y.detach().cpu().numpy(), ref) <= tol
    G = torch.randn_like(Y)
    (Y * G).sum().backward()
    At = torch_op._host_csr(crow, col, val, A.ncol, transposed=True)
    gref = oracle.spmm_f64(At.row_ptr, At.col, torch.from_numpy(At.values()).to(dt).float().numpy(),
                           G.to(dt).float().cpu().numpy())
    assert oracle.rel_l2(X.grad.float().cpu().numpy(), gref) <= (1e-5 if dt == torch.float32 else 1e-2)


@pytest.mark.gpu
def test_gcn_layer_reuses_its_plan():
    A, crow, col, val = _graph()
    torch_op.clear_plan_cache()
    layer = torch_op.GCNAggregate(crow, col, val)
    X = torch.randn(A.ncol, 32, device="cuda")
    y1 = layer(X)
    y2 = layer(X)
    assert len(torch_op._PLANS) == 1
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
