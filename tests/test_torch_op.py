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


def test_plan_cache_entry_matches_only_the_same_unedited_tensors():
    """A cached plan is reused only for the very tensor objects it was built from, at the
    versions it saw: an in-place edit or another tensor (even with equal contents, as a
    new graph at a recycled address would be) does not match."""
    A, crow, col, val = _graph()
    e = torch_op._Entry(plan=None, tensors=(crow, col, val))
    assert e.matches((crow, col, val))
    assert not e.matches((crow, col.clone(), val))
    col[0] = col[0]  # an in-place write bumps the version counter, whatever it writes
    assert not e.matches((crow, col, val))
    e = torch_op._Entry(plan=None, tensors=(crow, col, val))
    val.mul_(1.0)
    assert not e.matches((crow, col, val))


def _permuted_graph(crow, col, val, seed):
    """Same row offsets and shapes, different column indices (and so a different product)."""
    ncol = int(col.max()) + 1
    perm = torch.randperm(ncol, generator=torch.Generator().manual_seed(seed))
    rows = []
    for r in range(crow.shape[0] - 1):
        c = perm[col[crow[r]:crow[r + 1]].long()].sort().values
        rows.append(c)
    return torch.cat(rows).to(col.dtype)


@pytest.mark.gpu
def test_new_graph_at_recycled_addresses_gets_a_new_plan():
    """Free a device graph, allocate a different graph of the same shapes (the caching
    allocator hands back the same addresses), and the op must multiply by the new graph."""
    A, crow, col, val = _graph(scale=9, edges=4000, seed=8)
    X = torch.randn(A.ncol, 16, generator=torch.Generator().manual_seed(4)).cuda()
    torch_op.clear_plan_cache()
    col2_host = _permuted_graph(crow, col, val, seed=9)
    d1 = [t.cuda() for t in (crow, col, val)]
    ptrs = [t.data_ptr() for t in d1]
    Y1 = torch.ops.tcaspmm.spmm(*d1, X)
    del d1
    torch_op.clear_plan_cache()  # nothing holds the first graph any more: its memory is free
    d2 = [t.cuda() for t in (crow, col2_host, val)]
    reused = [t.data_ptr() for t in d2] == ptrs
    Y2 = torch.ops.tcaspmm.spmm(*d2, X)
    ref2 = oracle.spmm_f64(A.row_ptr, col2_host.numpy(), val.numpy(), X.cpu().numpy())
    assert oracle.rel_l2(Y2.cpu().numpy(), ref2) <= 1e-5, f"addresses reused: {reused}"
    assert oracle.rel_l2(Y1.cpu().numpy(), ref2) > 1e-2  # the two graphs differ
    # With the first graph still cached (it holds its tensors), a second graph of the same
    # shapes gets its own plan too.
    d3 = [t.cuda() for t in (crow, col, val)]
    Y3 = torch.ops.tcaspmm.spmm(*d3, X)
    ref1 = oracle.spmm_f64(A.row_ptr, A.col, val.numpy(), X.cpu().numpy())
    assert oracle.rel_l2(Y3.cpu().numpy(), ref1) <= 1e-5
    torch_op.clear_plan_cache()


@pytest.mark.gpu
def test_in_place_edit_of_the_graph_rebuilds_the_plan():
    A, crow, col, val = _graph(scale=9, edges=4000, seed=10)
    X = torch.randn(A.ncol, 16, generator=torch.Generator().manual_seed(5)).cuda()
    torch_op.clear_plan_cache()
    dcrow, dcol, dval = crow.cuda(), col.cuda(), val.cuda()
    Y1 = torch.ops.tcaspmm.spmm(dcrow, dcol, dval, X)
    ref1 = oracle.spmm_f64(A.row_ptr, A.col, val.numpy(), X.cpu().numpy())
    assert oracle.rel_l2(Y1.cpu().numpy(), ref1) <= 1e-5
    col2 = _permuted_graph(crow, col, val, seed=11)
    dcol.copy_(col2.cuda())                     # edit the columns in place
    Y2 = torch.ops.tcaspmm.spmm(dcrow, dcol, dval, X)
    ref2 = oracle.spmm_f64(A.row_ptr, col2.numpy(), val.numpy(), X.cpu().numpy())
    assert oracle.rel_l2(Y2.cpu().numpy(), ref2) <= 1e-5
    dval.mul_(2.0)                              # and the values
    Y3 = torch.ops.tcaspmm.spmm(dcrow, dcol, dval, X)
    assert oracle.rel_l2(Y3.cpu().numpy(), 2.0 * ref2) <= 1e-5
    assert len(torch_op._PLANS) == 1            # each edit replaced the stale plan
    torch_op.clear_plan_cache()


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


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_fused_op_forward_and_backward(out_dtype):
    """relu(s * (A X) + b): forward and dX, db against dense fp64 torch on the CPU."""
    A, crow, col, val = _graph(seed=4)
    g = torch.Generator().manual_seed(2)
    X = torch.randn(A.ncol, 48, generator=g).cuda().requires_grad_(True)
    s = torch.rand(A.nrow, generator=g) + 0.5
    b = torch.randn(48, generator=g).cuda().requires_grad_(True)
    Y = torch.ops.tcaspmm.spmm_fused(crow, col, val, X, s.cuda(), b, True, out_dtype)
    assert Y.dtype == out_dtype
    Ad = torch.from_numpy(A.to_scipy().toarray()).double()
    Xr = X.detach().cpu().double().requires_grad_(True)
    br = b.detach().cpu().double().requires_grad_(True)
    Yr = torch.relu(s.double()[:, None] * (Ad @ Xr) + br)
    tol = 1e-5 if out_dtype == torch.float32 else 2.0 ** -8
    assert oracle.rel_l2(Y.detach().float().cpu().numpy(), Yr.detach().numpy()) <= tol
    G = torch.randn(Y.shape, generator=g)
    (Y.float() * G.cuda()).sum().backward()
    (Yr * G.double()).sum().backward()
    # The ReLU mask comes from the rounded Y, so a bf16 output may flip entries at 0.
    gtol = 1e-5 if out_dtype == torch.float32 else 2e-2
    assert oracle.rel_l2(X.grad.cpu().numpy(), Xr.grad.numpy()) <= gtol
    assert oracle.rel_l2(b.grad.cpu().numpy(), br.grad.numpy()) <= gtol


@pytest.mark.gpu
def test_sage_mean_layer_with_bias():
    A, crow, col, val = _graph(seed=6)
    deg = torch.from_numpy(np.diff(A.row_ptr)).float()
    inv = torch.where(deg > 0, 1.0 / deg.clamp(min=1), torch.zeros_like(deg))
    ones = torch.ones_like(val)
    bias = torch.nn.Parameter(torch.zeros(32, device="cuda"))
    layer = torch_op.GCNAggregate(crow, col, ones, row_scale=inv, bias=bias, relu=False)
    X = torch.randn(A.ncol, 32, device="cuda")
    Y = layer(X)
    mean = oracle.spmm_f64(A.row_ptr, A.col, np.repeat(inv.numpy(), np.diff(A.row_ptr)), X.cpu().numpy())
    assert oracle.rel_l2(Y.detach().cpu().numpy(), mean) <= 1e-5
    Y.sum().backward()
    assert bias.grad is not None and torch.allclose(bias.grad, torch.full_like(bias, A.nrow))


@pytest.mark.gpu
def test_allow_tf32_routes_fp32_through_tf32_windows():
    A = T.gen_uniform(1024, 512, 0.3, 2)
    crow, col, val = torch.from_numpy(A.row_ptr), torch.from_numpy(A.col), torch.from_numpy(A.values())
    X = torch.randn(512, 64, generator=torch.Generator().manual_seed(3)).cuda()
    ref = oracle.spmm_f64(A.row_ptr, A.col, A.values(), X.cpu().numpy())
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        torch_op.clear_plan_cache()
        torch.backends.cuda.matmul.allow_tf32 = False
        Y32 = torch.ops.tcaspmm.spmm(crow, col, val, X)
        torch.backends.cuda.matmul.allow_tf32 = True
        Ytf = torch.ops.tcaspmm.spmm(crow, col, val, X)
        dts = {k[7] for k in torch_op._PLANS}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
        torch_op.clear_plan_cache()
    assert oracle.rel_l2(Y32.cpu().numpy(), ref) <= 1e-5
    assert oracle.rel_l2(Ytf.cpu().numpy(), ref) <= 5e-3
    assert dts == {"f32", "tf32"}
