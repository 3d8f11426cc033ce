"""Property test of the whole GPU path: random CSR matrices (empty rows, hub rows,
dense row blocks that become tensor-core windows, K below a tile), random widths,
dtypes and tuning variables -- gathered windows on or off, tile chains cut into
parts or not, TMA gather4 or cp.async producers, the two kernels side by side or
one after the other.  Values are small integers (A in [-3, 3], B in [-4, 4]), so
every product and partial sum is exact in every input type and in fp32
accumulation: the result must equal the fp64 oracle bit for bit.

Examples are derandomized so every run checks the same cases."""
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle
import spmm_b200 as T
from test_host_properties import _env, csr_cases

pytestmark = pytest.mark.gpu

_TORCH = {"f32": torch.float32, "tf32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@settings(max_examples=400, deadline=None, derandomize=True)
@given(A=csr_cases(),
       N=st.sampled_from([1, 8, 16, 24, 64, 128, 136, 256]),
       dt=st.sampled_from(["f32", "f16", "bf16", "tf32"]),
       seed=st.integers(0, 2**31 - 1),
       env=st.fixed_dictionaries({
           "TCASPMM_HUB_WINDOWS": st.sampled_from([0, 1]),
           "TCASPMM_TC_DENSITY": st.sampled_from([8, 32, 1024]),
           "TCASPMM_WINDOW_PARTS": st.sampled_from([0, 1, 3]),
           "TCASPMM_SPLIT_TILES": st.sampled_from([3, 128]),
           "TCASPMM_GATHER_TMA": st.sampled_from([0, 1]),
           "TCASPMM_OVERLAP": st.sampled_from([0, 1]),
       }))
def test_integer_products_are_exact_on_every_path(A, N, dt, seed, env):
    rng = np.random.default_rng(seed)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, rng.integers(-3, 4, A.nnz).astype(np.float32))
    B = rng.integers(-4, 5, (A.ncol, N)).astype(np.float32)
    Bd = torch.from_numpy(B).to(_TORCH[dt]).cuda()
    Cd = torch.full((A.nrow, N), float("nan"), dtype=torch.float32, device="cuda")
    with _env(env):
        with T.Plan(A, N, dt) as p:
            p.execute1(Bd, Cd, stream=torch.cuda.current_stream())
            p.sync_check()
            st_ = p.stats
    torch.cuda.synchronize()
    ref = oracle.spmm_f64(A.row_ptr, A.col, A.values().astype(np.float64), B.astype(np.float64))
    np.testing.assert_array_equal(Cd.cpu().numpy(), ref.astype(np.float32), err_msg=str((env, st_)))


@settings(max_examples=150, deadline=None, derandomize=True)
@given(A=csr_cases(),
       N=st.sampled_from([8, 16, 24, 64, 136, 256]),
       dt=st.sampled_from(["f32", "f16", "tf32"]),
       seed=st.integers(0, 2**31 - 1),
       layout=st.sampled_from([("columns", 2, None), ("columns", 3, None), ("rows", 2, None), ("rows", 3, None),
                               ("2d", 4, (2, 2)), ("2d", 2, (1, 2)), ("2d", 2, (2, 1))]))
def test_shards_on_one_device_reassemble_the_exact_product(A, N, dt, seed, layout):
    """Column, row and 2-D plans of 2-4 shards placed on cuda:0: every shard writes its
    block of C (row block x column block) and together they give the oracle's product
    bit for bit (integer values)."""
    split, g, grid = layout
    rng = np.random.default_rng(seed)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, rng.integers(-3, 4, A.nnz).astype(np.float32))
    B = rng.integers(-4, 5, (A.ncol, N)).astype(np.float32)
    Bd = torch.from_numpy(B).to(_TORCH[dt]).cuda()
    Cd = torch.full((A.nrow, N), float("nan"), dtype=torch.float32, device="cuda")
    with T.Plan(A, N, dt, num_gpus=g, devices=[0] * g, split=split, grid=grid) as p:
        blocks = []
        for s in range(g):
            r0, rc = p.shard_rows(s) if split != "columns" else (0, A.nrow)
            c0, cc = p.shard(s)[1:] if split != "rows" else (0, N)
            blocks.append((r0, rc, c0, cc))
        p.execute([Bd[:, c0:c0 + cc] for _, _, c0, cc in blocks],
                  [Cd[r0:r0 + rc, c0:c0 + cc] for r0, rc, c0, cc in blocks])
        p.sync_check()
    torch.cuda.synchronize()
    ref = oracle.spmm_f64(A.row_ptr, A.col, A.values().astype(np.float64), B.astype(np.float64))
    np.testing.assert_array_equal(Cd.cpu().numpy(), ref.astype(np.float32), err_msg=str((layout, blocks)))


@settings(max_examples=80, deadline=None, derandomize=True)
@given(A=csr_cases(),
       N=st.sampled_from([1, 8, 16, 64, 128]),
       dt=st.sampled_from([torch.float32, torch.float16, torch.bfloat16]),
       seed=st.integers(0, 2**31 - 1))
def test_torch_op_forward_and_backward_are_exact(A, N, dt, seed):
    """torch.ops.tcaspmm.spmm on random graphs with integer values: Y = A X (fp32) and,
    through autograd, dX = A^T dY (returned in X's dtype), both equal to the fp64
    oracle bit for bit after that one rounding (the op's plan cache sees a new graph
    every example)."""
    from spmm_b200 import torch_op  # registers the op

    rng = np.random.default_rng(seed)
    val = rng.integers(-3, 4, A.nnz).astype(np.float32)
    crow, col, vt = torch.from_numpy(A.row_ptr), torch.from_numpy(A.col), torch.from_numpy(val)
    X = torch.from_numpy(rng.integers(-4, 5, (A.ncol, N)).astype(np.float32)).to(dt).cuda().requires_grad_(True)
    Y = torch.ops.tcaspmm.spmm(crow, col, vt, X)
    ref = oracle.spmm_f64(A.row_ptr, A.col, val.astype(np.float64), X.detach().double().cpu().numpy())
    np.testing.assert_array_equal(Y.detach().float().cpu().numpy(), ref.astype(np.float32))
    G = torch.from_numpy(rng.integers(-2, 3, (A.nrow, N)).astype(np.float32)).cuda().to(Y.dtype)
    (Y * G).sum().backward()
    At = torch_op._host_csr(crow, col, vt, A.ncol, transposed=True)
    gref = oracle.spmm_f64(At.row_ptr, At.col, At.values().astype(np.float64), G.double().cpu().numpy())
    gref = torch.from_numpy(gref.astype(np.float32)).to(dt).float().numpy()
    np.testing.assert_array_equal(X.grad.float().cpu().numpy(), gref)


_OUT_T = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@settings(max_examples=120, deadline=None, derandomize=True)
@given(A=csr_cases(),
       N=st.sampled_from([8, 16, 64, 128, 136]),
       dt=st.sampled_from(["f32", "f16", "bf16", "tf32"]),
       out=st.sampled_from(["f32", "f16", "bf16"]),
       terms=st.fixed_dictionaries({"scale": st.booleans(), "bias": st.booleans(), "relu": st.booleans()}),
       seed=st.integers(0, 2**31 - 1))
def test_fused_epilogue_is_exact_up_to_the_output_rounding(A, N, dt, out, terms, seed):
    """relu?(row_scale * (A B) + bias) in one launch, on every kernel path: with integer
    values, power-of-two row scales and an integer bias every step is exact in fp32,
    so C equals the fp64 oracle rounded once to the output type."""
    rng = np.random.default_rng(seed)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, rng.integers(-3, 4, A.nnz).astype(np.float32))
    B = rng.integers(-4, 5, (A.ncol, N)).astype(np.float32)
    scale = (2.0 ** rng.integers(-2, 2, A.nrow)).astype(np.float32) if terms["scale"] else None
    bias = rng.integers(-3, 4, N).astype(np.float32) if terms["bias"] else None
    Bd = torch.from_numpy(B).to(_TORCH[dt]).cuda()
    Cd = torch.full((A.nrow, N), float("nan"), dtype=_OUT_T[out], device="cuda")
    ep = T.Epilogue(torch.from_numpy(scale).cuda() if scale is not None else None,
                    torch.from_numpy(bias).cuda() if bias is not None else None, terms["relu"], out)
    with T.Plan(A, N, dt) as p:
        p.execute1(Bd, Cd, stream=torch.cuda.current_stream(), epilogue=ep)
        p.sync_check()
    torch.cuda.synchronize()
    ref = oracle.spmm_f64(A.row_ptr, A.col, A.values().astype(np.float64), B.astype(np.float64))
    if scale is not None:
        ref = ref * scale.astype(np.float64)[:, None]
    if bias is not None:
        ref = ref + bias.astype(np.float64)[None, :]
    if terms["relu"]:
        ref = np.maximum(ref, 0.0)
    ref = torch.from_numpy(ref.astype(np.float32)).to(_OUT_T[out]).float().numpy()
    np.testing.assert_array_equal(Cd.float().cpu().numpy(), ref)
