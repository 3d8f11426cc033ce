"""The no-allocation entry point, tcaspmm_spmm_csr_noalloc.

It serves callers that may not allocate device memory when they multiply
(a plugin inside a framework that owns every allocation, a latency-critical
loop, a fixed memory budget): A in CSR, B and C all live in the caller's device
memory, and the only scratch is a fixed array inside the library.  These tests
call it through the C-ABI and compare it with the plan-based entry point
(tcaspmm_execute1) on the same inputs, twice in a row, so a second call that
reuses the scratch array left by the first is checked too.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle
import spmm_b200 as T
from test_host_properties import csr_cases

_fn = T.lib.tcaspmm_spmm_csr_noalloc
_fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_int64,
                C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p]
_fn.restype = C.c_int

TOL = 1e-5  # both paths accumulate in fp32 on the CUDA cores


def _noalloc(rp, col, val, M, K, nnz, B, Cout, dt, stream):
    st = _fn(rp.data_ptr(), col.data_ptr(), val.data_ptr(), M, K, nnz, B.data_ptr(), B.stride(0), Cout.data_ptr(),
             Cout.stride(0), B.shape[1], int(T.as_dtype(dt)), stream.cuda_stream)
    if st != 0:
        raise T.TcaspmmError(st, T.last_error())


def test_rejects_n_beyond_the_fixed_scratch():
    # Two partial rows of N floats must fit in the 16 MiB scratch: N <= 2097152.
    st = _fn(None, None, None, 10, 10, 0, None, 1 << 22, None, 1 << 22, 1 << 22, 0, None)
    assert st == T.Status.UNSUPPORTED
    assert "scratch" in T.last_error()


def test_rejects_nnz_near_the_32_bit_limit():
    # Nonzero indices are 32-bit in the kernels: nnz within 64 of 2^31 is refused on the
    # host, before any pointer is touched.
    st = _fn(None, None, None, 10, 10, (1 << 31) - 10, None, 8, None, 8, 8, 0, None)
    assert st == T.Status.UNSUPPORTED
    assert "nnz" in T.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("case,dt,N", [("skew", "f32", 64), ("gcn", "f32", 128), ("c1", "f16", 256),
                                       ("skew", "bf16", 24), ("empty_rows", "f32", 8), ("wide", "f32", 4096)])
def test_noalloc_matches_plan_entry_on_two_calls(case, dt, N):
    import torch

    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dt]
    if case == "skew":
        A = T.gen_skew(200000, 8, 30000, 3.0, seed=21)     # hub rows span many chunks
    elif case == "wide":
        # nnz * 2 * N above the 4M floats of scratch: the chunk grows past its 256-nonzero
        # minimum (about 500 here), so the scratch limit, not the floor, sets the split.
        A = T.gen_skew(50000, 4, 40000, 3.0, seed=24)
        assert -(-A.nnz // (4 * 2**20 // (2 * N))) > 256
    elif case == "gcn":
        A = T.gen_rmat(15, 200000, kind="gcn", seed=22)
    elif case == "c1":
        A = T.gen_uniform(2048, 512, 0.3, 23)
    else:
        A = T.CSR(6, 5, np.array([0, 0, 2, 2, 2, 3, 3]), np.array([1, 4, 0]), np.array([1.5, -2.0, 3.0], np.float32))
    dev = torch.device("cuda", 0)
    B = torch.from_numpy(T.gen_dense(A.ncol, N, 3, "f32")).to(tdt).to(dev)
    rp = torch.from_numpy(A.row_ptr.astype(np.int32)).to(dev)
    col = torch.from_numpy(A.col).to(dev)
    val = torch.from_numpy(A.values()).to(tdt).to(dev)
    stream = torch.cuda.current_stream(dev)

    ref = torch.empty((A.nrow, N), device=dev)
    with T.Plan(A, N, dt) as p:            # the existing entry point
        p.execute1(B, ref, stream)
        p.sync_check()
    ref = ref.cpu().numpy()
    exact = oracle.spmm_f64(A.row_ptr, A.col, val.float().cpu().numpy(), B.float().cpu().numpy())
    outs = [torch.full((A.nrow, N), float("nan"), device=dev) for _ in range(2)]
    torch.cuda.synchronize(dev)
    free = []
    for call in range(2):                  # second call reuses the scratch left by the first
        if call == 1:
            free.append(torch.cuda.mem_get_info(dev)[0])
        _noalloc(rp, col, val, A.nrow, A.ncol, A.nnz, B, outs[call], dt, stream)
        torch.cuda.synchronize(dev)
        if call == 1:
            free.append(torch.cuda.mem_get_info(dev)[0])
        got = outs[call].cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: rows left unwritten"
        assert oracle.rel_l2(got, ref) <= TOL, f"call {call}"
        assert oracle.rel_l2(got, exact) <= TOL, f"call {call}"
    # The first call may commit the library's device image (lazy loading); after it,
    # a call must leave the device's free memory exactly where it was.
    assert free[1] == free[0], f"device free memory moved by {free[0] - free[1]} bytes on the second call"



@pytest.mark.gpu
@settings(max_examples=120, deadline=None, derandomize=True)
@given(A=csr_cases(), N=st.sampled_from([1, 4, 8, 16, 64, 136, 256]),
       dt=st.sampled_from(["f32", "f16", "bf16"]), seed=st.integers(0, 2**31 - 1))
def test_noalloc_is_exact_on_random_integer_matrices(A, N, dt, seed):
    """Random matrices (empty rows, hub rows, dense blocks, K below a tile) with small
    integer values through the no-allocation entry point: exact against the fp64
    oracle in every input type."""
    import torch

    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dt]
    rng = np.random.default_rng(seed)
    vals = rng.integers(-3, 4, A.nnz).astype(np.float32)
    Bh = rng.integers(-4, 5, (A.ncol, N)).astype(np.float32)
    dev = torch.device("cuda", 0)
    B = torch.from_numpy(Bh).to(tdt).to(dev)
    rp = torch.from_numpy(A.row_ptr.astype(np.int32)).to(dev)
    col = torch.from_numpy(A.col).to(dev)
    val = torch.from_numpy(vals).to(tdt).to(dev)
    out = torch.full((A.nrow, N), float("nan"), device=dev)
    _noalloc(rp, col, val, A.nrow, A.ncol, A.nnz, B, out, dt, torch.cuda.current_stream(dev))
    torch.cuda.synchronize(dev)
    exact = oracle.spmm_f64(A.row_ptr, A.col, vals.astype(np.float64), Bh.astype(np.float64))
    np.testing.assert_array_equal(out.cpu().numpy(), exact.astype(np.float32))
