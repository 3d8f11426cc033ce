"""Property tests of the host schedule (no GPU): for random CSR matrices (empty
rows, hub rows, dense row blocks that become tensor-core windows, some with tile
chains of hundreds of tiles, K below a tile), random widths, dtypes and tuning
variables, the schedule covers every nonzero exactly once, splits the nonzeros
consistently between the tensor-core windows and the residue kernel, and never
puts fp32 on the tensor cores; one corruption of such a matrix is refused at the
boundary.

Examples are derandomized so every run checks the same cases."""
import contextlib
import os

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

import spmm_b200 as T


@contextlib.contextmanager
def _env(values: dict):
    old = {k: os.environ.get(k) for k in values}
    os.environ.update({k: str(v) for k, v in values.items()})
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@st.composite
def csr_cases(draw):
    shape = draw(st.sampled_from(["sparse", "hubs", "dense_block", "empty_rows", "long_windows"]))
    M = draw(st.integers(1, 400 if shape != "long_windows" else 160))
    K = draw(st.integers(1, 600) if shape != "long_windows" else st.integers(600, 6000))
    rng = np.random.default_rng(draw(st.integers(0, 2**31 - 1)))
    lam = {"sparse": 3.0, "hubs": 2.0, "dense_block": 1.0, "empty_rows": 0.3, "long_windows": 2.0}[shape]
    lens = np.minimum(rng.poisson(lam, M), K)
    if shape == "hubs":
        for r in rng.choice(M, size=min(M, 4), replace=False):
            lens[r] = rng.integers(K // 2, K + 1)
    if shape in ("dense_block", "long_windows"):
        # A block of rows dense enough for tensor-core windows; with long_windows
        # their tile chains run to hundreds of tiles (many index chunks and parts).
        lo, hi = (0.2, 0.9) if shape == "dense_block" else (0.05, 0.4)
        r0 = int(rng.integers(0, M))
        rows = np.arange(r0, min(M, r0 + int(rng.integers(16, 97))))
        lens[rows] = np.maximum(1, (K * rng.uniform(lo, hi, rows.size)).astype(np.int64))
    cols = [np.sort(rng.choice(K, size=int(n), replace=False)).astype(np.int32) for n in lens]
    rp = np.zeros(M + 1, np.int64)
    rp[1:] = np.cumsum(lens)
    col = np.concatenate(cols) if cols else np.zeros(0, np.int32)
    val = rng.standard_normal(col.size).astype(np.float32)
    return T.CSR(M, K, rp, col, val)


@settings(max_examples=200, deadline=None, derandomize=True)
@given(A=csr_cases(),
       N=st.sampled_from([1, 4, 7, 8, 16, 24, 64, 128, 200, 256]),
       dt=st.sampled_from(["f32", "f16", "bf16", "tf32"]),
       env=st.fixed_dictionaries({
           "TCASPMM_HUB_WINDOWS": st.sampled_from([0, 1]),
           "TCASPMM_TC_DENSITY": st.sampled_from([1, 8, 32, 1024]),
           "TCASPMM_BUDGET_MAX": st.sampled_from([16, 64, 1024]),
           "TCASPMM_BUDGET_MIN": st.sampled_from([1, 128]),
           "TCASPMM_WARPS_PER_SM": st.sampled_from([1, 32]),
       }))
def test_schedule_covers_every_nonzero_once(A, N, dt, env):
    with _env(env):
        cover, kind, s = T.schedule_coverage(A, N, dt)
    assert np.all(cover == 1), (np.bincount(cover), s)
    assert s["tc_nnz"] + s["residue_nnz"] == A.nnz
    assert int((kind == 3).sum()) == s["tc_nnz"]
    if dt == "f32":
        assert s["tc_windows"] == 0
    if env["TCASPMM_HUB_WINDOWS"] == 0:
        assert s["tc_gathered_windows"] == 0


@settings(max_examples=200, deadline=None, derandomize=True)
@given(A=csr_cases(), how=st.sampled_from(["col_high", "col_negative", "duplicate", "unsorted",
                                           "ptr_decreases", "ptr_end", "ptr_start"]),
       pick=st.integers(0, 2**31 - 1))
def test_malformed_csr_is_rejected_not_computed(A, how, pick):
    """One corruption of a valid CSR -- a column out of range or negative, a repeated
    or out-of-order column in a row, row offsets that decrease or do not span nnz --
    is refused at the boundary with a format error (never a crash, never a product
    that silently mis-sums a repeated column on the tensor cores)."""
    T.schedule_coverage(A, 16, "f16")  # the valid matrix passes
    rp, col = A.row_ptr.copy(), A.col.copy()
    multi = np.flatnonzero(np.diff(rp) >= 2)  # rows with two or more nonzeros
    rng = np.random.default_rng(pick)
    if how == "col_high" and A.nnz:
        col[rng.integers(A.nnz)] = A.ncol
    elif how == "col_negative" and A.nnz:
        col[rng.integers(A.nnz)] = -1
    elif how in ("duplicate", "unsorted") and multi.size:
        r = multi[rng.integers(multi.size)]
        j = rp[r] + rng.integers(rp[r + 1] - rp[r] - 1)
        if how == "duplicate":
            col[j + 1] = col[j]
        else:
            col[j], col[j + 1] = col[j + 1], col[j]
    elif how == "ptr_decreases" and A.nrow >= 2 and A.nnz:
        i = 1 + rng.integers(A.nrow - 1)
        rp[i] = rp[i + 1] + 1 if rp[i + 1] + 1 <= A.nnz else rp[i - 1] - 1
    elif how == "ptr_end":
        rp[-1] = A.nnz + 1
    elif how == "ptr_start":
        rp[0] = 1
    else:
        return  # this matrix has nothing to corrupt that way
    bad = T.CSR(A.nrow, A.ncol, rp, col, A.values())
    with pytest.raises(T.TcaspmmError) as e:
        T.schedule_coverage(bad, 16, "f16")
    assert e.value.status in (T.Status.FORMAT, T.Status.INVALID_ARG), e.value


@settings(max_examples=80, deadline=None, derandomize=True)
@given(A=csr_cases(), pattern=st.booleans())
def test_matrix_files_round_trip(A, pattern, tmp_path_factory):
    """A random matrix written as .smtx (with its .val values, or as a pattern) and as
    binary CSR reads back identical: offsets, columns and values bit for bit."""
    d = tmp_path_factory.mktemp("files")
    M = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, None if pattern else A.values())
    T.smtx_write(str(d / "a.smtx"), M)
    T.csrbin_write(str(d / "a.csrb"), M)
    for back in (T.smtx_read(str(d / "a.smtx")), T.csrbin_read(str(d / "a.csrb"))):
        assert (back.nrow, back.ncol, back.nnz) == (M.nrow, M.ncol, M.nnz)
        np.testing.assert_array_equal(back.row_ptr, M.row_ptr)
        np.testing.assert_array_equal(back.col, M.col)
        np.testing.assert_array_equal(back.values(), M.values())
