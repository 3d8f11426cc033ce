"""Full-size configs checked through size-independent properties.

At the GNN/skew sizes the fp64 oracle over every row would take minutes, so
each run is checked by:
  * column checksum  1^T C = (A^T 1)^T B   and row checksum  C 1 = A (B 1),
    both in fp64 on the host in O(nnz + K N);
  * exact fp64 oracle rows on a seeded sample of rows (hub rows included).
"""
import numpy as np
import pytest
import torch

import oracle
import spmm_b200 as T

pytestmark = pytest.mark.gpu


def _run_full(A, N, dt, seed=0):
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dt]
    B = T.gen_dense(A.ncol, N, seed, "f32")
    Bd = torch.from_numpy(B).to(tdt).cuda()
    Cd = torch.empty((A.nrow, N), device="cuda")
    with T.Plan(A, N, dt) as p:
        p.execute1(Bd, Cd)
        p.sync_check()
    Bq = Bd.float().cpu().numpy()
    vals = torch.from_numpy(A.values()).to(tdt).float().numpy()
    return Cd.cpu().numpy(), Bq, vals


def _checks(A, out, Bq, vals, tol):
    colsum_ref = np.bincount(A.col, weights=vals.astype(np.float64), minlength=A.ncol) @ Bq.astype(np.float64)
    assert oracle.rel_l2(out.sum(axis=0, dtype=np.float64), colsum_ref) < tol
    rowvec = Bq.astype(np.float64).sum(axis=1)
    rows = np.repeat(np.arange(A.nrow), np.diff(A.row_ptr))
    rowsum_ref = np.bincount(rows, weights=vals * rowvec[A.col], minlength=A.nrow)
    assert oracle.rel_l2(out.sum(axis=1, dtype=np.float64), rowsum_ref) < tol
    rng = np.random.default_rng(0)
    lens = np.diff(A.row_ptr)
    sample = np.unique(np.concatenate([rng.integers(0, A.nrow, 2000), np.argsort(lens)[-8:]]))
    sub_rp = np.concatenate([[0], np.cumsum(lens[sample])])
    idx = np.concatenate([np.arange(A.row_ptr[r], A.row_ptr[r + 1]) for r in sample])
    ref = oracle.spmm_f64(sub_rp, A.col[idx], vals[idx], Bq)
    assert oracle.rel_l2(out[sample], ref) < tol


def test_c3_gcn_1m_nodes_n128_f32():
    A = T.gen_rmat(20, 30_000_000, kind="gcn", seed=0)
    out, Bq, vals = _run_full(A, 128, "f32")
    _checks(A, out, Bq, vals, 1e-5)


def test_c4_sage_4m_nodes_n256_f16():
    A = T.gen_rmat(22, 100_000_000, kind="sage", seed=0)
    out, Bq, vals = _run_full(A, 256, "f16")
    _checks(A, out, Bq, vals, 1e-5)


def test_c5_extreme_skew_n64_f16():
    A = T.gen_skew(1 << 23, 64, 200_000, 3.0, seed=0)
    out, Bq, vals = _run_full(A, 64, "f16")
    _checks(A, out, Bq, vals, 1e-5)
