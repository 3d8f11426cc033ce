"""Library baselines reported beside tcaspmm (cuSPARSE CSR, cuSPARSE Blocked-ELL, cuBLAS):
they must compute the same product, or their timings mean nothing."""
import numpy as np
import pytest
import torch

import oracle
import spmm_b200 as T

pytestmark = pytest.mark.gpu


def _inputs(A, N, dt):
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    B = T.gen_dense(A.ncol, N, 3, "f32")
    Bd = torch.from_numpy(B).to(tdt).cuda()
    vals = torch.from_numpy(A.values()).to(tdt).float().numpy()
    ref = oracle.spmm_f64(A.row_ptr, A.col, vals, Bd.float().cpu().numpy())
    return Bd, ref


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("shape", [(2048, 512, 256), (1000, 300, 72)])
def test_blocked_ell_matches_the_oracle(dt, shape):
    M, K, N = shape
    A = T.gen_uniform(M, K, 0.3, 4)
    Bd, ref = _inputs(A, N, dt)
    C = torch.full((M, N), float("nan"), device="cuda")
    ms, nbytes = T.cusparse_blocked_ell(A, 32, Bd, C, dt, warmup=1, iters=2)
    assert ms > 0 and nbytes >= A.nnz * 2
    assert oracle.rel_l2(C.cpu().numpy(), ref) <= 5e-3


def test_cusparse_csr_matches_the_oracle():
    A = T.gen_rmat(12, 40000, kind="gcn", seed=1)
    Bd, ref = _inputs(A, 64, "f32")
    C = torch.empty((A.nrow, 64), device="cuda")
    with T.Plan(A, 64, "f32") as p:
        ms = T.cusparse_spmm(p, Bd, C, warmup=1, iters=2)
    assert ms > 0 and oracle.rel_l2(C.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
def test_cublas_gold_matches_the_oracle(dt):
    """The dense cuBLAS GemmEx that the ./test driver uses as its gold (the reference's
    perform_GemmEx, src/gemm_cublas.cu:3-112): fp32 accumulation of the rounded inputs,
    so it agrees with the fp64 oracle to fp32 accumulation error."""
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    A = T.gen_uniform(2048, 512, 0.3, 0)  # the C1 weight
    Bd, ref = _inputs(A, 256, dt)
    Ad = torch.from_numpy(A.to_scipy().toarray()).to(tdt).cuda()
    C = torch.full((A.nrow, 256), float("nan"), device="cuda")
    ms = T.cublas_gemm(Ad, Bd, C, dt, warmup=1, iters=2)
    assert ms > 0
    assert oracle.rel_l2(C.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("dt,N", [("f32", 128), ("f32", 16), ("f16", 64)])
def test_gather_floor_runs_on_the_plan_columns(dt, N):
    """The gather-floor measurement (reported beside the kernel's time) runs on the plan's
    own device columns and B and takes positive time."""
    tdt = {"f16": torch.float16, "f32": torch.float32}[dt]
    A = T.gen_rmat(13, 80000, kind="gcn", seed=1)
    Bd = torch.from_numpy(T.gen_dense(A.ncol, N, 1, "f32")).to(tdt).cuda()
    with T.Plan(A, N, dt) as p:
        assert T.gather_floor(p, Bd, warmup=1, iters=3) > 0
