"""Fused output epilogue (tcaspmm_execute_ex): C = relu?(row_scale[r] * (A B)[r, c] + bias[c]) as f32/f16/bf16.

The oracle is the fp64 CSR product with the same epilogue applied in fp64 and
rounded once to the output type.  Tolerances as in the plain parity tests
(1e-5 CUDA-core fp32, 5e-3 tensor-core path), plus the output type's own
rounding (half an ulp: 2^-11 fp16, 2^-8 bf16); integer-valued cases are
bit-exact on both kernels.
"""
import numpy as np
import pytest
import torch

import oracle
import spmm_b200 as T

pytestmark = pytest.mark.gpu

_TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "tf32": torch.float32}
_OUT_TOL = {"f32": 0.0, "f16": 2.0 ** -11, "bf16": 2.0 ** -8}


def _round(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(_TORCH[dt]).float().numpy()


def _run(A, B, dt, scale=None, bias=None, relu=False, out="f32", ldc_pad=0):
    K, N = B.shape
    Bd = torch.from_numpy(np.ascontiguousarray(B, np.float32)).to(_TORCH[dt]).cuda()
    Cd = torch.full((A.nrow, N + ldc_pad), float("nan"), dtype=_TORCH[out], device="cuda")
    sd = torch.from_numpy(scale).cuda() if scale is not None else None
    bd = torch.from_numpy(bias).cuda() if bias is not None else None
    with T.Plan(A, N, dt) as p:
        p.execute1(Bd, Cd[:, :N], stream=torch.cuda.current_stream(),
                   epilogue=T.Epilogue(sd, bd, relu, out))
        p.sync_check()
        st = p.stats
    torch.cuda.synchronize()
    if ldc_pad:
        assert torch.isnan(Cd[:, N:]).all(), "wrote outside the C view"
    return Cd[:, :N].float().cpu().numpy(), st


def _reference(A, B, dt, scale=None, bias=None, relu=False, out="f32"):
    R = oracle.spmm_f64(A.row_ptr, A.col, _round(A.values(), dt), _round(B, dt))
    if scale is not None:
        R = R * scale.astype(np.float64)[:, None]
    if bias is not None:
        R = R + bias.astype(np.float64)[None, :]
    if relu:
        R = np.maximum(R, 0.0)
    return R


def _check(A, N, dt, out, seed=0, **ep):
    rng = np.random.default_rng(seed)
    B = T.gen_dense(A.ncol, N, seed, "f32")
    ep = {k: (v(rng, A, N) if callable(v) else v) for k, v in ep.items()}
    got, st = _run(A, B, dt, out=out, **ep)
    ref = _reference(A, B, dt, **ep)
    base = 5e-3 if st["tc_nnz"] > 0 else 1e-5
    err = oracle.rel_l2(got, ref)
    assert err <= base + _OUT_TOL[out], (err, st)
    return st


def _scale(rng, A, N):
    return rng.uniform(0.25, 2.0, A.nrow).astype(np.float32)


def _bias(rng, A, N):
    return rng.standard_normal(N).astype(np.float32)


CASES = {
    "gcn": lambda: T.gen_rmat(14, 150000, kind="gcn", seed=2),
    "skew": lambda: T.gen_skew(100000, 8, 30000, 3.0, seed=4),
    "c1": lambda: T.gen_uniform(1024, 512, 0.3, 0),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("dt,N", [("f16", 128), ("f32", 64), ("bf16", 40), ("tf32", 96)])
@pytest.mark.parametrize("out", ["f32", "bf16", "f16"])
def test_scale_bias_relu(case, dt, N, out):
    st = _check(CASES[case](), N, dt, out, scale=_scale, bias=_bias, relu=True)
    if case == "c1" and dt != "f32" and N % 8 == 0:  # 16-bit and tf32 take the tensor cores
        assert st["tc_windows"] > 0
    if case == "skew":  # hub rows: residue segments, or gathered windows when those are on
        assert st["residue_segments"] > 0 or st["tc_gathered_windows"] > 0


@pytest.mark.parametrize("ep", [dict(scale=_scale), dict(bias=_bias), dict(relu=True), {}])
def test_each_epilogue_term_alone(ep):
    _check(T.gen_rmat(13, 60000, kind="gcn", seed=5), 64, "f16", "f32", **ep)
    _check(T.gen_uniform(512, 256, 0.4, 6), 64, "f16", "f32", **ep)


def test_unaligned_output_takes_the_scalar_path():
    _check(T.gen_uniform(300, 200, 0.1, 5), 37, "f16", "bf16", scale=_scale, bias=_bias, relu=True)
    A = T.gen_uniform(256, 256, 0.4, 12)
    B = T.gen_dense(256, 64, 1, "f32")
    got, st = _run(A, B, "f16", bias=np.ones(64, np.float32), out="bf16", ldc_pad=3)
    assert st["tc_windows"] > 0
    assert oracle.rel_l2(got, _reference(A, B, "f16", bias=np.ones(64, np.float32))) <= 5e-3 + 2.0 ** -8


@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_integer_values_bit_exact_on_both_kernels(out):
    """Integers, power-of-two scales, integer bias: every step is exact, bf16 output included."""
    rng = np.random.default_rng(9)
    dense = T.gen_uniform(512, 256, 0.5, 13)          # tensor-core windows
    sparse = T.gen_rmat(8, 3000, kind="gcn", seed=3)   # 256 x 256, mostly residue rows
    kinds = []
    for A in (dense, sparse):
        A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, rng.integers(-3, 4, A.nnz).astype(np.float32))
        B = np.round(T.gen_dense(256, 64, 2, "f32") * 2).astype(np.float32)
        scale = (2.0 ** rng.integers(-2, 2, A.nrow)).astype(np.float32)
        bias = rng.integers(-3, 4, 64).astype(np.float32)
        got, st = _run(A, B, "f16", scale=scale, bias=bias, relu=True, out=out)
        kinds.append((st["tc_nnz"], st["residue_nnz"]))
        ref = _reference(A, B, "f16", scale=scale, bias=bias, relu=True)
        ref = torch.from_numpy(ref.astype(np.float32)).to(_TORCH[out]).float().numpy()
        np.testing.assert_array_equal(got, ref)
    assert kinds[0][0] > 0 and kinds[1][1] > 0


def test_sage_mean_is_pattern_times_inverse_degree():
    """GraphSAGE mean: pattern A with row_scale = 1/deg equals A with values 1/deg."""
    A = T.gen_rmat(13, 80000, kind="gcn", seed=7)
    deg = np.diff(A.row_ptr).astype(np.float32)
    inv = np.where(deg > 0, 1.0 / np.maximum(deg, 1), 0.0).astype(np.float32)
    pattern = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, np.ones(A.nnz, np.float32))
    B = T.gen_dense(A.ncol, 64, 3, "f32")
    got, _ = _run(pattern, B, "f32", scale=inv)
    mean = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, np.repeat(inv, np.diff(A.row_ptr)))
    assert oracle.rel_l2(got, oracle.spmm_f64(mean.row_ptr, mean.col, mean.values(), B)) <= 1e-5


@pytest.mark.parametrize("out", ["f32", "bf16"])
@pytest.mark.parametrize("split", ["128", "4"])
def test_epilogue_through_gathered_windows(out, split, monkeypatch):
    """Row scales, bias and ReLU applied through the row lists of the gathered windows of
    long rows, with and without their tile chains split into parts."""
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    monkeypatch.setenv("TCASPMM_SPLIT_TILES", split)
    st = _check(T.gen_rmat(15, 400000, kind="gcn", seed=2), 128, "f16", out, scale=_scale, bias=_bias, relu=True)
    assert st["tc_gathered_windows"] > 0


@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_integer_epilogue_on_cut_chains_beside_the_residue(out):
    """16 long consecutive windows (their tile chains cut into parts for the idle SMs and
    reduced in part order) next to sparse rows on the residue kernel, the two kernels on
    two streams: integers, power-of-two scales and an integer bias, bit-exact."""
    rng = np.random.default_rng(17)
    d, s = T.gen_uniform(512, 1024, 0.5, 3), T.gen_uniform(3000, 1024, 0.005, 4)
    A = T.CSR(d.nrow + s.nrow, d.ncol, np.concatenate([d.row_ptr, s.row_ptr[1:] + d.nnz]),
              np.concatenate([d.col, s.col]), None)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, rng.integers(-3, 4, A.nnz).astype(np.float32))
    B = np.round(T.gen_dense(1024, 128, 2, "f32") * 2).astype(np.float32)
    scale = (2.0 ** rng.integers(-2, 2, A.nrow)).astype(np.float32)
    bias = rng.integers(-3, 4, 128).astype(np.float32)
    got, st = _run(A, B, "f16", scale=scale, bias=bias, relu=True, out=out)
    assert st["tc_windows"] == 16 and st["tc_tasks"] > 16 and st["tc_side_stream"] == 1, st
    ref = _reference(A, B, "f16", scale=scale, bias=bias, relu=True)
    ref = torch.from_numpy(ref.astype(np.float32)).to(_TORCH[out]).float().numpy()
    np.testing.assert_array_equal(got, ref)
