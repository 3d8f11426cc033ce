"""Host-side pieces of bench.py: the generator loader of the reference arm and the
parity sample that every bench line (each rank of a multi-GPU run) carries."""
import os
import subprocess
import sys

import numpy as np
import pytest

import bench
import oracle
import spmm_b200 as T


def test_reference_arm_generators_match_the_library_and_load_no_gpu_code():
    H = bench.HostGen()
    for f in (lambda m: m.gen_uniform(512, 256, 0.3, 2), lambda m: m.gen_rmat(12, 30000, kind="sage", seed=3),
              lambda m: m.gen_skew(50000, 3, 2000, 3.0, seed=4)):
        a, b = f(H), f(T)
        assert np.array_equal(a.row_ptr, b.row_ptr) and np.array_equal(a.col, b.col)
        assert np.array_equal(a.values(), b.values())
    for dt in ("f32", "f16", "bf16"):
        assert np.array_equal(H.gen_dense(64, 24, 5, dt), T.gen_dense(64, 24, 5, dt))
    # A fresh interpreter that builds the reference arm's inputs maps no CUDA library.
    code = ("import sys; sys.path.insert(0, %r); import bench; H = bench.HostGen(); H.gen_rmat(10, 5000); "
            "maps = open('/proc/self/maps').read(); "
            "print('libtcaspmm.so' in maps, 'libcudart' in maps)" % os.path.dirname(bench.__file__))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["False", "False"], out


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_parity_sample_is_zero_for_the_exact_product_and_catches_a_wrong_row(dt):
    A = T.gen_rmat(11, 20000, kind="gcn", seed=7)
    B = T.gen_dense(A.ncol, 32, 1, dt)
    vals = bench._round_to(A.values(), dt)
    exact = oracle.spmm_f64(A.row_ptr, A.col, vals, bench._as_f32(B, dt))
    rl = np.diff(A.row_ptr)
    rows = np.unique(np.concatenate([np.argsort(-rl)[:8], np.arange(0, A.nrow, 7)]))
    assert bench.parity_sample(A, B, exact[rows], rows, dt) < 1e-12
    assert bench.parity_sample(A, B, exact[rows], rows, dt, chunk=5) < 1e-12  # long rows in pieces
    wrong = exact[rows].copy()
    wrong[0] *= 1.01
    assert bench.parity_sample(A, B, wrong, rows, dt) > 1e-4


def test_parity_sample_applies_the_epilogue():
    A = T.gen_uniform(300, 200, 0.1, 3)
    B = T.gen_dense(A.ncol, 16, 2, "f32")
    rs = np.linspace(0.5, 1.5, A.nrow)
    bias = np.linspace(-1, 1, 16)
    ab = oracle.spmm_f64(A.row_ptr, A.col, A.values(), B)
    y = np.maximum(rs[:, None] * ab + bias, 0.0)
    rows = np.arange(A.nrow)
    assert bench.parity_sample(A, B, y, rows, "f32", (rs, bias)) < 1e-12
    assert bench.parity_sample(A, B, ab, rows, "f32", (rs, bias)) > 1e-3


def test_bf16_rounding_is_round_to_nearest_even():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(bench._round_to(x, "bf16"), ref)


def test_traffic_is_reported_only_for_the_profiled_configuration():
    """The committed ncu DRAM bytes belong to one configuration per workload (its own
    dtype and N, one GPU, column split, no tuning variables); any other run reports
    traffic null rather than a figure measured on something else."""
    assert bench.load_traffic("gcn") == bench.load_traffic("gcn", profiled_config=True)
    assert isinstance(bench.load_traffic("gcn"), int) and bench.load_traffic("gcn") > 0
    assert bench.load_traffic("gcn", profiled_config=False) is None
    assert bench.load_traffic("no-such-workload") is None
