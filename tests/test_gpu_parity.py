"""CUDA path vs the CPU oracle, through the C-ABI library.

Tolerances (north star): rel-L2 <= 1e-5 against the fp64 CSR oracle on the
same rounded inputs for the CUDA-core path, <= 5e-3 for the tensor-core path
(fp16/bf16 windows).  Integer-valued inputs are compared bit-exactly.
"""
import numpy as np
import pytest
import torch

import oracle
import spmm_b200 as T

pytestmark = pytest.mark.gpu

TOL_CORE = 1e-5
TOL_TC = 5e-3


def _torch_dt(dt):
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "tf32": torch.float32}[dt]


def _round(x: np.ndarray, dt: str) -> np.ndarray:
    """Values as the device sees them (rounded to dt), widened to float32."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(_torch_dt(dt)).float().numpy()


def run(A: T.CSR, B: np.ndarray, dt: str, ldb_pad: int = 0, ldc_pad: int = 0, stream=None):
    """C = A @ B on cuda:0 through tcaspmm_execute1; B given in fp32, rounded to dt."""
    K, N = B.shape
    Bt = torch.from_numpy(np.ascontiguousarray(B, np.float32)).to(_torch_dt(dt))
    Bd = torch.zeros((K, N + ldb_pad), dtype=_torch_dt(dt), device="cuda")
    Bd[:, :N] = Bt.cuda()
    Cd = torch.full((A.nrow, N + ldc_pad), float("nan"), dtype=torch.float32, device="cuda")
    with T.Plan(A, N, dt) as p:
        p.execute1(Bd[:, :N], Cd[:, :N], stream=stream or torch.cuda.current_stream())
        p.sync_check()
        st = p.stats
    torch.cuda.synchronize()
    if ldc_pad:
        assert torch.isnan(Cd[:, N:]).all(), "wrote outside the C view"
    return Cd[:, :N].cpu().numpy(), st


def reference(A: T.CSR, B: np.ndarray, dt: str) -> np.ndarray:
    return oracle.spmm_f64(A.row_ptr, A.col, _round(A.values(), dt), _round(B, dt))


def check(A, N, dt, seed=0, tol=None, **kw):
    B = T.gen_dense(A.ncol, N, seed, "f32")
    out, st = run(A, B, dt, **kw)
    ref = reference(A, B, dt)
    if tol is None:
        tol = TOL_TC if st["tc_nnz"] > 0 else TOL_CORE
    err = oracle.rel_l2(out, ref)
    assert err <= tol, (err, st)
    assert np.isfinite(out).all()
    return out, st


def test_bundled_integer_known_answer_bit_exact(bundled):
    A = T.CSR(int(bundled["M"]), int(bundled["K"]), bundled["row_ptr"], bundled["col"], None)
    out, _ = run(A, bundled["B_int"].astype(np.float32), "f16")
    np.testing.assert_array_equal(out, bundled["C_int"])


def test_bundled_random_matches_reference_gemm(bundled):
    A = T.CSR(int(bundled["M"]), int(bundled["K"]), bundled["row_ptr"], bundled["col"], None)
    out, _ = run(A, bundled["B_rand"].astype(np.float32), "f16")
    assert oracle.rel_l2(out, bundled["C_rand"]) < 1e-6


def test_small_reference_cases(small_cases):
    for c in small_cases:
        A = T.CSR(c["M"], c["K"], c["row_ptr"], c["col"], c["val"].astype(np.float32))
        out, _ = run(A, c["B"].astype(np.float32), "f16")
        assert oracle.rel_l2(out, c["C"]) < 1e-6, c["dense"].shape


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("N", [256, 1, 7, 24, 64, 129, 512])
def test_c1_ffn_uniform(dt, N):
    check(T.gen_uniform(2048, 512, 0.3, 0), N, dt)


@pytest.mark.parametrize("shape", [(512, 2048), (2048, 2048), (4096, 1024)])
@pytest.mark.parametrize("sparsity", [0.5, 0.7, 0.8, 0.9, 0.95, 0.98])
@pytest.mark.parametrize("kind", ["uniform", "magnitude"])
def test_c2_sweep(shape, sparsity, kind):
    """The full pruned-weight grid of the sweep config: three shapes x six sparsities x
    two structures, fp16 at N = 64 / 128 / 256 / 512 and fp32 at N = 64 / 256."""
    M, K = shape
    A = T.gen_uniform(M, K, 1 - sparsity, 1) if kind == "uniform" else T.gen_magnitude(M, K, sparsity, 1)
    for dt, N in (("f16", 64), ("f16", 128), ("f16", 256), ("f16", 512), ("f32", 64), ("f32", 256)):
        check(A, N, dt)


@pytest.mark.parametrize("dt,N", [("f32", 128), ("f16", 128), ("f32", 16), ("f16", 32), ("f32", 8), ("f32", 4), ("bf16", 16)])
def test_gcn_rmat_small(dt, N):
    check(T.gen_rmat(16, 500000, kind="gcn", seed=2), N, dt)


@pytest.mark.parametrize("dt,N", [("f16", 64), ("f32", 64), ("bf16", 8), ("f32", 8)])
def test_skew_hub_rows_use_segments(dt, N):
    A = T.gen_skew(300000, 16, 50000, 3.0, seed=4)
    _, st = check(A, N, dt)
    assert st["long_rows"] >= 16 and st["residue_segments"] > 16


def test_sage_mean_small():
    check(T.gen_rmat(15, 400000, kind="sage", seed=3), 256, "f16")


def test_unaligned_leading_dimensions_take_scalar_path():
    A = T.gen_uniform(300, 200, 0.1, 5)
    check(A, 37, "f16", ldb_pad=3, ldc_pad=1)
    check(A, 37, "f32", ldb_pad=1, ldc_pad=3)


def test_padded_views_do_not_write_outside_c():
    A = T.gen_uniform(100, 64, 0.2, 6)
    check(A, 64, "f16", ldb_pad=8, ldc_pad=4)


def test_edge_shapes():
    empty = T.CSR(50, 20, np.zeros(51, np.int64), np.zeros(0, np.int32), None)
    out, _ = run(empty, np.ones((20, 16), np.float32), "f32")
    assert np.all(out == 0)
    one = T.CSR(3, 4, np.array([0, 0, 1, 1]), np.array([2]), np.array([-2.5], np.float32))
    B = np.arange(4 * 8, dtype=np.float32).reshape(4, 8)
    out, _ = run(one, B, "f32")
    np.testing.assert_array_equal(out, np.vstack([np.zeros(8), -2.5 * B[2], np.zeros(8)]))
    out, _ = run(T.CSR(0, 5, np.zeros(1, np.int64), np.zeros(0, np.int32), None), np.ones((5, 8), np.float32), "f16")
    assert out.shape == (0, 8)
    check(T.gen_uniform(1, 1, 1.0, 0), 1, "f32")


def test_single_dense_row_and_column():
    row = T.gen_uniform(1, 50000, 1.0, 7)       # one hub row: segments + fix-up
    _, st = check(row, 64, "f32")
    assert st["residue_segments"] > 1
    colm = T.gen_uniform(20000, 1, 1.0, 8)      # every row has one nonzero
    check(colm, 256, "f16")


def test_deterministic_across_runs():
    A = T.gen_skew(100000, 8, 40000, 3.0, seed=9)
    B = T.gen_dense(A.ncol, 64, 1, "f32")
    a, _ = run(A, B, "f32")
    b, _ = run(A, B, "f32")
    np.testing.assert_array_equal(a, b)


def test_runs_on_a_side_stream():
    s = torch.cuda.Stream()
    A = T.gen_uniform(1000, 300, 0.05, 10)
    check(A, 128, "f32", stream=s)


def test_reference_entry_point_bit_exact(bundled):
    M, K, N = int(bundled["M"]), int(bundled["K"]), int(bundled["N"])
    Cout = np.zeros(M * N, np.float32)
    ms = T.our_spmm_balanced(bundled["row_ptr"].astype(np.int32), bundled["col"], bundled["val_bits"].view(np.float16),
                             bundled["B_int"], Cout, M, N, K, 10)
    assert ms > 0
    np.testing.assert_array_equal(Cout.reshape(M, N), bundled["C_int"])


@pytest.mark.parametrize("case", ["gcn_f32", "mixed_f16"])
def test_multi_gpu_column_shards(case):
    """One plan over two GPUs, each owning a column block of B and C.  mixed_f16:
    tensor-core windows beside residue rows, so each device's shard runs its tile
    kernel on its own side stream; integer values, bit-exact."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU")
    if case == "gcn_f32":
        A = T.gen_rmat(14, 100000, kind="gcn", seed=1)
        N, dt = 128, "f32"
        B = T.gen_dense(A.ncol, N, 3, "f32")
    else:
        g = np.random.default_rng(43)
        A = _vstack(T.gen_uniform(512, 1024, 0.5, 3), T.gen_uniform(3000, 1024, 0.005, 4))
        A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, g.integers(-3, 4, A.nnz).astype(np.float32))
        N, dt = 256, "f16"
        B = g.integers(-4, 5, (A.ncol, N)).astype(np.float32)
    with T.Plan(A, N, dt, num_gpus=2) as p:
        Bs, Cs = [], []
        for s in range(2):
            dev, b, c = p.shard(s)
            Bs.append(torch.from_numpy(B[:, b:b + c].copy()).to(_torch_dt(dt)).to(f"cuda:{dev}"))
            Cs.append(torch.empty((A.nrow, c), device=f"cuda:{dev}"))
        p.execute(Bs, Cs, streams=[torch.cuda.current_stream(f"cuda:{p.shard(s)[0]}") for s in range(2)])
        p.sync_check()
        st = p.stats
        out = np.hstack([c.cpu().numpy() for c in Cs])
    if case == "gcn_f32":
        assert oracle.rel_l2(out, reference(A, B, dt)) <= TOL_CORE
    else:
        assert st["tc_windows"] == 16 and st["tc_side_stream"] == 1, st
        np.testing.assert_array_equal(out, reference(A, B, dt).astype(np.float32))


@pytest.mark.parametrize("dt", ["f16", "bf16", "tf32"])
@pytest.mark.parametrize("N", [256, 128, 64, 8, 200])
def test_tensor_core_windows(dt, N):
    """C1 at 70% sparsity: every window is dense enough for the tcgen05 tiles."""
    _, st = check(T.gen_uniform(2048, 512, 0.3, 0), N, dt)
    assert st["tc_windows"] == 64 and st["tc_nnz"] == st["nnz"]


def _vstack(a: T.CSR, b: T.CSR) -> T.CSR:
    return T.CSR(a.nrow + b.nrow, a.ncol, np.concatenate([a.row_ptr, b.row_ptr[1:] + a.nnz]),
                 np.concatenate([a.col, b.col]), np.concatenate([a.values(), b.values()]))


def test_tensor_core_windows_mixed_with_residue():
    """Dense rows on tcgen05 next to sparse rows on CUDA cores in one matrix."""
    A = _vstack(T.gen_uniform(512, 1024, 0.5, 3), T.gen_uniform(3000, 1024, 0.005, 4))
    _, st = check(A, 128, "f16")
    assert st["tc_windows"] == 16 and st["residue_nnz"] > 0


@pytest.mark.parametrize("overlap", ["1", "0"])
def test_mixed_plan_captured_in_a_cuda_graph(overlap, monkeypatch):
    """A plan with tensor-core windows and residue rows forks its tensor-core kernel
    onto a side stream and joins it back: captured in a CUDA graph on a non-default
    stream and replayed, integer values bit-exact (and the same with both kernels on
    the caller's stream)."""
    monkeypatch.setenv("TCASPMM_OVERLAP", overlap)
    g = np.random.default_rng(41)
    A = _vstack(T.gen_uniform(512, 1024, 0.5, 3), T.gen_uniform(3000, 1024, 0.005, 4))
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, g.integers(-3, 4, A.nnz).astype(np.float32))
    B = g.integers(-4, 5, (A.ncol, 128)).astype(np.float32)
    Bd = torch.from_numpy(B).to(torch.float16).cuda()
    Cd = torch.zeros((A.nrow, 128), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with T.Plan(A, 128, "f16") as p:
        st = p.stats
        assert st["tc_windows"] == 16 and st["residue_nnz"] > 0, st
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            p.execute1(Bd, Cd, stream=s)  # warm-up outside the capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            p.execute1(Bd, Cd, stream=s)
        Cd.zero_()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        p.sync_check()
        del graph
    np.testing.assert_array_equal(Cd.cpu().numpy(), reference(A, B, "f16").astype(np.float32))


def test_few_windows_cut_into_parts_beside_the_residue():
    """16 consecutive windows x 1 column block leave most of 148 SMs idle: their tile
    chains are cut into parts and the tensor-core kernel runs beside the residue
    kernel on the plan's side stream.  C1's 64 windows x 2 column blocks stay whole,
    and with no residue rows nothing forks."""
    A = _vstack(T.gen_uniform(512, 1024, 0.5, 3), T.gen_uniform(3000, 1024, 0.005, 4))
    _, st = check(A, 128, "f16")
    assert st["tc_windows"] == 16 and st["tc_tasks"] > 16 and st["tc_side_stream"] == 1, st
    _, st = check(T.gen_uniform(2048, 512, 0.3, 0), 256, "f16")
    assert st["tc_tasks"] == 64 and st["tc_side_stream"] == 0, st


def test_tensor_core_partial_window_and_block():
    """M not a multiple of 32 rows, N not a multiple of 128 columns."""
    _, st = check(T.gen_uniform(1000, 300, 0.4, 11), 72, "f16")
    assert st["tc_windows"] > 0


@pytest.mark.parametrize("dt", ["f16", "tf32"])
def test_tensor_core_unaligned_b_falls_back_to_cuda_cores(dt):
    _, st = check(T.gen_uniform(256, 256, 0.4, 12), 64, dt, ldb_pad=3)
    assert st["tc_windows"] > 0


def test_tensor_core_integer_values_bit_exact():
    """Small integers: every product and partial sum is exact in fp32, on tcgen05 too."""
    A = T.gen_uniform(512, 256, 0.5, 13)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, np.round(A.val * 2).astype(np.float32))
    B = np.round(T.gen_dense(256, 128, 2, "f32") * 3).astype(np.float32)
    out, st = run(A, B, "f16")
    assert st["tc_windows"] > 0
    np.testing.assert_array_equal(out, reference(A, B, "f16").astype(np.float32))


@pytest.mark.parametrize("dt", ["f16", "tf32"])
@pytest.mark.parametrize("K", [12, 40, 64, 70])
def test_tensor_core_windows_with_few_b_rows(K, dt):
    """K below the 16- and 64-row TMA boxes: the boxes are clipped to K and only
    the forms that fit are issued (no index-free runs below K = 64)."""
    A = T.gen_uniform(256, K, 0.6, K)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, np.round(A.val * 4).astype(np.float32))
    B = np.round(T.gen_dense(K, 64, 3, "f32") * 4).astype(np.float32)
    out, st = run(A, B, dt)
    assert st["tc_windows"] > 0
    np.testing.assert_array_equal(out, reference(A, B, dt).astype(np.float32))


def test_fp32_never_uses_tensor_cores_tf32_does():
    """TCASPMM_F32 keeps the fp32 CUDA-core path (1e-5); TF32 is the opt-in tensor-core form (5e-3)."""
    A = T.gen_uniform(1024, 512, 0.3, 5)
    _, st32 = check(A, 128, "f32")
    _, sttf = check(A, 128, "tf32")
    assert st32["tc_windows"] == 0 and sttf["tc_windows"] == 32


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_row_split_plan_on_one_device(dt):
    """Row-split plan with two shards placed on cuda:0: each shard writes its row
    block of C from the whole B; tensor-core windows and residue rows in both."""
    A = _vstack(T.gen_uniform(256, 4096, 0.3, 1), T.gen_rmat(12, 60000, kind="gcn", seed=9))
    A = _vstack(A, T.gen_uniform(96, 4096, 0.3, 2))
    N = 64
    B = T.gen_dense(A.ncol, N, 4, "f32")
    Bd = torch.from_numpy(B).to(_torch_dt(dt)).cuda()
    Cd = torch.full((A.nrow, N), float("nan"), device="cuda")
    scale = torch.rand(A.nrow, device="cuda") + 0.5
    Ce = torch.full((A.nrow, N), float("nan"), device="cuda")
    with T.Plan(A, N, dt, num_gpus=2, devices=[0, 0], split="rows") as p:
        blocks = [p.shard_rows(s) for s in range(2)]
        assert blocks[0][0] == 0 and blocks[0][1] + blocks[1][1] == A.nrow and blocks[1][1] > 0
        p.execute([Bd, Bd], [Cd[r0:r0 + rc] for r0, rc in blocks])
        p.execute([Bd, Bd], [Ce[r0:r0 + rc] for r0, rc in blocks],
                  epilogues=[T.Epilogue(row_scale=scale[r0:r0 + rc]) for r0, rc in blocks])
        p.sync_check()
        st = p.stats
    if dt == "f16":
        assert st["tc_windows"] >= 10 and st["residue_nnz"] > 0
    ref = reference(A, B, dt)
    tol = TOL_TC if st["tc_nnz"] else TOL_CORE
    assert oracle.rel_l2(Cd.cpu().numpy(), ref) <= tol
    assert oracle.rel_l2(Ce.cpu().numpy(), ref * scale.cpu().numpy()[:, None]) <= tol
    # One plan per rank (the torchrun form) gives the same blocks.
    for r, (r0, rc) in enumerate(blocks):
        Cr = torch.empty((rc, N), device="cuda")
        with T.Plan(A, N, dt, rank=r, world=2, device=0, split="rows") as q:
            assert q.shard_rows(0) == (r0, rc)
            q.execute1(Bd, Cr)
            q.sync_check()
        torch.testing.assert_close(Cr, Cd[r0:r0 + rc], rtol=0, atol=0)


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_2d_plan_on_one_device(dt):
    """A 2 x 2 grid of shards placed on cuda:0: shard s writes row block s // 2 of
    column block s % 2; the per-rank form gives the same blocks."""
    A = _vstack(T.gen_uniform(256, 4096, 0.3, 1), T.gen_rmat(12, 60000, kind="gcn", seed=9))
    N = 96
    B = T.gen_dense(A.ncol, N, 4, "f32")
    Bd = torch.from_numpy(B).to(_torch_dt(dt)).cuda()
    Cd = torch.full((A.nrow, N), float("nan"), device="cuda")
    with T.Plan(A, N, dt, devices=[0, 0, 0, 0], split="2d", grid=(2, 2)) as p:
        blocks = [(p.shard_rows(s), p.shard(s)[1:]) for s in range(4)]
        p.execute([Bd[:, c0:c0 + cc] for _, (c0, cc) in blocks],
                  [Cd[r0:r0 + rc, c0:c0 + cc] for (r0, rc), (c0, cc) in blocks])
        p.sync_check()
        st = p.stats
    assert sorted(r for (r, _), _ in blocks) == [0, 0, blocks[2][0][0], blocks[2][0][0]]
    tol = TOL_TC if st["tc_nnz"] else TOL_CORE
    assert oracle.rel_l2(Cd.cpu().numpy(), reference(A, B, dt)) <= tol
    for s, ((r0, rc), (c0, cc)) in enumerate(blocks):
        Cr = torch.empty((rc, cc), device="cuda")
        with T.Plan(A, N, dt, rank=s, device=0, split="2d", grid=(2, 2)) as q:
            q.execute1(Bd[:, c0:c0 + cc], Cr)
            q.sync_check()
        torch.testing.assert_close(Cr, Cd[r0:r0 + rc, c0:c0 + cc], rtol=0, atol=0)


def test_tensor_core_wait_time_out_is_reported_and_recoverable():
    """A wait that nothing will satisfy ends in TCASPMM_ERR_TIMEOUT, not a hang, and the GPU stays usable."""
    import ctypes

    fn = T.lib.tcaspmm_selftest_tc_timeout
    fn.argtypes = [ctypes.c_int, ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_int)]
    fn.restype = ctypes.c_int
    code = ctypes.c_int(0)
    status = fn(0, 200_000_000, ctypes.byref(code))  # ~0.1 s of SM clocks
    assert status == T.Status.TIMEOUT, T.last_error()
    assert code.value & 2  # the MMA thread's wait on the producer ran out
    check(T.gen_uniform(256, 256, 0.4, 14), 128, "f16")  # the context still works


def _window_union_matrix(unions, K, seed=21, drop=0.1):
    """One 32-row window per column union; each row keeps ~90% of its window's columns, small integer values."""
    rng = np.random.default_rng(seed)
    rp, cols, vals = [0], [], []
    for u in unions:
        u = np.asarray(u, np.int32)
        for r in range(32):
            keep = u[rng.random(u.size) >= drop] if r else u  # row 0 carries the whole union
            cols.append(keep)
            vals.append(rng.integers(-3, 4, keep.size).astype(np.float32))
            rp.append(rp[-1] + keep.size)
    return T.CSR(32 * len(unions), K, np.asarray(rp, np.int64), np.concatenate(cols), np.concatenate(vals))


@pytest.mark.parametrize("gather_tma", ["1", "0"])
def test_tensor_core_stage_shapes_bit_exact(gather_tma, monkeypatch):
    """Every producer form: 64-row boxes, 16-row boxes, gather4 tiles, partial stages,
    index refills past 32 tiles, a padded last tile whose span looks like 16
    consecutive rows ({.., 40, 55, 55, ..}) but is not, and windows whose columns
    are one consecutive run (loaded without tile indices, boxes reaching past K);
    gathered 16-bit tiles by TMA gather4 (default) and by cp.async."""
    monkeypatch.setenv("TCASPMM_GATHER_TMA", gather_tma)
    K = 2048
    unions = [
        list(range(32)) + [40, 55],                                   # padded tile of span 15
        list(range(64)) + [70, 71, 72, 73] + list(range(100, 116)),   # one 64-row stage, then gather + padded
        [c for c in range(65) if c != 30],                            # span 64 over 64 columns: per-tile forms
        list(range(0, K, 2)),                                         # 64 gathered tiles, two index refills
        list(range(1024)),                                            # 16 stages of 64 consecutive rows
        list(range(1000, 1016)) + list(range(1017, 1033)),            # 16-row box, then a 16-span gap tile
        list(range(100, 140)),                                        # one run: 3 tiles, padded, no indices
        list(range(K - 20, K)),                                       # one run ending at K: boxes past K
    ]
    A = _window_union_matrix(unions, K)
    B = np.round(T.gen_dense(K, 256, 5, "f32") * 4).astype(np.float32)
    for dt in ("f16", "bf16", "tf32"):
        for N in (256, 136):
            out, st = run(A, B[:, :N], dt)
            assert st["tc_windows"] == len(unions) and st["tc_nnz"] == st["nnz"], st
            np.testing.assert_array_equal(out, reference(A, B[:, :N], dt).astype(np.float32))


@pytest.mark.parametrize("dt,gather_tma", [("f16", "1"), ("f16", "0"), ("tf32", "1")])
def test_gathered_tile_index_chunks_bit_exact(dt, gather_tma, monkeypatch):
    """Gathered tile chains long enough for many 16-tile index chunks, walked from a
    rotated first stage (work items run by decreasing tile count, item i starting at
    stage i mod its stages): chunk prefetches across the wrap from the last stage to
    the first, chains that start inside a chunk and come back to it, and a one-chunk
    chain that wraps within its chunk."""
    monkeypatch.setenv("TCASPMM_GATHER_TMA", gather_tma)
    K = 8192
    unions = [
        list(range(0, 200 * 32, 2)),      # 200 tiles (50 f16 stages), item 0: first stage 0
        list(range(0, 12 * 48, 3)),       # 12 tiles, item 4: one chunk, starts at stage 1, wraps in it
        list(range(1, 150 * 32, 2)),      # 150 tiles, item 1: starts one stage into its first chunk
        list(range(7, 70 * 32 + 7, 2)),   # 70 tiles, item 2: starts two stages in
        list(range(0, 17 * 32, 2)),       # 17 tiles, item 3: chunk 0 from stage 3, chunk 1, chunk 0 again
    ]
    A = _window_union_matrix(unions, K, seed=27)
    B = np.round(T.gen_dense(K, 128, 6, "f32") * 4).astype(np.float32)
    out, st = run(A, B, dt)
    assert st["tc_windows"] == len(unions) and st["tc_nnz"] == st["nnz"], st
    np.testing.assert_array_equal(out, reference(A, B, dt).astype(np.float32))


# ---------------------------------------------------- gathered windows (long rows)
@pytest.mark.parametrize("dt", ["f16", "bf16", "tf32"])
@pytest.mark.parametrize("N", [128, 64, 256, 200])
@pytest.mark.parametrize("split", ["128", "7"])
def test_gathered_windows_of_long_rows(dt, N, split, monkeypatch):
    """Long rows of a power-law graph grouped by length into tensor-core windows; their
    tile chains cut into parts of `split` tiles (reduced in part order), C written
    through the windows' row lists; N = 200 leaves a partial column block."""
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    monkeypatch.setenv("TCASPMM_SPLIT_TILES", split)
    A = T.gen_rmat(15, 400000, kind="gcn", seed=2)
    out, st = check(A, N, dt, seed=5)
    assert st["tc_gathered_windows"] > 0 and st["tc_tasks"] > st["tc_windows"], st


@pytest.mark.parametrize("gather_tma", ["1", "0"])
def test_gathered_windows_integer_values_bit_exact(gather_tma, monkeypatch):
    """Integer A and B small enough that every fp32 sum is exact: tiles, split parts
    and the fixed-order reduction must reproduce the oracle bit for bit (tiles fetched
    by TMA gather4 and by cp.async)."""
    monkeypatch.setenv("TCASPMM_GATHER_TMA", gather_tma)
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    monkeypatch.setenv("TCASPMM_SPLIT_TILES", "5")
    A = T.gen_rmat(13, 120000, kind="gcn", seed=9)
    g = np.random.default_rng(9)
    A = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, g.integers(-3, 4, A.nnz).astype(np.float32))
    B = g.integers(-4, 5, (A.ncol, 128)).astype(np.float32)
    out, st = run(A, B, "f16")
    assert st["tc_gathered_windows"] > 0, st
    np.testing.assert_array_equal(out, reference(A, B, "f16"))


def test_gathered_windows_are_deterministic(monkeypatch):
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    monkeypatch.setenv("TCASPMM_SPLIT_TILES", "3")
    A = T.gen_rmat(14, 200000, kind="gcn", seed=6)
    B = T.gen_dense(A.ncol, 128, 2, "f32")
    a, st = run(A, B, "bf16")
    b, _ = run(A, B, "bf16")
    assert st["tc_gathered_windows"] > 0
    np.testing.assert_array_equal(a, b)


def test_gathered_windows_with_unaligned_b_fall_back(monkeypatch):
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    A = T.gen_rmat(14, 200000, kind="gcn", seed=6)
    B = T.gen_dense(A.ncol, 64, 2, "f32")
    out, st = run(A, B, "f16", ldb_pad=3)  # ldb = 67 halves: rows not 16-byte aligned
    assert st["tc_gathered_windows"] > 0
    assert oracle.rel_l2(out, reference(A, B, "f16")) <= TOL_CORE


def test_gathered_windows_switched_off_gives_the_same_product(monkeypatch):
    A = T.gen_rmat(14, 200000, kind="gcn", seed=7)
    B = T.gen_dense(A.ncol, 128, 4, "f32")
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "1")
    on, st_on = run(A, B, "f16")
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "0")
    off, st_off = run(A, B, "f16")
    assert st_on["tc_gathered_windows"] > 0 and st_off["tc_gathered_windows"] == 0
    ref = reference(A, B, "f16")
    assert oracle.rel_l2(on, ref) <= TOL_TC and oracle.rel_l2(off, ref) <= TOL_TC


@pytest.mark.parametrize("K", [310, 316, 63 * 5])
def test_dense_window_whose_last_stage_runs_past_b(K):
    """Windows whose columns are one consecutive run: with K = 310 the run has 20 tiles,
    so its last four-tile stage starts 54 rows before B ends; it is fetched tile by
    tile rather than as one 64-row box past the last row."""
    A = T.gen_uniform(256, K, 0.5, 12)
    _, st = check(A, 128, "f16")
    assert st["tc_windows"] > 0
    g = np.random.default_rng(K)
    Ai = T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, g.integers(-3, 4, A.nnz).astype(np.float32))
    B = g.integers(-4, 5, (K, 128)).astype(np.float32)
    out, _ = run(Ai, B, "f16")
    np.testing.assert_array_equal(out, reference(Ai, B, "f16"))


@pytest.mark.parametrize("gather_tma", ["1", "0"])
def test_cta_running_a_tma_window_then_a_gathered_one(gather_tma, monkeypatch):
    """More work items than resident CTAs, so each CTA runs several: the first 320
    windows are one consecutive column run (tiles fetched by TMA boxes), the next 320
    skip four columns (tiles gathered by TMA gather4, or by cp.async).  Windows have
    equal tile counts, so a CTA's first item is a TMA-box window and a later one a
    gathered one -- the hand-over between producer forms, integer values bit-exact."""
    monkeypatch.setenv("TCASPMM_GATHER_TMA", gather_tma)
    g = np.random.default_rng(31)
    K, nd = 256, 320 * 32
    cols, rp = [], [0]
    keep_cols = np.setdiff1d(np.arange(K), np.arange(100, 104))
    for r in range(2 * nd):
        c = np.arange(K) if r < nd else np.sort(g.choice(keep_cols, 150, replace=False))
        if r >= nd and r % 32 == 0:
            c = keep_cols  # the window's union: every column but 100-103
        cols.append(c.astype(np.int32))
        rp.append(rp[-1] + c.size)
    col = np.concatenate(cols)
    A = T.CSR(2 * nd, K, np.asarray(rp, np.int64), col, g.integers(-3, 4, col.size).astype(np.float32))
    B = g.integers(-4, 5, (K, 128)).astype(np.float32)
    out, st = run(A, B, "f16")
    assert st["tc_windows"] == 640 and st["tc_ctas_per_sm"] * 148 < 640, st
    np.testing.assert_array_equal(out, reference(A, B, "f16"))


@pytest.mark.parametrize("parts", ["2", "3", "5", "8"])
def test_consecutive_windows_cut_into_parts(parts, monkeypatch):
    """Consecutive windows cut into parts of their tile chain (reduced in part order),
    including parts that start 48 rows into a 64-row stage (K = 300, 5 parts) and a last
    window that is not one column run, so CTAs mix TMA and cp.async work items."""
    monkeypatch.setenv("TCASPMM_WINDOW_PARTS", parts)
    _, st = check(T.gen_uniform(1000, 300, 0.4, 11), 72, "f16")
    assert st["tc_tasks"] > st["tc_windows"] > 0
    _, st = check(T.gen_uniform(2048, 512, 0.3, 0), 256, "f16")
    assert st["tc_tasks"] == 64 * int(parts), st
