"""Host logic of libtcaspmm through the C-ABI (no GPU needed): exports, .smtx
I/O, dense->CSR, generators, the column partitioner and the schedule's
exact-cover invariant."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import spmm_b200 as T
from conftest import ROOT


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)) - {"sizeof"}


def test_library_exports_every_declared_symbol():
    core = ctypes.CDLL(T.LIB_PATH)
    base = ctypes.CDLL(T.BASELINES_PATH)
    missing = []
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        for name in _declared(header):
            if not any(hasattr(l, name) for l in (core, base)):
                missing.append((header, name))
    assert not missing, missing
    assert "our_spmm_balanced" in _declared("tcaspmm.h")


def test_cxx_twin_symbol_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", T.LIB_PATH], capture_output=True, text=True).stdout
    # void our_spmm_balanced(CSR *, half *, float *, int, int, int, int, double *) (src/our_spmm.cuh:4)
    assert "_Z17our_spmm_balancedP3CSRP6__halfPfiiiiPd" in out


def test_smtx_reader_matches_reference_loader(bundled, bundled_smtx_path):
    A = T.smtx_read(bundled_smtx_path)
    assert (A.nrow, A.ncol) == (int(bundled["M"]), int(bundled["K"]))
    np.testing.assert_array_equal(A.row_ptr, bundled["row_ptr"])
    np.testing.assert_array_equal(A.col, bundled["col"])
    assert A.val is None  # pattern file: every value 1.0
    A.validate()


def test_smtx_roundtrip_with_values(tmp_path):
    A = T.gen_uniform(40, 70, 0.2, seed=3)
    p = str(tmp_path / "a.smtx")
    T.smtx_write(p, A)
    B = T.smtx_read(p)
    np.testing.assert_array_equal(A.row_ptr, B.row_ptr)
    np.testing.assert_array_equal(A.col, B.col)
    np.testing.assert_array_equal(A.val, B.val)
    # pattern write removes a stale sidecar
    T.smtx_write(p, T.CSR(A.nrow, A.ncol, A.row_ptr, A.col, None))
    assert T.smtx_read(p).val is None


def test_smtx_unsorted_and_repeated_columns_collapse_like_reference(tmp_path):
    # The reference scatters 1.0 into a dense matrix, so order and repeats vanish.
    p = tmp_path / "u.smtx"
    p.write_text("3, 5, 6\n0 3 3 6\n4 1 1\n\n0 2 0\n")
    A = T.smtx_read(str(p))
    np.testing.assert_array_equal(A.row_ptr, [0, 2, 2, 4])
    np.testing.assert_array_equal(A.col, [1, 4, 0, 2])


@pytest.mark.parametrize("text,status", [
    ("3 5 6\n0 1 2 3\n0 1 2\n", T.Status.FORMAT),          # header without commas
    ("2, 4, 3\n0 1\n0 1 2\n", T.Status.FORMAT),            # too few row offsets
    ("2, 4, 3\n0 1 3\n0 1\n", T.Status.FORMAT),            # too few columns
    ("2, 4, 2\n0 1 2\n0 9\n", T.Status.FORMAT),            # column out of range
    ("2, 4, 2\n0 2 1\n0 1\n", T.Status.FORMAT),            # decreasing offsets
    ("2, 4, 2\n0 1 2\n0 x\n", T.Status.FORMAT),            # bad token
    ("", T.Status.FORMAT),                                 # empty file
])
def test_smtx_malformed_inputs_are_rejected(tmp_path, text, status):
    p = tmp_path / "bad.smtx"
    p.write_text(text)
    with pytest.raises(T.TcaspmmError) as e:
        T.smtx_read(str(p))
    assert e.value.status == status


def test_smtx_missing_file_is_io_error(tmp_path):
    with pytest.raises(T.TcaspmmError) as e:
        T.smtx_read(str(tmp_path / "nope.smtx"))
    assert e.value.status == T.Status.IO


def test_smtx_empty_matrix(tmp_path):
    p = tmp_path / "e.smtx"
    p.write_text("0, 7, 0\n0\n")
    A = T.smtx_read(str(p))
    assert (A.nrow, A.ncol, A.nnz) == (0, 7, 0)


def test_dense_to_csr_matches_reference(small_cases):
    for c in small_cases:
        A = T.convert_dense_to_csr(c["dense"])
        np.testing.assert_array_equal(A.row_ptr, c["row_ptr"])
        np.testing.assert_array_equal(A.col, c["col"])
        np.testing.assert_array_equal(A.val.astype(np.float16).view(np.uint16), c["val"].view(np.uint16))


def test_dense_to_csr_drops_signed_zeros():
    d = np.array([[0.0, -0.0, 1.5], [-2.0, 0.0, 0.0]], np.float16)
    A = T.convert_dense_to_csr(d)
    np.testing.assert_array_equal(A.row_ptr, [0, 1, 2])
    np.testing.assert_array_equal(A.col, [2, 0])


def test_generators_are_seeded_and_valid():
    a1, a2 = T.gen_uniform(64, 80, 0.3, 1), T.gen_uniform(64, 80, 0.3, 1)
    np.testing.assert_array_equal(a1.col, a2.col)
    np.testing.assert_array_equal(a1.val, a2.val)
    assert T.gen_uniform(64, 80, 0.3, 2).col.shape != a1.col.shape or not np.array_equal(
        T.gen_uniform(64, 80, 0.3, 2).col, a1.col)
    assert abs(a1.nnz / (64 * 80) - 0.3) < 0.05
    for A in (a1, T.gen_magnitude(64, 128, 0.9, 0), T.gen_rmat(10, 4000, kind="gcn"),
              T.gen_rmat(10, 4000, kind="sage"), T.gen_skew(5000, 4, 1000, 3.0)):
        A.validate()
    m = T.gen_magnitude(64, 128, 0.9, 0)
    assert m.nnz == round(0.1 * 64 * 128)
    s = T.gen_skew(5000, 4, 1000, 3.0)
    lens = np.diff(s.row_ptr)
    assert sorted(lens)[-4:] == [1000] * 4
    g = T.gen_rmat(10, 4000, kind="gcn")
    assert np.all(np.diff(g.row_ptr) >= 1)  # self-loops
    B = T.gen_dense(3, 5, 7, "f32")
    np.testing.assert_array_equal(B, T.gen_dense(3, 5, 7, "f32"))
    np.testing.assert_array_equal(T.gen_dense(3, 5, 7, "f16"), B.astype(np.float16))


def test_generators_do_not_depend_on_thread_count():
    code = ("import sys; sys.path.insert(0, %r); import spmm_b200 as T, hashlib;"
            "A = T.gen_rmat(12, 20000, kind='gcn', seed=5);"
            "print(hashlib.sha1(A.col.tobytes() + A.val.tobytes()).hexdigest())") % ROOT
    outs = set()
    for n in ("1", "3"):
        env = dict(os.environ, OMP_NUM_THREADS=n)
        outs.add(subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                                check=True).stdout)
    assert len(outs) == 1


@pytest.mark.parametrize("N,dt,world", [(128, "f32", 8), (128, "f16", 8), (256, "f16", 3), (64, "f16", 8),
                                        (7, "f32", 2), (0, "f32", 4), (1000, "bf16", 5)])
def test_partition_columns_tile_n_disjointly(N, dt, world):
    vec = 4 if dt == "f32" else 8
    blocks = [T.partition_columns(N, dt, world, r) for r in range(world)]
    covered = np.zeros(N, int)
    for b, c in blocks:
        assert b % vec == 0 or c == 0
        covered[b:b + c] += 1
    assert np.all(covered == 1)


@pytest.mark.parametrize("parts", [1, 2, 3, 8, 5000])
def test_partition_rows_covers_rows_in_balanced_blocks(parts):
    A = T.gen_rmat(12, 40000, kind="gcn", seed=3)
    rb = T.partition_rows(A, parts)
    assert rb[0] == 0 and rb[-1] == A.nrow and np.all(np.diff(rb) >= 0)
    cost = np.diff(A.row_ptr[rb] + 2 * rb)
    row_cost = np.diff(A.row_ptr) + 2
    # Each block is within one row's cost of the ideal share.
    assert np.all(np.abs(cost - cost.sum() / parts) <= row_cost.max() + 1)
    assert np.array_equal(T.partition_rows(A, parts), rb)  # deterministic


@pytest.mark.parametrize("N", [4, 16, 128])
@pytest.mark.parametrize("env", [{}, {"TCASPMM_BUDGET_MAX": "64"}, {"TCASPMM_BUDGET_MAX": "4096"},
                                 {"TCASPMM_WARPS_PER_SM": "4", "TCASPMM_BUDGET_MIN": "16"},
                                 {"TCASPMM_WARPS_PER_SM": "128"}])
def test_schedule_coverage_at_narrow_widths_and_tuning_values(N, env, monkeypatch):
    """The residue schedule covers each nonzero exactly once whatever the lane-group
    count per warp (N = 4 / 16 / 128 fp32: 32 / 8 / 1 groups) and the tuning variables."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    A = T.gen_rmat(13, 60000, kind="gcn", seed=3)
    cover, _, st = T.schedule_coverage(A, N, "f32")
    assert np.all(cover == 1), (np.bincount(cover), st)
    assert st["residue_nnz"] == A.nnz


@pytest.mark.parametrize("env", [{"TCASPMM_BUDGET_MAX": "0"}, {"TCASPMM_BUDGET_MAX": "-5"},
                                 {"TCASPMM_BUDGET_MAX": "abc"}, {"TCASPMM_BUDGET_MAX": "12x"},
                                 {"TCASPMM_BUDGET_MIN": "0"}, {"TCASPMM_BUDGET_MIN": "-1"},
                                 {"TCASPMM_WARPS_PER_SM": "0"}, {"TCASPMM_WARPS_PER_SM": "-3"},
                                 {"TCASPMM_BUDGET_MAX": "99999999999999999999"}])
@pytest.mark.parametrize("N", [4, 128])
def test_out_of_range_tuning_values_are_clamped(env, N, monkeypatch):
    """Zero, negative, overflowing or non-numeric tuning values must neither crash plan
    creation (a zero budget used to divide by zero) nor drop a nonzero."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    A = T.gen_skew(20000, 4, 5000, 3.0, seed=5)  # hub rows exercise the segment split
    cover, _, st = T.schedule_coverage(A, N, "f32")
    assert np.all(cover == 1), (np.bincount(cover), st)
    assert st["residue_nnz"] == A.nnz


def test_partition_rows_edge_cases():
    empty = T.CSR(0, 5, np.zeros(1, np.int64), np.zeros(0, np.int32), np.zeros(0, np.float32))
    assert list(T.partition_rows(empty, 3)) == [0, 0, 0, 0]
    one = T.CSR(1, 4, np.array([0, 2], np.int64), np.array([0, 3], np.int32), np.ones(2, np.float32))
    rb = T.partition_rows(one, 4)
    assert rb[0] == 0 and rb[-1] == 1 and np.all(np.diff(rb) >= 0)
    with pytest.raises(T.TcaspmmError):
        T.partition_rows(one, 0)


@pytest.mark.parametrize("case", ["c1_f16", "c1_f32", "sweep_mag", "skew", "gcn", "bundled", "empty_rows", "tiny"])
def test_schedule_covers_every_nonzero_exactly_once(case, bundled):
    if case == "c1_f16":
        A, N, dt = T.gen_uniform(2048, 512, 0.3, 0), 256, "f16"
    elif case == "c1_f32":
        A, N, dt = T.gen_uniform(2048, 512, 0.3, 0), 256, "f32"
    elif case == "sweep_mag":
        A, N, dt = T.gen_magnitude(512, 2048, 0.9, 0), 128, "bf16"
    elif case == "skew":
        A, N, dt = T.gen_skew(200000, 8, 20000, 3.0), 64, "f16"
    elif case == "gcn":
        A, N, dt = T.gen_rmat(14, 200000, kind="gcn"), 128, "f32"
    elif case == "bundled":
        A = T.CSR(int(bundled["M"]), int(bundled["K"]), bundled["row_ptr"], bundled["col"], None)
        N, dt = 256, "f16"
    elif case == "empty_rows":
        A, N, dt = T.CSR(100, 10, np.zeros(101, np.int64), np.zeros(0, np.int32), None), 16, "f16"
    else:
        A, N, dt = T.CSR(1, 1, np.array([0, 1]), np.array([0]), np.array([2.0], np.float32)), 1, "f32"
    cover, kind, st = T.schedule_coverage(A, N, dt)
    assert np.all(cover == 1), (np.bincount(cover), st)
    assert st["tc_nnz"] + st["residue_nnz"] == A.nnz
    if case == "c1_f16":
        assert st["tc_windows"] > 0 and np.all(kind == 3)
    if case == "c1_f32":
        assert st["tc_windows"] == 0
    if case == "skew":
        assert st["long_rows"] == 8 and np.any(kind == 2)


def test_plan_without_device_reports_no_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    A = T.gen_uniform(8, 8, 0.5, 0)
    with pytest.raises(T.TcaspmmError) as e:
        T.Plan(A, 8, "f32")
    assert e.value.status in (T.Status.NO_DEVICE, T.Status.CUDA)


def test_reference_entry_without_device_returns_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rp = np.array([0, 1], np.int32)
    with pytest.raises(T.TcaspmmError):
        T.our_spmm_balanced(rp, np.array([0], np.int32), np.array([1.0], np.float16), np.ones((1, 8), np.float16),
                            np.zeros(8, np.float32), 1, 8, 1, 1)


def test_reference_entry_rejects_mismatched_shapes():
    rp = np.array([0, 1], np.int32)
    with pytest.raises(T.TcaspmmError) as e:
        T.our_spmm_balanced(rp, np.array([0], np.int32), np.array([1.0], np.float16), np.ones((1, 8), np.float16),
                            np.zeros(16, np.float32), 2, 8, 1, 1)
    assert e.value.status == T.Status.INVALID_ARG


def test_matrix_market_reader(tmp_path):
    p = tmp_path / "a.mtx"
    p.write_text("%%MatrixMarket matrix coordinate real general\n% comment\n3 4 5\n1 2 1.5\n3 1 -2\n1 1 4\n3 4 7\n1 2 0.5\n")
    A = T.mtx_read(str(p))
    np.testing.assert_array_equal(A.row_ptr, [0, 2, 2, 4])
    np.testing.assert_array_equal(A.col, [0, 1, 0, 3])
    np.testing.assert_allclose(A.val, [4.0, 2.0, -2.0, 7.0])  # repeated (1,2) entries summed
    p.write_text("%%MatrixMarket matrix coordinate pattern symmetric\n3 3 3\n1 1\n2 1\n3 2\n")
    S = T.mtx_read(str(p))
    assert S.val is None
    np.testing.assert_array_equal(S.to_scipy().toarray(), [[1, 1, 0], [1, 0, 1], [0, 1, 0]])
    p.write_text("2 2 1\n0 1 3.0\n")  # no banner, 0-based as the reference reader's default
    Z = T.mtx_read(str(p), zero_based=True)
    np.testing.assert_array_equal(Z.to_scipy().toarray(), [[0, 3], [0, 0]])
    p.write_text("2 2 2\n1 1 1\n")
    with pytest.raises(T.TcaspmmError):
        T.mtx_read(str(p))


def test_binary_csr_roundtrip(tmp_path):
    for A in (T.gen_rmat(10, 3000, kind="gcn"), T.CSR(4, 3, np.array([0, 1, 1, 1, 2]), np.array([2, 0]), None)):
        p = str(tmp_path / "a.csrb")
        T.csrbin_write(p, A)
        B = T.csrbin_read(p)
        np.testing.assert_array_equal(A.row_ptr, B.row_ptr)
        np.testing.assert_array_equal(A.col, B.col)
        assert (A.val is None) == (B.val is None)
        if A.val is not None:
            np.testing.assert_array_equal(A.val, B.val)
    with open(p, "ab") as f:
        f.write(b"x")
    with pytest.raises(T.TcaspmmError):
        T.csrbin_read(p)


@pytest.mark.parametrize("case,dt,N", [("gcn", "f16", 128), ("gcn", "bf16", 64), ("gcn", "tf32", 128),
                                       ("sage", "f16", 256), ("skew", "f16", 64)])
def test_gathered_windows_cover_long_rows_exactly_once(case, dt, N):
    """Long rows grouped by length into tensor-core windows (row lists): every nonzero
    is still covered exactly once, and the windows appear in the stats."""
    os.environ["TCASPMM_HUB_WINDOWS"] = "1"
    if case == "gcn":
        A = T.gen_rmat(15, 400000, kind="gcn", seed=2)
    elif case == "sage":
        A = T.gen_rmat(15, 400000, kind="sage", seed=3)
    else:
        A = T.gen_skew(100000, 16, 20000, 3.0, seed=4)
    try:
        cover, kind, st = T.schedule_coverage(A, N, dt)
    finally:
        del os.environ["TCASPMM_HUB_WINDOWS"]
    assert np.all(cover == 1), np.bincount(cover)
    assert st["tc_gathered_windows"] > 0, st
    assert st["tc_nnz"] + st["residue_nnz"] == A.nnz
    assert (kind == 3).sum() == st["tc_nnz"]


def test_gathered_windows_are_off_unless_asked_for(monkeypatch):
    A = T.gen_rmat(15, 400000, kind="gcn", seed=2)
    monkeypatch.delenv("TCASPMM_HUB_WINDOWS", raising=False)
    cover, _, st = T.schedule_coverage(A, 128, "f16")
    assert np.all(cover == 1) and st["tc_gathered_windows"] == 0
    monkeypatch.setenv("TCASPMM_HUB_WINDOWS", "0")
    assert T.schedule_coverage(A, 128, "f16")[2]["tc_gathered_windows"] == 0


@pytest.mark.parametrize("mirror,ctype", [("_Stats", "tcaspmm_plan_stats"), ("_CSR", "tcaspmm_csr"),
                                           ("_RefCSR", "tcaspmm_ref_csr"), ("_Epilogue", "tcaspmm_epilogue")])
def test_ctypes_structs_match_the_header(mirror, ctype, tmp_path):
    """Each ctypes mirror of a header struct has the header's size and field offsets
    (a field added on one side only would make the library read or write past the
    caller's buffer)."""
    import shutil

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    cls = getattr(T, mirror)
    fields = [name for name, _ in cls._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"tcaspmm.h\"\nint main(void) {\n"
                   f"  printf(\"%zu\\n\", sizeof({ctype}));\n"
                   + "".join(f"  printf(\"%zu\\n\", offsetof({ctype}, {f}));\n" for f in fields)
                   + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(cls)
    assert out[1:] == [getattr(cls, f).offset for f in fields]
