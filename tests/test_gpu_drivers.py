"""The ./test command-line surface on a GPU (src/test.cu:29-88 of the reference).

* spmm_b200/bin/test: this library's driver, with the reference's CLI, timing lines
  and compare_mat validation against a dense cuBLAS gold; its C is also dumped and
  checked against the fp64 oracle here.
* oracle/_ref/ref_test_dropin: the reference's own, unmodified test.cu (and its
  cuBLAS / cuSPARSE baselines) compiled from the reference sources and linked against
  libtcaspmm.so in place of src/our_spmm.cu -- the drop-in claim run end to end.  It
  exists only where the reference tree was present at build time.
"""
import json
import os
import re
import subprocess

import numpy as np
import pytest

import oracle
import spmm_b200 as T

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
REF_DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_test_dropin")


def _run(cmd, timeout=300):
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    assert p.returncode == 0, f"{cmd} exited {p.returncode}\n{p.stdout}\n{p.stderr}"
    return p.stdout


def _json_line(out):
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out
    return json.loads(lines[0])


def _round(x, dt):
    import torch

    t = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(t).float().numpy()


def _check_dump(path, A, N, dt, seed, tol):
    C = np.fromfile(path, dtype=np.float32).reshape(A.nrow, N)
    B = T.gen_dense(A.ncol, N, seed, dt)
    Bf = (B.astype(np.uint32) << 16).view(np.float32) if dt == "bf16" else B.astype(np.float32)
    ref = oracle.spmm_f64(A.row_ptr, A.col, _round(A.values(), dt), Bf)
    err = oracle.rel_l2(C, ref)
    assert err <= tol, err
    return err


@pytest.mark.parametrize("dt,N", [("f16", 256), ("f32", 64), ("bf16", 128)])
def test_driver_on_the_bundled_matrix(bundled_smtx_path, tmp_path, dt, N):
    dump = str(tmp_path / "C.bin")
    out = _run([T.TEST_DRIVER, bundled_smtx_path, "-n", str(N), "-d", dt, "-i", "3", "--dump", dump])
    assert "validation failed" not in out, out
    for line in ("GemmEx :", "cuSPARSE:", "our:", "preprocess "):
        assert line in out, out
    j = _json_line(out)
    assert j["ms"]["ours"] > 0 and j["ms"]["cusparse"] > 0 and j["ms"]["gemm_cublas"] > 0
    A = T.smtx_read(bundled_smtx_path)
    assert (j["M"], j["K"], j["nnz"]) == (A.nrow, A.ncol, A.nnz)
    _check_dump(dump, A, N, dt, 0, 1e-5 if j["tc_windows"] == 0 else 5e-3)


def test_driver_on_a_written_c1_matrix_with_values(tmp_path):
    """C1: the 2048 x 512 70%-sparse N(0,1) weight written as .smtx plus its .val
    companion, run through ./test at the reference's N = 256 in fp16."""
    A = T.gen_uniform(2048, 512, 0.3, 0)
    path = str(tmp_path / "c1.smtx")
    T.smtx_write(path, A)
    assert os.path.exists(path + ".val")
    dump = str(tmp_path / "C.bin")
    out = _run([T.TEST_DRIVER, path, "-d", "f16", "-i", "5", "--dump", dump])
    assert "validation failed" not in out, out
    j = _json_line(out)
    assert j["N"] == 256 and j["nnz"] == A.nnz and j["tc_windows"] > 0
    _check_dump(dump, A, 256, "f16", 0, 5e-3)


@pytest.mark.skipif(not os.path.exists(REF_DRIVER), reason="reference driver not built (no reference tree at build)")
def test_reference_driver_linked_against_this_library(bundled_smtx_path):
    """The reference's unmodified main(): GemmEx gold, its cuSPARSE call, then
    our_spmm_balanced -- which binds to this library -- validated with its own
    compare_mat.  No 'validation failed' line may appear for our entry point."""
    out = _run([REF_DRIVER, bundled_smtx_path])
    assert "validation failed (Our, balanced)" not in out, out
    assert "validation failed" not in out, out
    for line in ("Input file - ", "GemmEx :", "cuSPARSE:", "our:", "preprocess "):
        assert line in out, out
    # "our: \033[36m[<ms>] ms\033[0m": the timing sits between the colour codes.
    m = re.search(r"our:\s*(?:\x1b\[[0-9;]*m)?\[([0-9.eE+-]+)\] ms", out)
    assert m, out
    assert float(m.group(1)) > 0
