"""CPU oracle for C = A @ B (CSR A, dense row-major B) -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline and
``--impl reference`` legs may import this package, and only as the checker or
the timed CPU baseline.  The product (spmm_b200/) never imports it.

``liboracle.so`` is built from oracle.c (see its header for the reference
lines it restates); ``_ref/libref_host.so`` wraps the reference's own host code
and exists only where the reference tree was available at build time.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_host.so")

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = C.CDLL(LIB)
        vp, i64 = C.c_void_p, C.c_int64
        _lib.oracle_spmm_f64.argtypes = [i64, i64, vp, vp, vp, vp, i64, vp, i64]
        _lib.oracle_spmm_f32.argtypes = [i64, i64, vp, vp, vp, vp, i64, vp, i64, C.c_int]
        _lib.oracle_spmm_f32_rows.argtypes = [i64, vp, i64, vp, vp, vp, vp, i64, vp, C.c_int]
        _lib.oracle_max_threads.restype = C.c_int
        _lib.oracle_smtx_header.argtypes = [C.c_char_p, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]
        _lib.oracle_smtx_read.argtypes = [C.c_char_p, i64, i64, vp, vp]
    return _lib


def _arrays(row_ptr, col, val, B):
    rp = np.ascontiguousarray(row_ptr, dtype=np.int64)
    ci = np.ascontiguousarray(col, dtype=np.int32)
    va = np.ascontiguousarray(val, dtype=np.float32)
    Bf = np.ascontiguousarray(B, dtype=np.float32)
    return rp, ci, va, Bf


def spmm_f64(row_ptr, col, val, B) -> np.ndarray:
    """fp64 C = A @ B with inputs already rounded to the path's dtype (widened to float32)."""
    rp, ci, va, Bf = _arrays(row_ptr, col, val, B)
    M, N = rp.shape[0] - 1, Bf.shape[1]
    out = np.empty((M, N), dtype=np.float64)
    lib().oracle_spmm_f64(M, N, rp.ctypes.data, ci.ctypes.data, va.ctypes.data, Bf.ctypes.data, N,
                          out.ctypes.data, N)
    return out


def spmm_f32(row_ptr, col, val, B, threads: int = 0) -> np.ndarray:
    """fp32 OpenMP CSR loop (the CPU baseline)."""
    rp, ci, va, Bf = _arrays(row_ptr, col, val, B)
    M, N = rp.shape[0] - 1, Bf.shape[1]
    out = np.empty((M, N), dtype=np.float32)
    lib().oracle_spmm_f32(M, N, rp.ctypes.data, ci.ctypes.data, va.ctypes.data, Bf.ctypes.data, N,
                          out.ctypes.data, N, threads)
    return out


def spmm_f32_rows(rows, row_ptr, col, val, B, threads: int = 0) -> np.ndarray:
    """fp32 CSR loop over a subset of rows (bounded CPU-baseline sample)."""
    rp, ci, va, Bf = _arrays(row_ptr, col, val, B)
    rw = np.ascontiguousarray(rows, dtype=np.int64)
    N = Bf.shape[1]
    out = np.empty((rw.shape[0], N), dtype=np.float32)
    lib().oracle_spmm_f32_rows(rw.shape[0], rw.ctypes.data, N, rp.ctypes.data, ci.ctypes.data, va.ctypes.data,
                               Bf.ctypes.data, N, out.ctypes.data, threads)
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def smtx_read(path: str):
    """Pattern .smtx -> (M, K, row_ptr int64, col int32), restating src/file_input.cu:135-193."""
    M, K, Z = C.c_int64(), C.c_int64(), C.c_int64()
    rc = lib().oracle_smtx_header(os.fsencode(path), C.byref(M), C.byref(K), C.byref(Z))
    if rc != 0:
        raise ValueError(f"oracle: bad .smtx header ({rc})")
    rp = np.empty(M.value + 1, np.int64)
    col = np.empty(max(Z.value, 1), np.int32)
    rc = lib().oracle_smtx_read(os.fsencode(path), M.value, Z.value, rp.ctypes.data, col.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle: bad .smtx body ({rc})")
    return M.value, K.value, rp, col[: Z.value]


def rel_l2(x: np.ndarray, ref: np.ndarray) -> float:
    """||x - ref||_2 / ||ref||_2 in fp64 (0 when both are zero)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    if den == 0.0:
        return 0.0 if num == 0.0 else float("inf")
    return float(num / den)
