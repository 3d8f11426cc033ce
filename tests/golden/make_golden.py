"""Generate the golden fixtures from the reference's own host code.

Runs here, where the YaoLingF/SPMM tree is present: ``make -C oracle ref``
compiles the reference's src/file_input.cu and src/miscalleneous.cu into
oracle/_ref/libref_host.so, and this script calls, through ctypes,
  smtx_input_to_Dense + convert_dense_to_csr  (the reference loader), and
  naive_gemm                                   (its only CPU product of A and B).
The outputs pin oracle/oracle.c and the product's .smtx reader; tests read the
.npz files only (the reference tree is not needed at test time).

    python tests/golden/make_golden.py [--ref-src /path/to/reference/src]
"""
from __future__ import annotations

import argparse
import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
BUNDLED = "data/body_decoder_layer_2_ffn_conv1.smtx"


def load_ref(ref_src: str) -> C.CDLL:
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF_SRC={ref_src}"], check=True)
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_host.so"))
    ip, vp = C.POINTER(C.c_int), C.c_void_p
    lib.ref_smtx_to_csr.argtypes = [C.c_char_p, ip, ip, ip, ip, C.POINTER(ip), C.POINTER(ip),
                                    C.POINTER(C.POINTER(C.c_uint16))]
    lib.ref_dense_to_csr.argtypes = [vp, C.c_int, C.c_int, ip, C.POINTER(ip), C.POINTER(ip),
                                     C.POINTER(C.POINTER(C.c_uint16))]
    lib.ref_naive_gemm.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int]
    lib.ref_free.argtypes = [vp]
    return lib


def _take(lib, M, nnz, rp, col, val):
    out = (np.ctypeslib.as_array(rp, shape=(M + 1,)).copy(),
           np.ctypeslib.as_array(col, shape=(max(nnz, 1),))[:nnz].copy(),
           np.ctypeslib.as_array(val, shape=(max(nnz, 1),))[:nnz].copy())
    for p in (rp, col, val):
        lib.ref_free(C.cast(p, C.c_void_p))
    return out


def ref_smtx(lib, path):
    M, K, zh, zc = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    rp, col = C.POINTER(C.c_int)(), C.POINTER(C.c_int)()
    val = C.POINTER(C.c_uint16)()
    rc = lib.ref_smtx_to_csr(os.fsencode(path), C.byref(M), C.byref(K), C.byref(zh), C.byref(zc), C.byref(rp),
                             C.byref(col), C.byref(val))
    assert rc == 0, rc
    return (M.value, K.value, zh.value) + _take(lib, M.value, zc.value, rp, col, val)


def ref_dense_to_csr(lib, dense_f16):
    d = np.ascontiguousarray(dense_f16, dtype=np.float16)
    M, K = d.shape
    z = C.c_int()
    rp, col = C.POINTER(C.c_int)(), C.POINTER(C.c_int)()
    val = C.POINTER(C.c_uint16)()
    lib.ref_dense_to_csr(d.ctypes.data, M, K, C.byref(z), C.byref(rp), C.byref(col), C.byref(val))
    return _take(lib, M, z.value, rp, col, val)


def ref_gemm(lib, A_f16, B_f16):
    A = np.ascontiguousarray(A_f16, dtype=np.float16)
    B = np.ascontiguousarray(B_f16, dtype=np.float16)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.zeros((M, N), dtype=np.float32)
    lib.ref_naive_gemm(A.ctypes.data, B.ctypes.data, Cm.ctypes.data, M, N, K)
    return Cm


def dense_from_csr(M, K, rp, col, val_bits):
    A = np.zeros((M, K), dtype=np.float16)
    for i in range(M):
        A[i, col[rp[i]:rp[i + 1]]] = val_bits[rp[i]:rp[i + 1]].view(np.float16)
    return A


def main():
    ap = argparse.ArgumentParser()
    here = os.path.dirname(os.path.abspath(__file__))
    default_ref = os.environ.get("TCASPMM_REF_SRC") or os.path.abspath(
        os.path.join(here, "..", "..", "..", "reference", "src"))  # a reference checkout beside the repo
    ap.add_argument("--ref-src", default=default_ref)
    args = ap.parse_args()
    lib = load_ref(args.ref_src)

    # 1. The bundled matrix through the reference loader, times two B's.
    smtx_path = os.path.join(os.path.dirname(os.path.abspath(args.ref_src)), BUNDLED)
    M, K, nnz_header, rp, col, val = ref_smtx(lib, smtx_path)
    A = dense_from_csr(M, K, rp, col, val)
    N = 256  # src/test.cu:47
    kk, nn = np.meshgrid(np.arange(K), np.arange(N), indexing="ij")
    B_int = (((kk * 7 + nn * 13) % 9) - 4).astype(np.float16)        # small integers: fp32 sums are exact
    rng = np.random.default_rng(20241201)
    B_rand = rng.standard_normal((K, N)).astype(np.float16)
    with open(smtx_path, "rb") as f:
        smtx_text = np.frombuffer(f.read(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "bundled_smtx.npz"), M=M, K=K, N=N, nnz_header=nnz_header,
                        row_ptr=rp, col=col, val_bits=val, smtx_text=smtx_text,
                        B_int=B_int, C_int=ref_gemm(lib, A, B_int), B_rand=B_rand, C_rand=ref_gemm(lib, A, B_rand))

    # 2. Small dense matrices with zeros through convert_dense_to_csr + naive_gemm.
    cases = [(37, 53, 24, 0.3), (1, 1, 1, 1.0), (64, 16, 8, 0.05), (5, 300, 40, 0.5), (33, 70, 129, 0.2),
             (16, 16, 256, 0.0), (128, 96, 64, 0.7)]
    out = {}
    for t, (m, k, n, dens) in enumerate(cases):
        keep = rng.random((m, k)) < dens
        Ad = np.where(keep, rng.standard_normal((m, k)), 0.0).astype(np.float16)
        if t == 2:
            Ad[::3] = 0  # empty rows
        Bd = rng.standard_normal((k, n)).astype(np.float16)
        crp, ccol, cval = ref_dense_to_csr(lib, Ad)
        out[f"c{t}_shape"] = np.array([m, k, n])
        out[f"c{t}_dense"] = Ad
        out[f"c{t}_row_ptr"] = crp
        out[f"c{t}_col"] = ccol
        out[f"c{t}_val_bits"] = cval
        out[f"c{t}_B"] = Bd
        out[f"c{t}_C"] = ref_gemm(lib, Ad, Bd)
    out["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "small_csr.npz"), **out)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    sys.exit(main())
