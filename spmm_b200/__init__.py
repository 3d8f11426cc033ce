"""tcaspmm: B200-native SpMM, C = A @ B with CSR A and dense row-major B.

Python mirror of the reference surface of YaoLingF/SPMM (the .smtx loader,
``mat_format``, ``convert_dense_to_csr``, ``our_spmm_balanced``) over the C-ABI
library ``spmm_b200/lib/libtcaspmm.so``.  Every call goes through that library;
there is no Python or CPU fallback, and importing this module fails loudly when
the library has not been built (``python -c "import __graft_entry__ as g; g.build()"``
or ``make -C spmm_b200/csrc``).
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libtcaspmm.so")
BASELINES_PATH = os.path.join(LIB_DIR, "libtcaspmm_baselines.so")
TEST_DRIVER = os.path.join(_HERE, "bin", "test")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {os.path.join(_HERE, 'csrc')}`")
lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)


class Status(enum.IntEnum):
    OK = 0
    INVALID_ARG = 1
    IO = 2
    FORMAT = 3
    ALLOC = 4
    CUDA = 5
    UNSUPPORTED = 6
    TIMEOUT = 7
    NO_DEVICE = 8


class TcaspmmError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = Status(status)
        super().__init__(f"{self.status.name}: {message}")


class dtype(enum.IntEnum):
    f32 = 0
    f16 = 1
    bf16 = 2
    tf32 = 3  # fp32 storage; tensor-core windows multiply in TF32


class mat_format(enum.IntEnum):
    """Same members as the reference enum (src/mat_format.cuh:10-15)."""

    dense = 0
    csr = 1
    coo = 2


MATTYPE_STRING = ("DENSE", "CSR", "COO")

_NP_OF = {dtype.f32: np.float32, dtype.f16: np.float16, dtype.bf16: np.uint16, dtype.tf32: np.float32}


def as_dtype(d) -> dtype:
    if isinstance(d, dtype):
        return d
    if isinstance(d, str):
        return {"f32": dtype.f32, "fp32": dtype.f32, "float32": dtype.f32, "f16": dtype.f16, "fp16": dtype.f16,
                "float16": dtype.f16, "half": dtype.f16, "bf16": dtype.bf16, "bfloat16": dtype.bf16, "tf32": dtype.tf32}[d]
    try:
        import torch

        if isinstance(d, torch.dtype):
            return {torch.float32: dtype.f32, torch.float16: dtype.f16, torch.bfloat16: dtype.bf16}[d]
    except ImportError:  # pragma: no cover
        pass
    return dtype(int(d))


class _CSR(C.Structure):
    _fields_ = [("nrow", C.c_int64), ("ncol", C.c_int64), ("nnz", C.c_int64),
                ("row_ptr", C.POINTER(C.c_int64)), ("col_idx", C.POINTER(C.c_int32)),
                ("val", C.POINTER(C.c_float))]


class _RefCSR(C.Structure):
    _fields_ = [("nRow", C.c_int), ("nCol", C.c_int), ("nnz", C.c_int), ("row_offset", C.POINTER(C.c_int)),
                ("col_idx", C.POINTER(C.c_int)), ("value", C.POINTER(C.c_uint16))]


class _Stats(C.Structure):
    _fields_ = [("nrow", C.c_int64), ("ncol", C.c_int64), ("nnz", C.c_int64), ("ncols_total", C.c_int64),
                ("num_shards", C.c_int32), ("window_rows", C.c_int32), ("tc_windows", C.c_int64),
                ("tc_tiles", C.c_int64), ("tc_nnz", C.c_int64), ("residue_nnz", C.c_int64),
                ("residue_row_warps", C.c_int64), ("residue_segments", C.c_int64), ("long_rows", C.c_int64),
                ("preprocess_ms", C.c_double), ("upload_ms", C.c_double), ("device_bytes", C.c_int64),
                ("algorithmic_bytes", C.c_int64), ("tc_gathered_windows", C.c_int64), ("tc_tasks", C.c_int64),
                ("tc_ctas_per_sm", C.c_int64), ("tc_side_stream", C.c_int64)]

    def to_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class _Epilogue(C.Structure):
    _fields_ = [("row_scale", C.c_void_p), ("bias", C.c_void_p), ("relu", C.c_int), ("out_dtype", C.c_int)]


_vp, _i64, _i32 = C.c_void_p, C.c_int64, C.c_int32
_P = C.POINTER


def _sig(name, args, res=C.c_int):
    f = getattr(lib, name)
    f.argtypes = args
    f.restype = res
    return f


_sig("tcaspmm_status_string", [C.c_int], C.c_char_p)
_sig("tcaspmm_last_error", [], C.c_char_p)
_sig("tcaspmm_csr_alloc", [_i64, _i64, _i64, C.c_int, _P(_CSR)])
_sig("tcaspmm_csr_free", [_P(_CSR)])
_sig("tcaspmm_csr_validate", [_P(_CSR)])
_sig("tcaspmm_smtx_read", [C.c_char_p, _P(_CSR)])
_sig("tcaspmm_smtx_write", [C.c_char_p, _P(_CSR)])
_sig("tcaspmm_dense_to_csr", [_vp, _i64, _i64, _P(_CSR)])
_sig("tcaspmm_mtx_read", [C.c_char_p, C.c_int, _P(_CSR)])
_sig("tcaspmm_csrbin_write", [C.c_char_p, _P(_CSR)])
_sig("tcaspmm_csrbin_read", [C.c_char_p, _P(_CSR)])
_sig("tcaspmm_gen_dense", [_i64, _i64, C.c_uint64, C.c_int, _vp])
_sig("tcaspmm_gen_uniform", [_i64, _i64, C.c_double, C.c_uint64, _P(_CSR)])
_sig("tcaspmm_gen_magnitude", [_i64, _i64, C.c_double, C.c_uint64, _P(_CSR)])
_sig("tcaspmm_gen_rmat", [C.c_int, _i64, C.c_double, C.c_double, C.c_double, C.c_int, C.c_uint64, _P(_CSR)])
_sig("tcaspmm_gen_skew", [_i64, _i64, _i64, C.c_double, C.c_uint64, _P(_CSR)])
_sig("tcaspmm_partition_columns", [_i64, C.c_int, C.c_int, C.c_int, _P(_i64), _P(_i64)])
_sig("tcaspmm_plan_create", [_P(_CSR), _i64, C.c_int, C.c_int, _P(C.c_int), _P(_vp)])
_sig("tcaspmm_plan_create_shard", [_P(_CSR), _i64, C.c_int, C.c_int, C.c_int, C.c_int, _P(_vp)])
_sig("tcaspmm_partition_rows", [_P(_CSR), C.c_int, _P(_i64)])
_sig("tcaspmm_plan_create_rows", [_P(_CSR), _i64, C.c_int, C.c_int, _P(C.c_int), _P(_vp)])
_sig("tcaspmm_plan_create_rows_shard", [_P(_CSR), _i64, C.c_int, C.c_int, C.c_int, C.c_int, _P(_vp)])
_sig("tcaspmm_plan_shard_rows", [_vp, C.c_int, _P(_i64), _P(_i64)])
_sig("tcaspmm_plan_create_2d", [_P(_CSR), _i64, C.c_int, C.c_int, C.c_int, _P(C.c_int), _P(_vp)])
_sig("tcaspmm_plan_create_2d_shard", [_P(_CSR), _i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P(_vp)])
_sig("tcaspmm_plan_destroy", [_vp])
_sig("tcaspmm_plan_get_stats", [_vp, _P(_Stats)])
_sig("tcaspmm_plan_shard", [_vp, C.c_int, _P(C.c_int), _P(_i64), _P(_i64)])
_sig("tcaspmm_execute", [_vp, _P(_vp), _P(_i64), _P(_vp), _P(_i64), _P(_vp)])
_sig("tcaspmm_execute1", [_vp, _vp, _i64, _vp, _i64, _vp])
_sig("tcaspmm_execute_ex", [_vp, _P(_vp), _P(_i64), _P(_vp), _P(_i64), _P(_vp), _P(_Epilogue)])
_sig("tcaspmm_execute1_ex", [_vp, _vp, _i64, _vp, _i64, _vp, _P(_Epilogue)])
_sig("tcaspmm_plan_sync_check", [_vp])
_sig("tcaspmm_plan_device_csr", [_vp, C.c_int, _P(_vp), _P(_vp), _P(_vp)])
_sig("tcaspmm_schedule_coverage", [_P(_CSR), _i64, C.c_int, _vp, _vp, _P(_Stats)])
_sig("tcaspmm_our_spmm_balanced", [_P(_RefCSR), _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _P(C.c_double)])


def _check(status: int) -> None:
    if status != 0:
        raise TcaspmmError(status, lib.tcaspmm_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib.tcaspmm_last_error().decode(errors="replace")


# --------------------------------------------------------------------- CSR
@dataclass
class CSR:
    """Host CSR: row_ptr int64 [M+1], col int32 [nnz], val float32 [nnz] or None (pattern, all 1.0)."""

    nrow: int
    ncol: int
    row_ptr: np.ndarray
    col: np.ndarray
    val: Optional[np.ndarray] = None

    def __post_init__(self):
        self.row_ptr = np.ascontiguousarray(self.row_ptr, dtype=np.int64)
        self.col = np.ascontiguousarray(self.col, dtype=np.int32)
        if self.val is not None:
            self.val = np.ascontiguousarray(self.val, dtype=np.float32)

    @property
    def nnz(self) -> int:
        return int(self.col.shape[0])

    def values(self) -> np.ndarray:
        return self.val if self.val is not None else np.ones(self.nnz, np.float32)

    def _c(self) -> _CSR:
        s = _CSR()
        s.nrow, s.ncol, s.nnz = self.nrow, self.ncol, self.nnz
        s.row_ptr = self.row_ptr.ctypes.data_as(_P(C.c_int64))
        s.col_idx = self.col.ctypes.data_as(_P(C.c_int32))
        s.val = self.val.ctypes.data_as(_P(C.c_float)) if self.val is not None else _P(C.c_float)()
        return s

    @staticmethod
    def _from_c(s: _CSR) -> "CSR":
        try:
            rp = np.ctypeslib.as_array(s.row_ptr, shape=(s.nrow + 1,)).copy()
            col = np.ctypeslib.as_array(s.col_idx, shape=(max(s.nnz, 1),))[: s.nnz].copy()
            val = None
            if bool(s.val):
                val = np.ctypeslib.as_array(s.val, shape=(max(s.nnz, 1),))[: s.nnz].copy()
            return CSR(int(s.nrow), int(s.ncol), rp, col, val)
        finally:
            lib.tcaspmm_csr_free(C.byref(s))

    def validate(self) -> None:
        _check(lib.tcaspmm_csr_validate(C.byref(self._c())))

    def to_scipy(self):
        import scipy.sparse as sp

        return sp.csr_matrix((self.values(), self.col, self.row_ptr), shape=(self.nrow, self.ncol))


def _gen(fn, *args) -> CSR:
    s = _CSR()
    _check(fn(*args, C.byref(s)))
    return CSR._from_c(s)


def smtx_read(path: str) -> CSR:
    """Read a .smtx file into CSR (smtx_input_to_Dense, src/file_input.cu:135-193)."""
    return _gen(lib.tcaspmm_smtx_read, os.fsencode(path))


smtx_input_to_CSR = smtx_read


def smtx_write(path: str, A: CSR) -> None:
    _check(lib.tcaspmm_smtx_write(os.fsencode(path), C.byref(A._c())))


def mtx_read(path: str, zero_based: bool = False) -> CSR:
    """Matrix Market coordinate file -> CSR (mtx_input_to_CSR, src/file_input.cu:64-134)."""
    return _gen(lib.tcaspmm_mtx_read, os.fsencode(path), int(bool(zero_based)))


mtx_input_to_CSR = mtx_read


def csrbin_write(path: str, A: CSR) -> None:
    _check(lib.tcaspmm_csrbin_write(os.fsencode(path), C.byref(A._c())))


def csrbin_read(path: str) -> CSR:
    return _gen(lib.tcaspmm_csrbin_read, os.fsencode(path))


def convert_dense_to_csr(dense_f16: np.ndarray) -> CSR:
    """Dense binary16 matrix -> CSR (src/miscalleneous.cu:29-65)."""
    d = np.ascontiguousarray(dense_f16, dtype=np.float16)
    M, K = d.shape
    return _gen(lib.tcaspmm_dense_to_csr, d.ctypes.data, M, K)


def gen_dense(rows: int, cols: int, seed: int = 0, dt="f32") -> np.ndarray:
    """Seeded N(0,1) matrix rounded to dt (bf16 returned as uint16 bit patterns)."""
    dt = as_dtype(dt)
    out = np.empty((rows, cols), dtype=_NP_OF[dt])
    _check(lib.tcaspmm_gen_dense(rows, cols, seed, int(dt), out.ctypes.data))
    return out


def gen_uniform(M: int, K: int, density: float, seed: int = 0) -> CSR:
    return _gen(lib.tcaspmm_gen_uniform, M, K, density, seed)


def gen_magnitude(M: int, K: int, sparsity: float, seed: int = 0) -> CSR:
    return _gen(lib.tcaspmm_gen_magnitude, M, K, sparsity, seed)


def partition_rows(A: CSR, parts: int) -> np.ndarray:
    """Row blocks of about equal cost (tcaspmm_partition_rows): parts + 1 boundaries."""
    out = np.zeros(parts + 1, np.int64)
    cA = A._c()
    _check(lib.tcaspmm_partition_rows(C.byref(cA), parts, out.ctypes.data_as(_P(_i64))))
    return out


def gen_rmat(scale: int, edges: int, a=0.57, b=0.19, c=0.19, kind: str = "gcn", seed: int = 0) -> CSR:
    return _gen(lib.tcaspmm_gen_rmat, scale, edges, a, b, c, {"gcn": 0, "sage": 1}[kind], seed)


def gen_skew(n: int, hubs: int, hub_nnz: int, lam: float = 3.0, seed: int = 0) -> CSR:
    return _gen(lib.tcaspmm_gen_skew, n, hubs, hub_nnz, lam, seed)


def partition_columns(N: int, dt, world: int, rank: int):
    b, c = _i64(), _i64()
    _check(lib.tcaspmm_partition_columns(N, int(as_dtype(dt)), world, rank, C.byref(b), C.byref(c)))
    return b.value, c.value


def schedule_coverage(A: CSR, N: int, dt):
    """Host-only schedule walk: (cover[nnz] int32, kind[nnz] int8, stats dict)."""
    cover = np.empty(max(A.nnz, 1), np.int32)
    kind = np.empty(max(A.nnz, 1), np.int8)
    st = _Stats()
    _check(lib.tcaspmm_schedule_coverage(C.byref(A._c()), N, int(as_dtype(dt)), cover.ctypes.data,
                                         kind.ctypes.data, C.byref(st)))
    return cover[: A.nnz], kind[: A.nnz], st.to_dict()


# -------------------------------------------------------------------- plans
def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(s) -> int:
    if s is None:
        return 0
    if isinstance(s, int):
        return s
    return int(s.cuda_stream)


@dataclass
class Epilogue:
    """Fused output epilogue (tcaspmm_epilogue): C = relu?(row_scale[r] * (A @ B)[r, c] + bias[c]).

    row_scale (M floats) and bias (one float per column of the shard's block) are
    device tensors / pointers on the shard's device or None (1 and 0); out_dtype
    is the type C is stored in: "f32", "f16" or "bf16".
    """
    row_scale: object = None
    bias: object = None
    relu: bool = False
    out_dtype: object = "f32"

    def _c(self) -> _Epilogue:
        return _Epilogue(_ptr(self.row_scale) if self.row_scale is not None else None,
                         _ptr(self.bias) if self.bias is not None else None, int(bool(self.relu)),
                         int(as_dtype(self.out_dtype)))


class Plan:
    """Preprocessed A on one or more GPUs (tcaspmm_plan_create / _create_shard)."""

    def __init__(self, A: CSR, N: int, dt="f16", num_gpus: int = 1, devices: Optional[Sequence[int]] = None,
                 *, rank: Optional[int] = None, world: Optional[int] = None, device: Optional[int] = None,
                 split: str = "columns", grid: Optional[Sequence[int]] = None):
        """split="columns": shards own column blocks of B and C (A replicated);
        split="rows": shards own row blocks of A and C (B replicated);
        split="2d": a grid = (row blocks, column blocks) of shards, shard s owning row
        block s // grid[1] and column block s % grid[1]."""
        if split not in ("columns", "rows", "2d"):
            raise ValueError(f"split must be 'columns', 'rows' or '2d', not {split!r}")
        if split == "2d" and (grid is None or len(grid) != 2):
            raise ValueError("split='2d' needs grid=(row blocks, column blocks)")
        self._h = _vp()
        self.dt = as_dtype(dt)
        self.split = split
        self.N, self.M, self.K, self.nnz = int(N), A.nrow, A.ncol, A.nnz
        cA = A._c()
        if split == "2d":
            gr, gc = int(grid[0]), int(grid[1])
            if rank is not None:
                _check(lib.tcaspmm_plan_create_2d_shard(C.byref(cA), N, int(self.dt), rank, gr, gc, device,
                                                        C.byref(self._h)))
            else:
                devs = (C.c_int * len(devices))(*devices) if devices is not None else None
                _check(lib.tcaspmm_plan_create_2d(C.byref(cA), N, int(self.dt), gr, gc, devs, C.byref(self._h)))
        elif rank is not None:
            fn = lib.tcaspmm_plan_create_shard if split == "columns" else lib.tcaspmm_plan_create_rows_shard
            _check(fn(C.byref(cA), N, int(self.dt), rank, world, device, C.byref(self._h)))
        else:
            devs = None
            if devices is not None:
                devs = (C.c_int * len(devices))(*devices)
            fn = lib.tcaspmm_plan_create if split == "columns" else lib.tcaspmm_plan_create_rows
            _check(fn(C.byref(cA), N, int(self.dt), num_gpus, devs, C.byref(self._h)))
        # Nonzeros per shard (row blocks hold part of A).
        if split == "2d":
            rb = partition_rows(A, gr)
            parts = [rank] if rank is not None else range(gr * gc)
            self._shard_nnz = [int(A.row_ptr[rb[i // gc + 1]] - A.row_ptr[rb[i // gc]]) for i in parts]
        elif split == "rows":
            rb = partition_rows(A, world if rank is not None else num_gpus)
            parts = [rank] if rank is not None else range(num_gpus)
            self._shard_nnz = [int(A.row_ptr[rb[i + 1]] - A.row_ptr[rb[i]]) for i in parts]
        else:
            self._shard_nnz = [A.nnz] * (1 if rank is not None else num_gpus)

    def close(self) -> None:
        if self._h:
            lib.tcaspmm_plan_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:  # pragma: no cover - interpreter teardown
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def stats(self) -> dict:
        st = _Stats()
        _check(lib.tcaspmm_plan_get_stats(self._h, C.byref(st)))
        return st.to_dict()

    @property
    def num_shards(self) -> int:
        return int(self.stats["num_shards"])

    def shard(self, s: int):
        """(device, col_begin, col_count) of shard s."""
        dev, b, c = C.c_int(), _i64(), _i64()
        _check(lib.tcaspmm_plan_shard(self._h, s, C.byref(dev), C.byref(b), C.byref(c)))
        return dev.value, b.value, c.value

    def shard_nnz(self, s: int) -> int:
        return self._shard_nnz[s]

    def shard_rows(self, s: int):
        """(row_begin, row_count) of shard s (0, M for column-split plans)."""
        b, c = _i64(), _i64()
        _check(lib.tcaspmm_plan_shard_rows(self._h, s, C.byref(b), C.byref(c)))
        return b.value, c.value

    def execute(self, B: Sequence, Cs: Sequence, ldb: Optional[Sequence[int]] = None,
                ldc: Optional[Sequence[int]] = None, streams: Optional[Sequence] = None,
                epilogues: Optional[Sequence[Epilogue]] = None) -> None:
        """Launch C[s] = A @ B[s] for every shard s (device tensors or raw pointers),
        through epilogues[s] when given."""
        n = len(B)
        ldb = ldb or [int(b.stride(0)) for b in B]
        ldc = ldc or [int(c.stride(0)) for c in Cs]
        pb = (_vp * n)(*[_ptr(b) for b in B])
        pc = (_vp * n)(*[_ptr(c) for c in Cs])
        lb = (_i64 * n)(*ldb)
        lc = (_i64 * n)(*ldc)
        st = (_vp * n)(*[_stream_handle(s) for s in (streams or [None] * n)])
        if epilogues is None:
            _check(lib.tcaspmm_execute(self._h, pb, lb, pc, lc, st))
        else:
            eps = (_Epilogue * n)(*[e._c() for e in epilogues])
            _check(lib.tcaspmm_execute_ex(self._h, pb, lb, pc, lc, st, eps))

    def execute1(self, B, Cout, stream=None, ldb: Optional[int] = None, ldc: Optional[int] = None,
                 epilogue: Optional[Epilogue] = None) -> None:
        lb = ldb if ldb is not None else int(B.stride(0))
        lc = ldc if ldc is not None else int(Cout.stride(0))
        if epilogue is None:
            _check(lib.tcaspmm_execute1(self._h, _ptr(B), lb, _ptr(Cout), lc, _stream_handle(stream)))
        else:
            ep = epilogue._c()
            _check(lib.tcaspmm_execute1_ex(self._h, _ptr(B), lb, _ptr(Cout), lc, _stream_handle(stream),
                                           C.byref(ep)))

    def sync_check(self) -> None:
        _check(lib.tcaspmm_plan_sync_check(self._h))

    def device_csr(self, s: int = 0):
        rp, col, val = _vp(), _vp(), _vp()
        _check(lib.tcaspmm_plan_device_csr(self._h, s, C.byref(rp), C.byref(col), C.byref(val)))
        return rp.value or 0, col.value or 0, val.value or 0

    @property
    def handle(self) -> int:
        return self._h.value or 0


def spmm(A: CSR, B, dt=None):
    """One-shot C = A @ B for a CUDA tensor B (K x N); returns a new fp32 tensor."""
    import torch

    dt = as_dtype(dt if dt is not None else B.dtype)
    B = B.contiguous()
    out = torch.empty((A.nrow, B.shape[1]), device=B.device, dtype=torch.float32)
    with Plan(A, B.shape[1], dt, 1, [B.device.index or 0]) as p:
        p.execute1(B, out, torch.cuda.current_stream(B.device))
        p.sync_check()
    return out


# ------------------------------------------------- reference entry point
# our_spmm_balanced keeps the reference's argument name C, which shadows the
# ctypes module inside it; these aliases are what it uses instead.
C_int, C_uint16, C_double, C_byref = C.c_int, C.c_uint16, C.c_double, C.byref


def our_spmm_balanced(row_offset: np.ndarray, col_idx: np.ndarray, value_f16: np.ndarray, B_f16: np.ndarray,
                      C: np.ndarray, M: int, N: int, K: int, n_iter: int = 10) -> float:
    """Reference signature (src/our_spmm.cu:478): host CSR (int32, half), host half B, host fp32 C
    overwritten in place; returns the average kernel milliseconds."""
    ro = np.ascontiguousarray(row_offset, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    va = np.ascontiguousarray(value_f16, dtype=np.float16)
    Bh = np.ascontiguousarray(B_f16, dtype=np.float16)
    if not (C.dtype == np.float32 and C.flags.c_contiguous and C.size == M * N):
        raise TcaspmmError(Status.INVALID_ARG, "C must be a C-contiguous float32 array of M*N elements")
    if ro.shape[0] != M + 1 or Bh.size != K * N or va.shape[0] != ci.shape[0]:
        raise TcaspmmError(Status.INVALID_ARG, "row_offset must hold M+1 entries, B K*N, value one per column")
    r = _RefCSR(M, K, int(ci.shape[0]), ro.ctypes.data_as(_P(C_int)), ci.ctypes.data_as(_P(C_int)),
                va.view(np.uint16).ctypes.data_as(_P(C_uint16)))
    ms = C_double()
    _check(lib.tcaspmm_our_spmm_balanced(C_byref(r), Bh.ctypes.data, C.ctypes.data, M, N, K, n_iter,
                                         C_byref(ms)))
    return ms.value


# ------------------------------------------------------------- baselines
_blib = None


def baselines():
    """ctypes handle of libtcaspmm_baselines.so (cuSPARSE / cuBLAS, reported only)."""
    global _blib
    if _blib is None:
        _blib = C.CDLL(BASELINES_PATH)
        _blib.tcaspmm_cusparse_spmm.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64,
                                                C.c_int, C.c_int, C.c_int, _vp, _P(C.c_double)]
        _blib.tcaspmm_cusparse_spmm.restype = C.c_int
        _blib.tcaspmm_cublas_gemm.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, C.c_int, C.c_int, C.c_int, _vp,
                                              _P(C.c_double)]
        _blib.tcaspmm_cublas_gemm.restype = C.c_int
        _blib.tcaspmm_cusparse_blocked_ell.argtypes = [_P(_CSR), C.c_int, _vp, _i64, _vp, _i64, _i64, C.c_int,
                                                       C.c_int, C.c_int, _vp, _P(C.c_double), _P(_i64)]
        _blib.tcaspmm_cusparse_blocked_ell.restype = C.c_int
        _blib.tcaspmm_gather_floor.argtypes = [_vp, _i64, _vp, _i64, _i64, C.c_int, C.c_int, C.c_int, _vp,
                                               _P(C.c_double)]
        _blib.tcaspmm_gather_floor.restype = C.c_int
        _blib.tcaspmm_baselines_set_flush.argtypes = [_vp, C.c_size_t]
        _blib.tcaspmm_baselines_set_flush.restype = None
    return _blib


def baselines_set_flush(buf) -> None:
    """Flush L2 by writing `buf` (a device tensor larger than L2) before every timed baseline call;
    None restores back-to-back timing."""
    if buf is None:
        baselines().tcaspmm_baselines_set_flush(None, 0)
    else:
        baselines().tcaspmm_baselines_set_flush(_ptr(buf), buf.numel() * buf.element_size())


def cusparse_blocked_ell(A: CSR, block: int, B, Cout, dt, warmup: int = 5, iters: int = 10, stream=None):
    """Time cusparseSpMM on A converted to Blocked-ELL (block x block); returns (ms per call, ELL bytes)."""
    ms, nbytes = C.c_double(), _i64()
    cA = A._c()
    _check(baselines().tcaspmm_cusparse_blocked_ell(C.byref(cA), block, _ptr(B), int(B.stride(0)), _ptr(Cout),
                                                    int(Cout.stride(0)), int(B.shape[1]), int(as_dtype(dt)), warmup,
                                                    iters, _stream_handle(stream), C.byref(ms), C.byref(nbytes)))
    return ms.value, nbytes.value


def cusparse_spmm(plan: Plan, B, Cout, warmup: int = 10, iters: int = 10, stream=None, shard: int = 0) -> float:
    """Time cusparseSpMM on the plan's device CSR; returns ms per call."""
    rp, col, val = plan.device_csr(shard)
    ms = C.c_double()
    _, _, ncols = plan.shard(shard)
    _, rows = plan.shard_rows(shard)
    _check(baselines().tcaspmm_cusparse_spmm(rp, col, val, rows, plan.K, plan.shard_nnz(shard), _ptr(B),
                                             int(B.stride(0)),
                                             _ptr(Cout), int(Cout.stride(0)), ncols, int(plan.dt), warmup, iters,
                                             _stream_handle(stream), C.byref(ms)))
    return ms.value


def gather_floor(plan: Plan, B, warmup: int = 3, iters: int = 10, stream=None, shard: int = 0) -> float:
    """Time the per-nonzero B-row gathers of the plan's shard alone (no arithmetic, no C
    write): the floor of a gather-per-nonzero SpMM on this GPU.  Returns ms per call."""
    _, col, _ = plan.device_csr(shard)
    _, _, ncols = plan.shard(shard)
    ms = C.c_double()
    _check(baselines().tcaspmm_gather_floor(col, plan.shard_nnz(shard), _ptr(B), int(B.stride(0)), ncols,
                                            int(plan.dt), warmup, iters, _stream_handle(stream), C.byref(ms)))
    return ms.value


def cublas_gemm(A_dense, B, Cout, dt, warmup: int = 5, iters: int = 10, stream=None) -> float:
    M, K = A_dense.shape
    N = B.shape[1]
    ms = C.c_double()
    _check(baselines().tcaspmm_cublas_gemm(_ptr(A_dense), _ptr(B), _ptr(Cout), M, N, K, int(as_dtype(dt)), warmup,
                                           iters, _stream_handle(stream), C.byref(ms)))
    return ms.value
