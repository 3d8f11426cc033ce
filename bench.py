"""Benchmark of the tcaspmm hot path, C = A @ B (CSR A, dense row-major B).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gcn|ffn|sage|skew] [--impl ours|reference]

Default workload: the GCN aggregation config (R-MAT a=0.57 b=0.19 c=0.19, 2^20
nodes, 30M directed draws, symmetrised + self-loops, values 1/sqrt(d_i d_j),
X 1M x 128 N(0,1) fp32), seeded synthetic data.  One step = one SpMM over the
whole matrix.  With N GPUs (torchrun, one rank per GPU) each rank owns a column
block of B and C (A replicated, no collective on the data path); value = total
GFLOP/s of the whole job (2 nnz N / max-over-ranks time).

``--impl reference`` times the reference semantics on the host cores instead:
the reference ships no CPU CSR loop, so this is the fp32 OpenMP CSR loop of
oracle/oracle.c (a restatement of src/our_spmm.cu's arithmetic), run by rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMM GFLOP/s (2*nnz*N)"
UNIT = "GFLOP/s"
L2_BYTES = 126 * 2**20

WORKLOADS = {
    # name: (description, builder, N, dtype)
    "gcn": ("C3 GCN aggregation: R-MAT(0.57,0.19,0.19) 2^20 nodes, 30M draws, symmetrised + self-loops, "
            "1/sqrt(d_i d_j); X 1M x 128 fp32", lambda T: T.gen_rmat(20, 30_000_000, kind="gcn", seed=0), 128, "f32"),
    "ffn": ("C1 pruned FFN: A 2048x512 70% uniform sparsity, N(0,1); B 512x256 N(0,1) fp16",
            lambda T: T.gen_uniform(2048, 512, 0.3, 0), 256, "f16"),
    "sage": ("C4 GraphSAGE mean: R-MAT 2^22 nodes, 100M draws, 1/deg(i); X 4M x 256 fp16",
             lambda T: T.gen_rmat(22, 100_000_000, kind="sage", seed=0), 256, "f16"),
    "skew": ("C5 extreme skew: 8M x 8M, 64 hub rows x 200k nnz + Poisson(3) rows, U(-1,1); B 8M x 64 fp16",
             lambda T: T.gen_skew(1 << 23, 64, 200_000, 3.0, seed=0), 64, "f16"),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(workload: str, profiled_config: bool = True):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, or None
    when there is none or this run is not the configuration that was profiled."""
    p = os.path.join(ROOT, "profiles", "traffic.json.txt")
    if not profiled_config or not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d.get(workload)


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) in a thread during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, local_rank: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            # NVML numbers GPUs physically; map through CUDA_VISIBLE_DEVICES.
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            entry = vis.split(",")[local_rank].strip() if vis else str(local_rank)
            if entry.isdigit():
                self._h = pynvml.nvmlDeviceGetHandleByIndex(int(entry))
            else:
                self._h = pynvml.nvmlDeviceGetHandleByUUID(entry)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - reported in the JSON
            self.error = str(e)
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                mask = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t.is_alive():
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def host_threads() -> int:
    """All host threads this process may use (torchrun sets OMP_NUM_THREADS=1, so ask the OS)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def pin_to_gpu_numa_node(local_rank: int):
    """Bind this process to the CPUs NVML reports as local to the GPU (its NUMA
    node), so pinned host buffers are first touched there and the host side of the
    copies runs next to the GPU's PCIe root.  Only this process's CPU affinity
    changes; returns the previous affinity (to restore), or None."""
    try:
        import pynvml

        before = os.sched_getaffinity(0)
        pynvml.nvmlInit()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        entry = vis.split(",")[local_rank].strip() if vis else str(local_rank)
        h = (pynvml.nvmlDeviceGetHandleByIndex(int(entry)) if entry.isdigit()
             else pynvml.nvmlDeviceGetHandleByUUID(entry))
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= before
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return before
    except Exception:  # no NVML or no affinity information: leave the process as it is
        return None


def algorithmic_bytes(M, K, nnz, N, elem):
    return (M + 1) * 4 + nnz * (4 + elem) + K * N * elem + M * N * 4


class HostGen:
    """The seeded input generators of libtcaspmm_host.so (host code only: no CUDA runtime,
    no GPU kernels), so the reference arm builds the same inputs as the GPU arm without
    loading the product library.  Mirrors the gen_* functions of spmm_b200."""

    class _CSR(ctypes.Structure):
        _fields_ = [("nrow", ctypes.c_int64), ("ncol", ctypes.c_int64), ("nnz", ctypes.c_int64),
                    ("row_ptr", ctypes.POINTER(ctypes.c_int64)), ("col_idx", ctypes.POINTER(ctypes.c_int32)),
                    ("val", ctypes.POINTER(ctypes.c_float))]

    class Matrix:
        def __init__(self, nrow, ncol, row_ptr, col, val):
            self.nrow, self.ncol, self.row_ptr, self.col, self.val = nrow, ncol, row_ptr, col, val
            self.nnz = int(col.shape[0])

        def values(self):
            return self.val if self.val is not None else np.ones(self.nnz, np.float32)

    def __init__(self):
        self.lib = ctypes.CDLL(os.path.join(ROOT, "spmm_b200", "lib", "libtcaspmm_host.so"))
        self.lib.tcaspmm_last_error.restype = ctypes.c_char_p

    def _take(self, st, s):
        if st != 0:
            raise RuntimeError(f"generator failed ({st}): {self.lib.tcaspmm_last_error().decode()}")
        try:
            rp = np.ctypeslib.as_array(s.row_ptr, shape=(s.nrow + 1,)).copy()
            col = np.ctypeslib.as_array(s.col_idx, shape=(max(s.nnz, 1),))[: s.nnz].copy()
            val = np.ctypeslib.as_array(s.val, shape=(max(s.nnz, 1),))[: s.nnz].copy() if bool(s.val) else None
            return self.Matrix(int(s.nrow), int(s.ncol), rp, col, val)
        finally:
            self.lib.tcaspmm_csr_free(ctypes.byref(s))

    def gen_rmat(self, scale, edges, a=0.57, b=0.19, c=0.19, kind="gcn", seed=0):
        s = self._CSR()
        f = self.lib.tcaspmm_gen_rmat
        f.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_int,
                      ctypes.c_uint64, ctypes.POINTER(self._CSR)]
        return self._take(f(scale, edges, a, b, c, {"gcn": 0, "sage": 1}[kind], seed, ctypes.byref(s)), s)

    def gen_uniform(self, M, K, density, seed=0):
        s = self._CSR()
        f = self.lib.tcaspmm_gen_uniform
        f.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_double, ctypes.c_uint64, ctypes.POINTER(self._CSR)]
        return self._take(f(M, K, density, seed, ctypes.byref(s)), s)

    def gen_skew(self, n, hubs, hub_nnz, lam=3.0, seed=0):
        s = self._CSR()
        f = self.lib.tcaspmm_gen_skew
        f.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_double, ctypes.c_uint64,
                      ctypes.POINTER(self._CSR)]
        return self._take(f(n, hubs, hub_nnz, lam, seed, ctypes.byref(s)), s)

    def gen_dense(self, rows, cols, seed=0, dt="f32"):
        code = {"f32": 0, "f16": 1, "bf16": 2, "tf32": 3}[dt]
        out = np.empty((rows, cols), dtype={0: np.float32, 1: np.float16, 2: np.uint16, 3: np.float32}[code])
        f = self.lib.tcaspmm_gen_dense
        f.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p]
        st = f(rows, cols, seed, code, out.ctypes.data)
        if st != 0:
            raise RuntimeError(f"gen_dense failed ({st})")
        return out


def _round_to(x: np.ndarray, dt: str) -> np.ndarray:
    """fp32 values rounded as the plan stores them (f16 / bf16 round to nearest even)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dt == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        return u.astype(np.uint32).view(np.float32)
    return x


def _as_f32(b: np.ndarray, dt: str) -> np.ndarray:
    """A host B block in the plan dtype (bf16 as uint16 bits) -> float32."""
    if dt == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.astype(np.float32)


def parity_sample(A, Bblk: np.ndarray, C_rows: np.ndarray, rows: np.ndarray, dt: str, ep_host=None,
                  chunk: int = 8192) -> float:
    """rel-L2 of the device rows C_rows (one per entry of `rows`, this rank's column
    block) against an fp64 sum over each row's nonzeros, computed here in numpy from
    the same rounded inputs; ep_host = (row_scale, bias) applies the bench's epilogue
    (relu(s * AB + b)) to the reference."""
    vals = _round_to(A.values(), dt).astype(np.float64)
    num = den = 0.0
    for i, r in enumerate(rows):
        b, e = int(A.row_ptr[r]), int(A.row_ptr[r + 1])
        ref = np.zeros(Bblk.shape[1], np.float64)
        for j in range(b, e, chunk):
            k = min(e, j + chunk)
            ref += vals[j:k] @ _as_f32(Bblk[A.col[j:k]], dt).astype(np.float64)
        if ep_host is not None:
            rs, bias = ep_host
            ref = np.maximum(rs[r] * ref + bias, 0.0)
        num += float(np.sum((C_rows[i].astype(np.float64) - ref) ** 2))
        den += float(np.sum(ref ** 2))
    return (num / den) ** 0.5 if den > 0 else (num ** 0.5)


def measure_c1(T, torch, dev, steps: int = 100, warmup: int = 10) -> dict:
    """The C1 pruned-FFN config (A 2048 x 512 at 70% uniform sparsity, B 512 x 256
    fp16; all rows on the tensor-core windows) timed the way `--workload ffn` times
    it -- L2 flushed with a 2x L2 write before every step, CUDA events around each
    step's graph replay -- with its parity sample and dense cuBLAS / cuSPARSE CSR on
    the same data under the same flush.  Reported beside the default line so the
    north star's second target config is in every default run."""
    A = T.gen_uniform(2048, 512, 0.3, 0)
    N = 256
    Bh = T.gen_dense(A.ncol, N, 1, "f16")
    Bd = torch.from_numpy(Bh).to(dev)
    Cd = torch.empty((A.nrow, N), device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    with T.Plan(A, N, "f16", rank=0, world=1, device=dev.index) as plan:
        for _ in range(warmup):
            plan.execute1(Bd, Cd, stream)
        plan.sync_check()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            plan.execute1(Bd, Cd, cap)
        stream.wait_stream(cap)
        for _ in range(3):
            graph.replay()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            graph.replay()
            b.record(stream)
        torch.cuda.synchronize(dev)
        plan.sync_check()
        ms = sum(a.elapsed_time(b) for a, b in evs) / steps
        st = plan.stats
        rows = np.unique(np.concatenate([np.arange(0, A.nrow, 7), [A.nrow - 1]]))
        rel = parity_sample(A, Bh, Cd[torch.from_numpy(rows).to(dev)].cpu().numpy(), rows, "f16")
        T.baselines_set_flush(flush)
        try:
            Cs = torch.empty_like(Cd)
            ms_cusparse = T.cusparse_spmm(plan, Bd, Cs, warmup=3, iters=50, stream=stream)
            Ad = torch.zeros((A.nrow, A.ncol), dtype=torch.float16, device=dev)
            r_idx = torch.from_numpy(np.repeat(np.arange(A.nrow), np.diff(A.row_ptr))).to(dev)
            Ad[r_idx, torch.from_numpy(A.col.astype(np.int64)).to(dev)] = \
                torch.from_numpy(A.values()).to(dev).to(torch.float16)
            Cg = torch.empty_like(Cd)
            ms_cublas = T.cublas_gemm(Ad, Bd, Cg, "f16", warmup=3, iters=50, stream=stream)
        finally:
            T.baselines_set_flush(None)
        del graph
    flops = 2.0 * A.nnz * N
    alg = algorithmic_bytes(A.nrow, A.ncol, A.nnz, N, 2)
    return {"workload": "C1 pruned FFN: A 2048x512 70% uniform sparsity, N(0,1); B 512x256 N(0,1) fp16",
            "ms_per_step": round(ms, 5), "value": round(flops / (ms * 1e-3) / 1e9, 3), "unit": UNIT,
            "l2": "flushed between steps (2x L2 buffer)", "tc_windows": st["tc_windows"],
            "hbm_frac": round(alg / (ms * 1e-3) / 1e9 / load_peaks()[0], 4),
            "gemm_cublas_ms": round(ms_cublas, 5), "spmm_cusparse_ms": round(ms_cusparse, 5),
            "parity": {"rel_l2": float(f"{rel:.3e}"), "tol": 5e-3, "ok": bool(rel <= 5e-3),
                       "rows": int(rows.shape[0])}}


def cpu_reference(A, B, threads: int, budget_s: float = 12.0):
    """Time the fp32 CPU CSR loop; whole-matrix passes until budget_s, else a row sample."""
    import oracle

    vals = A.values()
    t0 = time.perf_counter()
    oracle.spmm_f32(A.row_ptr, A.col, vals, B, threads)
    one = time.perf_counter() - t0
    flops_one = 2.0 * A.nnz * B.shape[1]
    if one > budget_s / 2:
        return flops_one / one / 1e9, f"one full pass over all {A.nrow} rows ({one:.1f} s)"
    reps = max(1, int(budget_s / max(one, 1e-4)))
    reps = min(reps, 200)
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.spmm_f32(A.row_ptr, A.col, vals, B, threads)
    dt = time.perf_counter() - t0
    return flops_one * reps / dt / 1e9, f"{reps} full passes over all {A.nrow} rows ({dt:.1f} s)"


def run_reference(args, wl):
    """Reference arm: rank 0 times the fp32 CPU CSR loop on all host threads.

    Each step is a bounded, strided row sample of the same workload, sized so
    the whole --warmup + --steps run stays within about two minutes."""
    import oracle

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    desc, build, N, dt = wl
    if args.dtype:
        dt = args.dtype
        desc += f" [dtype {dt}]"
    if args.cols:
        N = args.cols
        desc += f" [N {N}]"
    T = HostGen()  # the same seeded inputs, without loading the GPU library
    A = build(T)
    B = T.gen_dense(A.ncol, N, 1, "f32")
    if dt in ("f16", "bf16"):
        B = B.astype(np.float16).astype(np.float32)
    threads = host_threads()
    vals = A.values()
    t0 = time.perf_counter()
    oracle.spmm_f32(A.row_ptr, A.col, vals, B, threads)  # one full pass: sizes the sample
    t_full = time.perf_counter() - t0
    per_step = min(t_full, 120.0 / (args.steps + args.warmup))
    stride = max(1, int(round(t_full / max(per_step, 1e-6))))
    rows = np.arange(0, A.nrow, stride, dtype=np.int64)
    sample_nnz = int(np.diff(A.row_ptr)[rows].sum())
    for _ in range(args.warmup):
        oracle.spmm_f32_rows(rows, A.row_ptr, A.col, vals, B, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.spmm_f32_rows(rows, A.row_ptr, A.col, vals, B, threads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    value = 2.0 * sample_nnz * N / t / 1e9
    which = "all rows" if stride == 1 else f"every {stride}th row"
    sample = (f"{which} ({rows.shape[0]} rows, {sample_nnz} nnz) per step; "
              f"full pass {t_full:.2f} s")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "ms_per_step": round(2.0 * A.nnz * N / (value * 1e9) * 1e3, 4),
            "config": {"workload": desc, "nnz": A.nnz, "M": A.nrow, "K": A.ncol, "N": N,
                       "parallelism": "host cores (OpenMP)"},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="gcn", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c1", action="store_true",
                    help="skip the C1 pruned-FFN record the default one-GPU run adds to its line")
    ap.add_argument("--dtype", default=None, choices=["f32", "tf32", "f16", "bf16"],
                    help="override the workload's dtype (e.g. tf32: fp32 B through the TF32 tensor-core path)")
    ap.add_argument("--epilogue", action="store_true",
                    help="fused epilogue: C = relu(row_scale * (A B) + bias) stored as bf16")
    ap.add_argument("--gather", action="store_true",
                    help="also time the step followed by an NCCL all-gather of C (N > 1)")
    ap.add_argument("--split", default="columns", choices=["columns", "rows", "2d"],
                    help="multi-GPU partition: column blocks of B/C (A replicated), row blocks of A/C "
                         "(B replicated), or a 2-D grid of both (--grid)")
    ap.add_argument("--numa", type=int, default=1, choices=[0, 1],
                    help="1: bind each rank to its GPU's local CPUs (pinned buffers on that NUMA node)")
    ap.add_argument("--launch", default="graph", choices=["graph", "eager"],
                    help="timed step: replay a CUDA graph of the plan's launches, or call execute directly")
    ap.add_argument("--cols", type=int, default=None,
                    help="override the workload's N (e.g. --cols 16 on one GPU: the per-rank work of C3's "
                         "8-GPU column split, for profiling)")
    ap.add_argument("--grid", default=None,
                    help="RxC shard grid for --split 2d (default: two column blocks when N GPUs is even)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)

    import torch
    import torch.distributed as dist

    import spmm_b200 as T

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"bench: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    torch.cuda.set_device(local)
    affinity_before = pin_to_gpu_numa_node(local) if args.numa else None
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    desc, build, N, dt = wl
    if args.dtype:
        dt = args.dtype
        desc += f" [dtype {dt}]"
    if args.cols:
        N = args.cols
        desc += f" [N {N}]"
    tdt = {"f32": torch.float32, "tf32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dt]
    elem = 4 if dt in ("f32", "tf32") else 2
    A = build(T)
    M, K, nnz = A.nrow, A.ncol, A.nnz
    Bfull = T.gen_dense(K, N, 1, dt)  # host, dt (bf16 as uint16 bits)
    grid = None
    if args.split == "2d":
        if args.grid:
            grid = tuple(int(x) for x in args.grid.lower().split("x"))
        else:
            gc = 2 if world % 2 == 0 else 1
            grid = (world // gc, gc)
        if grid[0] * grid[1] != world:
            raise SystemExit(f"bench: grid {grid} does not match {world} GPUs")
    if args.split == "columns":
        col0, ncols = T.partition_columns(N, dt, world, rank)
        row0, mrows = 0, M
    elif args.split == "2d":
        col0, ncols = T.partition_columns(N, dt, grid[1], rank % grid[1])
    else:
        col0, ncols = 0, N
    plan = T.Plan(A, N, dt, rank=rank, world=world, device=local, split=args.split, grid=grid)
    if args.split in ("rows", "2d"):
        row0, mrows = plan.shard_rows(0)
    pst = plan.stats
    Bblk = np.ascontiguousarray(Bfull[:, col0:col0 + ncols])
    Bh = torch.from_numpy(Bblk.view(np.int16) if dt == "bf16" else Bblk)
    if dt == "bf16":
        Bh = Bh.view(torch.bfloat16)
    Bd = Bh.to(dev)
    cdt = torch.bfloat16 if args.epilogue else torch.float32
    Cd = torch.empty((mrows, max(ncols, 1)), dtype=cdt, device=dev)[:, :ncols]
    ep = None
    if args.epilogue:
        g = torch.Generator().manual_seed(11)
        ep = T.Epilogue((torch.rand(mrows, generator=g) + 0.5).to(dev), torch.randn(ncols, generator=g).to(dev),
                        True, "bf16")
    stream = torch.cuda.current_stream(dev)
    in_l2 = algorithmic_bytes(M, K, nnz, ncols, elem) <= L2_BYTES
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if in_l2 else None

    def step():
        plan.execute1(Bd, Cd, stream, epilogue=ep)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- kernel-resident timing (inputs already in HBM) ----
    for _ in range(args.warmup):
        step()
    plan.sync_check()
    # With --launch graph (the default) the timed step replays a CUDA graph of the
    # plan's launches (same kernels, same arguments; launch latency paid once at
    # capture); with --launch eager it calls the C-ABI execute directly.
    graph = None
    if args.launch == "graph":
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            plan.execute1(Bd, Cd, cap, epilogue=ep)
        stream.wait_stream(cap)

        def step():  # noqa: F811 -- the graph replaces the eager launch from here on
            graph.replay()

    for _ in range(2):
        step()
    plan.sync_check()
    barrier()
    sampler = ClockSampler(local)
    with sampler:
        if flush is None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms_total = e0.elapsed_time(e1)
        else:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for a, b in evs:
                flush.zero_()
                a.record(stream)
                step()
                b.record(stream)
            torch.cuda.synchronize(dev)
            ms_total = sum(a.elapsed_time(b) for a, b in evs)
    barrier()
    plan.sync_check()
    ms_step = max_over_ranks(ms_total / args.steps)
    flops = 2.0 * nnz * N
    value = flops / (ms_step * 1e-3) / 1e9

    # ---- correctness of this rank's C block (outside the timed region): a seeded
    # sample of its rows, the longest rows included, against an fp64 sum computed on
    # the host from the same rounded inputs; the worst rank is reported ----
    rl = np.diff(A.row_ptr[row0:row0 + mrows + 1])
    g = np.random.default_rng(1234 + rank)
    hub = row0 + np.argsort(-rl, kind="stable")[:8]
    rows_s = np.unique(np.concatenate([hub, row0 + g.choice(mrows, size=min(mrows, 2000), replace=False)]))
    C_rows = Cd[torch.from_numpy(rows_s - row0).to(dev)].float().cpu().numpy()
    ep_host = None
    if ep is not None:
        ep_host = (ep.row_scale.cpu().numpy().astype(np.float64), ep.bias.cpu().numpy().astype(np.float64))
        ep_rows = np.zeros(M, np.float64)
        ep_rows[row0:row0 + mrows] = ep_host[0]
        ep_host = (ep_rows, ep_host[1])
    rel = parity_sample(A, Bblk, C_rows, rows_s, dt, ep_host)
    rel = max_over_ranks(rel)
    # fp32 on the CUDA cores: 1e-5; 16-bit / TF32 inputs through the tensor cores:
    # 5e-3; bf16 output of the epilogue adds its own rounding (2^-9 relative).
    tol = 1e-5 if dt == "f32" and ep is None else 5e-3 if ep is None else 8e-3
    parity = {"rel_l2": float(f"{rel:.3e}"), "tol": tol, "ok": bool(rel <= tol),
              "rows_per_rank": int(rows_s.shape[0]), "hub_rows_per_rank": 8,
              "reference": "fp64 host sum over the sampled rows, same rounded inputs", "ranks": world}

    # ---- optional: the step followed by the all-gather of C over NVLink (NCCL), so
    # every rank holds the whole M x N product; reported beside value, not in it ----
    gather = None
    if args.gather and world > 1 and args.split != "2d":
        if args.split == "rows":
            counts = [None] * world
            dist.all_gather_object(counts, int(mrows))
            Cfull = torch.empty((world, max(counts), ncols), dtype=Cd.dtype, device=dev)  # row blocks, padded
            parts = list(Cfull.unbind(0))
        else:
            b0 = T.partition_columns(N, dt, world, 0)[1]  # block width (the last block may be narrower)
            Cfull = torch.empty((world, M, b0), dtype=Cd.dtype, device=dev)
            parts = list(Cfull.unbind(0))
        Cpad = torch.zeros(parts[rank].shape, dtype=Cd.dtype, device=dev)

        Cview = Cpad[:mrows, :ncols]

        def gathered_step():
            plan.execute1(Bd, Cview, stream, epilogue=ep)  # straight into the send buffer
            dist.all_gather(parts, Cpad)

        for _ in range(3):
            gathered_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gsteps = max(5, min(args.steps, 50))
        e0.record(stream)
        for _ in range(gsteps):
            gathered_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        gms = max_over_ranks(e0.elapsed_time(e1) / gsteps)
        gather = {"ms_per_step": round(gms, 5), "collective": "all_gather of C blocks (NCCL)",
                  "bytes_per_rank": int(M * N * Cd.element_size())}

    # ---- end to end through the public API: every step copies its B from pinned
    # host memory, executes, and reads its C back into pinned host memory.  The
    # steps are pipelined over three streams with two device B and C buffers:
    # step i's host-to-device copy overlaps step i-1's product and step i-2's
    # device-to-host copy (PCIe moves both directions at once). ----
    Bpin = Bh.pin_memory()
    Cpins = [torch.empty((mrows, ncols), dtype=cdt).pin_memory() for _ in range(2)]
    Bds = [Bd, torch.empty_like(Bd)]
    Cds = [Cd, torch.empty_like(Cd)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for k in range(2):  # buffers start free
        ev_comp[k].record(stream)
        ev_out[k].record(stream)
    e2e_steps = max(3, min(args.steps, 50))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(e2e_steps):
        k = i & 1
        s_in.wait_event(ev_comp[k])  # B buffer k no longer read by step i-2
        with torch.cuda.stream(s_in):
            Bds[k].copy_(Bpin, non_blocking=True)
        ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_out[k])  # C buffer k already read back (step i-2)
        plan.execute1(Bds[k], Cds[k], stream, epilogue=ep)
        ev_comp[k].record(stream)
        s_out.wait_event(ev_comp[k])
        with torch.cuda.stream(s_out):
            Cpins[k].copy_(Cds[k], non_blocking=True)
        ev_out[k].record(s_out)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    del Bds[1], Cds[1]
    # Row split: every rank copies all of B; 2-D: every row block copies all of B.
    h2d = K * N * elem * (world if args.split == "rows" else grid[0] if args.split == "2d" else 1)
    d2h = M * N * (2 if args.epilogue else 4)

    # ---- library baselines on this rank's block (reported, not targets), timed
    # with the same L2 protocol as the step above ----
    T.baselines_set_flush(flush)
    Cs = torch.empty_like(Cd, dtype=torch.float32)
    try:
        ms_cusparse = max_over_ranks(T.cusparse_spmm(plan, Bd, Cs, warmup=3, iters=max(5, min(args.steps, 50)),
                                                     stream=stream))
        cs_err = float((Cs - Cd).norm() / max(Cd.norm(), 1e-30)) if ep is None else None
    except Exception as e:  # reported
        ms_cusparse, cs_err = None, str(e)
    # Blocked-ELL (32 x 32 blocks) where A is small enough to be dense-ish (C1 / C2 shapes).
    bell = None
    if dt in ("f16", "bf16") and M * K <= 1 << 26 and args.split == "columns" and ep is None:
        try:
            Cb = torch.empty_like(Cd, dtype=torch.float32)
            bell_ms, _ = T.cusparse_blocked_ell(A, 32, Bd, Cb, dt, warmup=3, iters=max(5, min(args.steps, 50)),
                                                stream=stream) if world == 1 else (None, None)
            bell = {"ms": bell_ms, "block": 32,
                    "rel_diff": float((Cb - Cd).norm() / max(Cd.norm(), 1e-30)) if bell_ms else None}
        except Exception as e:  # reported
            bell = {"error": str(e)}
    gemm = None
    if M * K * elem <= 2**31 and args.split == "columns" and ep is None:
        Ad = torch.zeros((M, K), dtype=tdt, device=dev)
        rows = torch.from_numpy(np.repeat(np.arange(M), np.diff(A.row_ptr))).to(dev)
        Ad[rows, torch.from_numpy(A.col.astype(np.int64)).to(dev)] = torch.from_numpy(A.values()).to(dev).to(tdt)
        Cg = torch.empty_like(Cd)
        gemm = max_over_ranks(T.cublas_gemm(Ad, Bd, Cg, dt, warmup=3, iters=20, stream=stream))
    # The per-nonzero gather floor: the same B-row gathers with no arithmetic and no C
    # write, timed alone under the same L2 protocol (what any SpMM that gathers each
    # nonzero's B row needs at least on this GPU).
    try:
        ms_gather = max_over_ranks(T.gather_floor(plan, Bd, warmup=3, iters=max(5, min(args.steps, 30)),
                                                  stream=stream))
    except Exception as e:  # reported
        ms_gather = str(e)
    T.baselines_set_flush(None)

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if affinity_before is not None:
        os.sched_setaffinity(0, affinity_before)  # the CPU baseline uses every host core
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        Bf = Bfull.astype(np.float32) if dt != "bf16" else torch.from_numpy(Bfull.view(np.int16)).view(
            torch.bfloat16).float().numpy()
        threads = host_threads()
        v, sample = cpu_reference(A, Bf, threads)
        cpu = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    peak, peak_kind = load_peaks()
    alg = algorithmic_bytes(M, K, nnz, N, elem)
    if args.epilogue:  # 16-bit C, plus the row scales and the bias
        alg += -M * N * 2 + M * 4 + N * 4
    achieved = alg / (ms_step * 1e-3) / 1e9
    kernels_per_step = (1 if pst["residue_row_warps"] + pst["residue_segments"] > 0 else 0) + (
        1 if pst["tc_windows"] > 0 else 0)
    c1 = None
    if world == 1 and args.workload == "gcn" and not args.no_c1:
        try:
            c1 = measure_c1(T, torch, dev)
        except Exception as e:  # reported
            c1 = {"error": str(e)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": dt, "data": "synthetic",
            "config": {"workload": desc, "M": M, "K": K, "N": N, "nnz": nnz,
                       "parallelism": f"column shards x{world} (A replicated, no data-path collective)"
                       if args.split == "columns" else
                       f"row shards x{world} (A split by rows, B replicated, no data-path collective)"
                       if args.split == "rows" else
                       f"2-D shards {grid[0]}x{grid[1]} (row blocks of A x column blocks of B, no data-path "
                       f"collective)",
                       "l2": "flushed between steps (2x L2 buffer)" if flush is not None
                       else "inputs larger than L2 (126 MB)",
                       "launch": "CUDA graph of the plan's launches" if graph is not None
                       else "direct C-ABI execute per step",
                       "host": "bound to the GPU's local CPUs" if affinity_before is not None else "unbound",
                       "preprocess_ms": round(pst["preprocess_ms"], 3), "upload_ms": round(pst["upload_ms"], 3),
                       "tc_windows": pst["tc_windows"], "residue_segments": pst["residue_segments"],
                       **({"epilogue": "C = relu(row_scale * (A B) + bias) stored as bf16"} if args.epilogue
                          else {})},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": load_traffic(args.workload, profiled_config=(
                             dt == wl[3] and N == wl[2] and not args.epilogue and world == 1
                             and args.split == "columns"
                             and not any(k.startswith("TCASPMM_") for k in os.environ))),
                         "peak_kind": peak_kind, "algorithmic_bytes": alg,
                         "kernel": "residue_kernel" if pst["tc_windows"] == 0 else "tc + residue"},
            "roofline_gather": {
                "bound": "L2-to-SM gathers: every nonzero's B row slice, loaded alone (tcaspmm_gather_floor)",
                "floor_ms": round(ms_gather, 5) if isinstance(ms_gather, float) else ms_gather,
                "kernel_ms": round(ms_step, 5),
                "frac": round(ms_gather / ms_step, 4) if isinstance(ms_gather, float) else None,
                "gathered_bytes": int(pst["nnz"]) * ncols * elem if args.split == "columns" else None},
            "e2e": {"value": round(flops / (ms_e2e * 1e-3) / 1e9, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 4),
                    "pipeline": "copy-in, execute, copy-out on three streams, two device buffers"},
            "baselines": {"spmm_cusparse_ms": ms_cusparse, "spmm_cusparse_rel_diff": cs_err,
                          "gemm_cublas_ms": gemm, "spmm_cusparse_blocked_ell": bell,
                          "timing": "same L2 protocol as value (flushed between calls)" if flush is not None
                          else "back to back, inputs larger than L2",
                          "spmm_cusparse_gflops": round(flops / (ms_cusparse * 1e-3) / 1e9, 3)
                          if isinstance(ms_cusparse, float) else None},
            "cpu_baseline": cpu,
            "parity": parity,
            **({"c1": c1} if c1 else {}),
            **({"with_gather": gather} if gather else {}),
            "clocks": sampler.summary(),
            "gpu_launches": kernels_per_step * args.steps * world,
        }
        print(json.dumps(line), flush=True)
    del graph  # holds the plan's launches: released before the plan
    plan.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
