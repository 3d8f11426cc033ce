"""Column and row sharding across ranks, host side, on CPU with gloo (world size 2).

Each rank takes its column block from tcaspmm_partition_columns, checks that its
schedule covers every nonzero once (the plan each rank would build), and computes
its C block with the oracle; the gathered blocks must equal the unsharded result,
and a rank that fails is reported to the others through the store, not a hang.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, N, dt, result_q):
    import sys

    sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..")))
    import oracle
    import spmm_b200 as T

    from datetime import timedelta

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        A = T.gen_rmat(12, 30000, kind="gcn", seed=7)
        B = T.gen_dense(A.ncol, N, 5, "f32")
        b, c = T.partition_columns(N, dt, world, rank)
        cover, _, _ = T.schedule_coverage(A, c, dt)
        assert np.all(cover == 1)
        blk = oracle.spmm_f64(A.row_ptr, A.col, A.values(), B[:, b:b + c]) if c else np.zeros((A.nrow, 0))
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([c], dtype=torch.int64))
        width = int(max(s.item() for s in sizes))
        pad = np.zeros((A.nrow, width))
        pad[:, :c] = blk
        gathered = [torch.zeros((A.nrow, width), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(pad))
        if rank == 0:
            full = np.hstack([g.numpy()[:, : int(s.item())] for g, s in zip(gathered, sizes)])
            ref = oracle.spmm_f64(A.row_ptr, A.col, A.values(), B)
            result_q.put(("ok", float(np.abs(full - ref).max()), [int(s.item()) for s in sizes]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N,dt", [(128, "f32"), (256, "f16"), (20, "f32")])
def test_column_shards_reassemble_the_full_product(N, dt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, N, dt, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    status, err, sizes = q.get(timeout=10)
    assert status == "ok" and err == 0.0
    assert sum(sizes) == N


def _row_worker(rank, world, port, N, result_q):
    import sys

    sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..")))
    import oracle
    import spmm_b200 as T

    from datetime import timedelta

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        A = T.gen_rmat(12, 30000, kind="gcn", seed=8)
        B = T.gen_dense(A.ncol, N, 6, "f32")
        rb = T.partition_rows(A, world)
        r0, r1 = int(rb[rank]), int(rb[rank + 1])
        # The row block a row-split plan builds: rebased offsets, A's columns and values.
        base = int(A.row_ptr[r0])
        sub = T.CSR(r1 - r0, A.ncol, A.row_ptr[r0:r1 + 1] - base, A.col[base:A.row_ptr[r1]],
                    A.values()[base:A.row_ptr[r1]])
        cover, _, _ = T.schedule_coverage(sub, N, "f16")
        assert np.all(cover == 1)
        blk = oracle.spmm_f64(sub.row_ptr, sub.col, sub.values(), B)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([r1 - r0], dtype=torch.int64))
        height = int(max(s.item() for s in sizes))
        pad = np.zeros((height, N))
        pad[: r1 - r0] = blk
        gathered = [torch.zeros((height, N), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(pad))
        if rank == 0:
            full = np.vstack([g.numpy()[: int(s.item())] for g, s in zip(gathered, sizes)])
            ref = oracle.spmm_f64(A.row_ptr, A.col, A.values(), B)
            result_q.put(("ok", float(np.abs(full - ref).max()), [int(s.item()) for s in sizes]))
    finally:
        dist.destroy_process_group()


def test_row_shards_reassemble_the_full_product():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_worker, args=(r, 2, port, 64, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    status, err, sizes = q.get(timeout=10)
    assert status == "ok" and err == 0.0
    assert sum(sizes) == 4096 and min(sizes) > 0


def _failing_worker(rank, world, port, out_q):
    from datetime import timedelta

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    if rank == 1:
        store.set("rank1_status", "failed: plan_create raised")   # host-side failure, announced
        return
    out_q.put(store.get("rank1_status").decode())


def test_a_failing_rank_is_seen_through_the_store():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    assert q.get(timeout=10).startswith("failed")
