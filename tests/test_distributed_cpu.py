"""Host-side logic of the row-sharded multi-GPU path, run as 2 gloo ranks on CPU.

Each rank computes its row block of C with the CPU oracle standing in for the per-GPU engine
call (the logic under test is the partition, the replicated operand, the upper-triangle
row_base and the nnz-offset exchange), then rank 0 assembles the blocks and compares them with
the unsharded product.
"""
import os
import socket

import numpy as np
import pytest

from appt_spgemm import distributed as D
from appt_spgemm import matrices as M


def test_partition_rows_balances_products():
    rng = np.random.default_rng(0)
    flops = rng.integers(0, 1000, 10_000)
    for world in (1, 2, 3, 4, 8):
        b = D.partition_rows(flops, world)
        assert b[0] == 0 and b[-1] == flops.size and len(b) == world + 1
        assert all(x <= y for x, y in zip(b, b[1:]))
        parts = [int(flops[b[r]:b[r + 1]].sum()) for r in range(world)]
        assert max(parts) - min(parts) <= 2 * int(flops.max())


def test_partition_rows_degenerate():
    assert D.partition_rows(np.zeros(5, np.int64), 4) == [0, 0, 0, 0, 5] or \
        D.partition_rows(np.zeros(5, np.int64), 4)[-1] == 5
    b = D.partition_rows(np.array([0, 0, 100, 0]), 2)
    assert b[0] == 0 and b[-1] == 4
    assert D.partition_rows(np.zeros(0, np.int64), 2) == [0, 0, 0]


def test_block_offsets():
    assert D.block_offsets([3, 0, 5]).tolist() == [0, 3, 3, 8]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, op, q):
    import torch.distributed as dist
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        A0 = M.random_csr(301, 301 if op == "ab" else 97, 0.05, 5, empty_rows=0.1)
        # replicate A from rank 0 (as the B operand broadcast)
        t = [torch.from_numpy(A0.row_ptr.copy()), torch.from_numpy(A0.col_idx.copy()),
             torch.from_numpy(A0.val.copy())]
        if rank != 0:
            t = [torch.zeros_like(x) for x in t]
        D.replicate(dist, t, 0)
        A = M.Csr(A0.rows, A0.cols, t[0].numpy(), t[1].numpy(), t[2].numpy())
        B = oracle.transpose(A) if op == "aat_upper" else A
        flops = oracle.row_products(A, B)
        b = D.partition_rows(flops, world)
        r0, r1 = b[rank], b[rank + 1]
        blk = M.Csr(r1 - r0, A.cols, A.row_ptr[r0:r1 + 1], A.col_idx, A.val)
        C = oracle.spgemm(blk, B, op="ab" if op == "ab" else "ab_upper", row_base=r0)
        offs = D.exchange_nnz(dist, C.nnz, torch.device("cpu"))
        grp = D.global_row_ptr(C.row_ptr - C.row_ptr[0], offs[rank])
        # point-to-point assembly on rank 0 (the library's gather helper)
        got = D.gather_csr(dist, b, A.cols,
                           torch.from_numpy(np.asarray(C.row_ptr - C.row_ptr[0], np.int64)),
                           torch.from_numpy(np.ascontiguousarray(C.col_idx, np.int32)),
                           torch.from_numpy(np.ascontiguousarray(C.val)), offs, dst=0)
        payload = [None] * world
        dist.all_gather_object(payload, (r0, r1, grp, C.col_idx, C.val))
        if rank == 0:
            full = oracle.spgemm(A, op=op)
            rp = np.zeros(A.rows + 1, np.int64)
            cols, vals = [], []
            for (a0, a1, g, c, v) in payload:
                rp[a0:a1 + 1] = g
                cols.append(c)
                vals.append(v)
            ok = (np.array_equal(rp, full.row_ptr) and
                  np.array_equal(np.concatenate(cols), full.col_idx) and
                  np.array_equal(np.concatenate(vals), full.val) and offs[-1] == full.nnz)
            grp_, gci, gva = got
            ok = ok and (np.array_equal(grp_.numpy(), full.row_ptr) and
                         np.array_equal(gci.numpy(), full.col_idx) and
                         np.array_equal(gva.numpy(), full.val))
            q.put(bool(ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("op", ["ab", "aat_upper"])
def test_two_gloo_ranks_assemble_the_full_product(op):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, op, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True
