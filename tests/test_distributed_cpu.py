"""Host-side logic of the row-sharded multi-GPU path, run as gloo ranks on CPU.

The row split (appt_split_rows, host code of the library) is checked against a restatement, and
2 and 3 gloo ranks each compute their row block of C with the CPU oracle standing in for the
per-GPU engine call. torch.distributed carries what NCCL carries on the GPU path -- the
replication of B and the exchange of the ranks' nnz -- and rank 0 assembles the blocks with the
library's block_offsets / assemble_blocks and compares them with the unsharded product.
"""
import os
import socket

import numpy as np
import pytest

from appt_spgemm import distributed as D
from appt_spgemm import matrices as M


def _split_restated(products, parts):
    """Cut r at the prefix nearest to r/parts of the total (ties to the earlier cut), cuts
    non-decreasing."""
    cum = np.concatenate([[0], np.cumsum(np.asarray(products, np.int64))])
    total = int(cum[-1])
    out = [0]
    for r in range(1, parts):
        t = total * r / parts
        b = int(np.searchsorted(cum, t, side="left"))
        if b > 0 and t - cum[b - 1] <= cum[min(b, cum.size - 1)] - t:
            b -= 1
        out.append(max(out[-1], b))
    out.append(len(products))
    return out


def test_split_rows_balances_products():
    rng = np.random.default_rng(0)
    flops = rng.integers(0, 1000, 10_000)
    for world in (1, 2, 3, 4, 8):
        b = D.split_rows(flops, world)
        assert b == _split_restated(flops, world)
        assert b[0] == 0 and b[-1] == flops.size and len(b) == world + 1
        assert all(x <= y for x, y in zip(b, b[1:]))
        parts = [int(flops[b[r]:b[r + 1]].sum()) for r in range(world)]
        assert max(parts) - min(parts) <= 2 * int(flops.max())


def test_split_rows_skewed_and_degenerate():
    zipf = np.minimum(np.random.default_rng(1).zipf(1.3, 50_000), 10**7)
    for world in (2, 8):
        assert D.split_rows(zipf, world) == _split_restated(zipf, world)
    assert D.split_rows(np.zeros(5, np.int64), 4)[-1] == 5
    b = D.split_rows(np.array([0, 0, 100, 0]), 2)
    assert b[0] == 0 and b[-1] == 4
    assert D.split_rows(np.zeros(0, np.int64), 2) == [0, 0, 0]
    with pytest.raises(Exception):
        D.split_rows(np.array([3, -1, 2]), 2)


def test_block_offsets_and_assembly():
    assert D.block_offsets([3, 0, 5]).tolist() == [0, 3, 3, 8]
    import oracle
    A = M.random_csr(120, 120, 0.06, 2)
    full = oracle.spgemm(A)
    bounds = [0, 50, 50, 120]
    blocks = []
    for r in range(3):
        r0, r1 = bounds[r], bounds[r + 1]
        blk = M.Csr(r1 - r0, A.cols, A.row_ptr[r0:r1 + 1], A.col_idx, A.val)
        C = oracle.spgemm(blk, A)
        blocks.append(M.Csr(C.rows, C.cols, C.row_ptr - C.row_ptr[0], C.col_idx, C.val))
    offs = D.block_offsets([b.nnz for b in blocks])
    got = D.assemble_blocks(bounds, A.cols, blocks, offs)
    assert np.array_equal(got.row_ptr, full.row_ptr)
    assert np.array_equal(got.col_idx, full.col_idx)
    assert np.array_equal(got.val, full.val)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, op, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        A0 = M.random_csr(301, 301 if op == "ab" else 97, 0.05, 5, empty_rows=0.1)
        # replicate A from rank 0 (the broadcast of the B operand)
        t = [torch.from_numpy(A0.row_ptr.copy()), torch.from_numpy(A0.col_idx.copy()),
             torch.from_numpy(A0.val.copy())]
        if rank != 0:
            t = [torch.zeros_like(x) for x in t]
        for x in t:
            dist.broadcast(x, 0)
        A = M.Csr(A0.rows, A0.cols, t[0].numpy(), t[1].numpy(), t[2].numpy())
        B = oracle.transpose(A) if op == "aat_upper" else A
        b = D.split_rows(oracle.row_products(A, B), world)
        r0, r1 = b[rank], b[rank + 1]
        blk = M.Csr(r1 - r0, A.cols, A.row_ptr[r0:r1 + 1], A.col_idx, A.val)
        C = oracle.spgemm(blk, B, op="ab" if op == "ab" else "ab_upper", row_base=r0)
        # the nnz exchange
        nnz = [None] * world
        dist.all_gather_object(nnz, int(C.nnz))
        offs = D.block_offsets(nnz)
        payload = [None] * world
        dist.all_gather_object(payload, (C.row_ptr - C.row_ptr[0], C.col_idx, C.val))
        if rank == 0:
            full = oracle.spgemm(A, op=op)
            blocks = [M.Csr(b[r + 1] - b[r], full.cols, p[0], p[1], p[2])
                      for r, p in enumerate(payload)]
            got = D.assemble_blocks(b, full.cols, blocks, offs)
            ok = (np.array_equal(got.row_ptr, full.row_ptr) and
                  np.array_equal(got.col_idx, full.col_idx) and
                  np.array_equal(got.val, full.val) and offs[-1] == full.nnz)
            q.put(bool(ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("op", ["ab", "aat_upper"])
def test_gloo_ranks_assemble_the_full_product(op, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, op, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True
