"""The multi-GPU C entry points (appt_comm_*) on real GPUs, against the CPU oracle.

With one GPU a one-rank communicator still runs every step of the sharded path -- the NCCL
broadcast of B, the row split, the per-block product with its nnz all-gather -- on two row blocks
in turn, with device and with host A blocks (the end-to-end form), and the blocks are stitched
with the published offsets. With two or more GPUs, two ranks (one process per GPU) compute the
product together, and a rank whose block fails (an operand index out of range, detected on the
device and reported as an error, no fault) makes the other rank's call fail instead of hang.
"""
import os

import numpy as np
import pytest

from conftest import abs_product, assert_same_structure, assert_values_close, to_device

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
import oracle  # noqa: E402
from appt_spgemm import distributed as D  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402


def _spec(A, t):
    return (A.rows, A.cols, A.nnz, t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr())


def _block_spec(A, t, r0, r1):
    rp = np.asarray(A.row_ptr, np.int64)
    return (r1 - r0, A.cols, int(rp[r1] - rp[r0]), t[0].data_ptr() + 4 * r0, t[1].data_ptr(),
            t[2].data_ptr())


def _host_block(A, r0, r1):
    return M.Csr(r1 - r0, A.cols, np.asarray(A.row_ptr[r0:r1 + 1]), A.col_idx, A.val)


@pytest.mark.parametrize("op", ["ab", "ab_upper"])
@pytest.mark.parametrize("a_where", ["device", "host"])
def test_one_rank_two_blocks_match_oracle(op, a_where):
    torch = pytest.importorskip("torch")
    comm = D.Communicator(D.Communicator.unique_id(), 1, 0, 0)
    try:
        A = M.stencil27(g=28) if op == "ab" else M.random_csr(900, 300, 0.03, 4, empty_rows=0.1)
        B = A if op == "ab" else oracle.transpose(A)
        tA, tB = to_device(torch, A), to_device(torch, B)
        specB, ms, owned = comm.broadcast_csr(0, _spec(B, tB))
        assert not owned and ms >= 0.0
        assert comm.row_split(0, _spec(A, tA), specB) == [0, A.rows]
        bounds = D.split_rows(oracle.row_products(A, B), 2)
        blocks = []
        for r0, r1 in zip(bounds[:-1], bounds[1:]):
            blk = _host_block(A, r0, r1) if a_where == "host" else _block_spec(A, tA, r0, r1)
            C, offs = comm.spgemm(blk, specB, op=op, row_base=r0, out="host")
            assert offs.tolist() == [0, C.nnz]
            blocks.append(C)
        got = D.assemble_blocks(bounds, B.cols, blocks, D.block_offsets([c.nnz for c in blocks]))
        full_op = "ab" if op == "ab" else "aat_upper"
        R = oracle.spgemm(A, op=full_op)
        assert_same_structure(got, R)
        assert_values_close(got, R, abs_product(A, op=full_op))
    finally:
        comm.destroy()


def _rank_main(rank, world, uid, fail_rank, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    torch.cuda.set_device(rank)
    try:
        comm = D.Communicator(uid, world, rank, rank)
        A = M.stencil27(g=30)
        spec = None
        tA = None
        if rank == 0:
            tA = to_device(torch, A, rank)
            spec = _spec(A, tA)
        specA, _, owned = comm.broadcast_csr(0, spec)
        bounds = comm.row_split(0, specA if rank == 0 else None)
        r0, r1 = bounds[rank], bounds[rank + 1]
        rp = np.asarray(A.row_ptr, np.int64)
        blk = (r1 - r0, A.cols, int(rp[r1] - rp[r0]), specA[3] + 4 * r0, specA[4], specA[5])
        bad = None
        if rank == fail_rank:   # a column index past B's rows: the engine reports an error
            ci = np.asarray(A.col_idx[rp[r0]:rp[r1]]).copy()
            ci[len(ci) // 2] = A.rows + 5
            bad = torch.from_numpy(ci).to(torch.device("cuda", rank))
            rpb = torch.from_numpy((rp[r0:r1 + 1] - rp[r0]).astype(np.int32)).to(bad.device)
            vb = torch.from_numpy(np.asarray(A.val[rp[r0]:rp[r1]])).to(bad.device)
            blk = (r1 - r0, A.cols, int(rp[r1] - rp[r0]), rpb.data_ptr(), bad.data_ptr(),
                   vb.data_ptr())
        try:
            C, offs = comm.spgemm(blk, specA, row_base=r0, out="host")
            q.put((rank, "ok", bounds, C.row_ptr, C.col_idx, C.val, offs))
        except ap.ApptError as e:
            q.put((rank, "error", str(e)))
        if owned:
            comm.free_csr(specA)
        comm.destroy()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "exception", repr(e)))


def _run_ranks(world, fail_rank):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    uid = D.Communicator.unique_id()
    procs = [ctx.Process(target=_rank_main, args=(r, world, uid, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        item = q.get(timeout=600)
        out[item[0]] = item
    for p in procs:
        p.join(timeout=120)
    return out


def test_two_ranks_match_oracle():
    if ap.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = _run_ranks(2, fail_rank=-1)
    assert all(v[1] == "ok" for v in out.values()), out
    A = M.stencil27(g=30)
    bounds = out[0][2]
    offs = out[0][6]
    assert np.array_equal(offs, out[1][6])
    blocks = [M.Csr(bounds[r + 1] - bounds[r], A.cols, out[r][3], out[r][4], out[r][5])
              for r in range(2)]
    got = D.assemble_blocks(bounds, A.cols, blocks, offs)
    R = oracle.spgemm(A)
    assert_same_structure(got, R)
    assert_values_close(got, R, abs_product(A))


def test_failed_rank_fails_the_others_without_hanging():
    if ap.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = _run_ranks(2, fail_rank=1)
    assert out[1][1] == "error" and "out of range" in out[1][2], out[1]
    assert out[0][1] == "error" and "another rank" in out[0][2], out[0]
