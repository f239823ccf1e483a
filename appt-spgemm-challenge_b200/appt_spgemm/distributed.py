"""Row-sharded multi-GPU SpGEMM plumbing (one process per GPU, torch.distributed).

The reference is single-GPU (src/main.cu:44 pins device 0). Here rows of A are independent
units: each rank computes a contiguous block of rows of C, the blocks balanced by
intermediate-product count; B (or A^T) is replicated to every GPU once with an NCCL broadcast,
and the only per-product collective is an all-gather of each rank's nnz(C block), from which
every rank derives the global row offsets of its block. C stays sharded.

Everything here is host-side logic on top of the C ABI; the per-rank compute is the engine's
device-pointer entry point (appt_spgemm with APPT_MEM_DEVICE operands).
"""
from __future__ import annotations

import numpy as np


def partition_rows(row_products: np.ndarray, world: int) -> list[int]:
    """Contiguous row bounds [b_0 = 0, b_1, ..., b_world = rows] splitting the cumulative
    products as evenly as contiguous blocks allow (prefix-balanced)."""
    rows = int(row_products.shape[0])
    if world <= 0:
        raise ValueError("world must be positive")
    cum = np.concatenate([[0], np.cumsum(np.asarray(row_products, dtype=np.int64))])
    total = int(cum[-1])
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        b = int(np.searchsorted(cum, target, side="left"))
        # take the closer of the two candidate cut points
        if b > 0 and abs(cum[b - 1] - target) <= abs(cum[min(b, rows)] - target):
            b -= 1
        bounds.append(max(bounds[-1], min(b, rows)))
    bounds.append(rows)
    return bounds


def block_offsets(nnz_per_rank) -> np.ndarray:
    """Exclusive prefix of the ranks' nnz(C block): the global offset of each block's first
    entry (int64), plus the total as the last element."""
    v = np.asarray(nnz_per_rank, dtype=np.int64)
    out = np.zeros(v.size + 1, dtype=np.int64)
    np.cumsum(v, out=out[1:])
    return out


def exchange_nnz(dist, my_nnz: int, device) -> np.ndarray:
    """All-gather of every rank's int64 nnz (one collective); returns block_offsets()."""
    import torch
    world = dist.get_world_size()
    mine = torch.tensor([int(my_nnz)], dtype=torch.int64, device=device)
    parts = [torch.empty(1, dtype=torch.int64, device=device) for _ in range(world)]
    dist.all_gather(parts, mine)
    return block_offsets(torch.cat(parts).cpu().numpy())


def exchange_nnz_into(dist, my_nnz: int, out) -> None:
    """The same all-gather into a preallocated int64 tensor of world_size entries, without
    waiting for it on the host (block_offsets(out.cpu().numpy()) gives the offsets later)."""
    import torch
    mine = torch.full((1,), int(my_nnz), dtype=torch.int64, device=out.device)
    dist.all_gather_into_tensor(out, mine)


def replicate(dist, tensors, src: int = 0) -> None:
    """Broadcast operand arrays (already allocated with the right sizes on every rank)."""
    for t in tensors:
        dist.broadcast(t, src)


def global_row_ptr(local_row_ptr: np.ndarray, offset: int) -> np.ndarray:
    """Row pointers of a block shifted to global entry positions."""
    return np.asarray(local_row_ptr, dtype=np.int64) + int(offset)


def gather_csr(dist, bounds, cols: int, row_ptr, col_idx, val, offsets, dst: int = 0):
    """Assemble the sharded C on rank `dst` with point-to-point transfers: every rank passes its
    block (row_ptr relative to the block, starting at 0, as int64; col_idx int32; val float64 --
    torch tensors on the rank's device for NCCL, on the CPU for gloo) and `offsets` from
    exchange_nnz. Returns (row_ptr int64, col_idx, val) of the whole C on `dst`, None elsewhere.
    All ranks must call it."""
    import torch
    rank, world = dist.get_rank(), dist.get_world_size()
    if rank != dst:
        dist.send(row_ptr.contiguous(), dst)
        if int(offsets[rank + 1] - offsets[rank]) > 0:
            dist.send(col_idx.contiguous(), dst)
            dist.send(val.contiguous(), dst)
        return None
    rows = int(bounds[-1])
    total = int(offsets[-1])
    dev = col_idx.device
    rp = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    ci = torch.empty(total, dtype=torch.int32, device=dev)
    va = torch.empty(total, dtype=torch.float64, device=dev)
    for r in range(world):
        r0, r1 = int(bounds[r]), int(bounds[r + 1])
        e0, e1 = int(offsets[r]), int(offsets[r + 1])
        if r == dst:
            brp, bci, bva = row_ptr, col_idx, val
        else:
            brp = torch.empty(r1 - r0 + 1, dtype=torch.int64, device=dev)
            dist.recv(brp, r)
            bci, bva = None, None
            if e1 > e0:
                bci = torch.empty(e1 - e0, dtype=torch.int32, device=dev)
                bva = torch.empty(e1 - e0, dtype=torch.float64, device=dev)
                dist.recv(bci, r)
                dist.recv(bva, r)
        rp[r0:r1 + 1] = brp.to(dev) + e0
        if e1 > e0:
            ci[e0:e1] = bci
            va[e0:e1] = bva
    return rp, ci, va
