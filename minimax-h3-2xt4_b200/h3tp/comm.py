"""Collective steps of the row-parallel path.

`comm` is the reference's duck-typed collective object (patches/logical_dual_gpu.py:
22-114 and torch.distributed itself): get_rank(), get_world_size(), all_reduce(t, op),
ReduceOp, plus all_to_all_single / all_gather_into_tensor for the B200 row exchange.

The only large exchange of the path is the reduction of the FP16 row partials.  On
B200 it is done as a row-block reduce-scatter + all-gather instead of an all-reduce:

  1. all_to_all_single: rank r receives every rank's partial rows of block r;
  2. h3_row_reduce_finish on that block only: fixed rank-order FP32 sum, one fp16
     rounding, decode, dequant and the gated residual (1/t of the epilogue per rank);
  3. all_gather_into_tensor of the finished fp16 block (the updated residual rows).

The bytes over NVLink equal a ring all-reduce's, the sum order is fixed (so the
result is deterministic for any TP size), and at TP=2 it is bit-identical to the
reference's NCCL fp16 SUM + epilogue (one RN fp16 addition of two partials).
"""
from __future__ import annotations

import torch


def world_of(comm) -> int:
    if comm is None:
        return 1
    if hasattr(comm, "is_initialized") and not comm.is_initialized():
        return 1
    return int(comm.get_world_size())


def rank_of(comm) -> int:
    if comm is None or (hasattr(comm, "is_initialized") and not comm.is_initialized()):
        return 0
    return int(comm.get_rank())


def all_reduce_max(t: torch.Tensor, comm) -> torch.Tensor:
    """In-place MAX all-reduce of the [M, 1] row maxima (tilelang_swiglu_quant.py:87)."""
    if world_of(comm) > 1:
        comm.all_reduce(t, op=comm.ReduceOp.MAX)
    return t


def row_blocks(rows: int, world: int) -> list[tuple[int, int]]:
    """Row ranges [a, b) owned by each rank for the reduction (ceil-sized blocks)."""
    per = -(-rows // world) if rows else 0
    return [(min(rows, j * per), min(rows, (j + 1) * per)) for j in range(world)]


def exchange_row_blocks(payload: torch.Tensor, comm) -> tuple[torch.Tensor, int, int]:
    """Step 1: returns (parts [world, b-a, N] of this rank's block, a, b)."""
    world, rank = world_of(comm), rank_of(comm)
    rows, n = payload.shape
    blocks = row_blocks(rows, world)
    a, b = blocks[rank]
    counts = [e - s for s, e in blocks]
    recv = torch.empty((world * (b - a), n), dtype=payload.dtype, device=payload.device)
    comm.all_to_all_single(recv, payload.contiguous(), output_split_sizes=[b - a] * world,
                           input_split_sizes=counts)
    return recv.view(world, b - a, n), a, b


def gather_row_blocks(block: torch.Tensor, full: torch.Tensor, comm) -> torch.Tensor:
    """Step 3: gathers every rank's finished block into `full` [M, N] (in place when
    the blocks are equal sized and `block` is this rank's slice of `full`)."""
    world, rank = world_of(comm), rank_of(comm)
    rows, n = full.shape
    blocks = row_blocks(rows, world)
    per = blocks[0][1] - blocks[0][0]
    if per * world == rows and full.is_contiguous():
        a, b = blocks[rank]
        if block.data_ptr() != full[a:b].data_ptr():
            full[a:b].copy_(block)
        comm.all_gather_into_tensor(full, full[a:b])
        return full
    padded = torch.empty((world * per, n), dtype=full.dtype, device=full.device)
    mine = torch.zeros((per, n), dtype=full.dtype, device=full.device)
    mine[: block.shape[0]].copy_(block)
    comm.all_gather_into_tensor(padded, mine)
    for j, (s, e) in enumerate(blocks):
        if e > s:
            full[s:e].copy_(padded[j * per: j * per + (e - s)])
    return full
