"""Scaled-FP16 row transport (mirror of patches/tilelang_transport_tradeoffs.py and
patches/tilelang_transport_p2.py) on B200.

  encode:  P -> f16(f32(P) * 2^-shift)         (fused into the row GEMM epilogue)
  collect: fp16 SUM over ranks                  ('allreduce': NCCL all_reduce, or
                                                 'rowblock': all_to_all + fixed-order sum)
  finish:  restored = int(f32(S) * 2^shift); y = (restored * A) * W   (+ gated residual)

The shift generalises shift_for(local_k) (tilelang_transport_tradeoffs.py:20-22), which
hard-codes two ranks, to shift_for_full(K) = max(0, ceil(log2(K * 127^2 / 60000))) on
the full reduction length K = local_k * world_size; both agree at TP=2.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch

from . import comm as C
from . import ops


@contextmanager
def label(name: str):
    """NVTX range 'linear/<name>' (tilelang_transport_tradeoffs.py:13-17)."""
    torch.cuda.nvtx.range_push("linear/" + name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def shift_for(local_k: int, world_size: int = 2) -> int:
    return ops.transport_shift(int(local_k) * int(world_size))


def encode(partial: torch.Tensor, scheme: str, local_k: int, world_size: int = 2) -> torch.Tensor:
    """Standalone encode of an INT32 partial (tilelang_transport_p2.py:50-54)."""
    if scheme != "fp16":
        raise ValueError(scheme)
    return ops.fp16_encode(partial, shift_for(local_k, world_size))


def collect(payload: torch.Tensor, scheme: str, comm) -> torch.Tensor:
    """NCCL fp16 SUM (tilelang_transport_p2.py:57-58)."""
    if scheme != "fp16":
        raise ValueError(scheme)
    if C.world_of(comm) > 1:
        comm.all_reduce(payload, op=comm.ReduceOp.SUM)
    return payload


def finish(payload, activation_scale, weight_scale, scheme, local_k, world_size: int = 2,
           out_dtype=torch.float32):
    """Decode + FP32 dequant of a reduced payload (tilelang_transport_p2.py:65-69)."""
    if scheme != "fp16":
        raise ValueError(scheme)
    return ops.row_reduce_finish(payload, shift_for(local_k, world_size), activation_scale,
                                 weight_scale, out_dtype)


def reduce(partial: torch.Tensor, comm, scheme: str, local_k: int) -> torch.Tensor:
    """tilelang_transport_tradeoffs.reduce: INT32 partial -> reduced INT32."""
    world = C.world_of(comm)
    if partial.dtype != torch.int32 or not partial.is_contiguous():
        raise ValueError("Contiguous INT32 partial required")
    if scheme == "int32":
        if world > 1:
            comm.all_reduce(partial, op=comm.ReduceOp.SUM)
        return partial
    if scheme == "fp16":
        shift = shift_for(local_k, world)
        with label("encode_fp16"):
            payload = ops.fp16_encode(partial, shift)
        if world > 1:
            comm.all_reduce(payload, op=comm.ReduceOp.SUM)
        with label("decode_fp16"):
            return ops.fp16_decode(payload, shift)
    raise ValueError("Unknown transport scheme")


def reduce_and_finish(payload: torch.Tensor, comm, shift: int, activation_scale, weight_scale,
                      *, transport: str = "rowblock", out_dtype=torch.float32, residual=None,
                      gate=None, labels=None):
    """Sums the per-rank fp16 partial `payload` [M, N] over the TP group and applies
    the fused epilogue.  With `residual` the gated residual is updated in place on every
    rank and returned; otherwise the [M, N] output in out_dtype is returned."""
    world = C.world_of(comm)
    if world == 1 or transport == "allreduce":
        if world > 1:
            with label("scaled_fp16_sum"):
                comm.all_reduce(payload, op=comm.ReduceOp.SUM)
        with label("scaled_fp16_fused_epilogue"):
            return ops.row_reduce_finish(payload, shift, activation_scale, weight_scale, out_dtype,
                                         residual=residual, gate=gate, labels=labels)
    if transport not in ("rowblock", "p2p"):
        # 'p2p' reaches here only for the forms the peer kernels do not cover (no
        # residual, or a non-NCCL comm); the row-block exchange gives the same bits.
        raise ValueError("Unknown row transport")
    with label("scaled_fp16_exchange"):
        parts, a, b = C.exchange_row_blocks(payload, comm)
    rows, n = payload.shape
    A = activation_scale.reshape(-1)[a:b]
    lab = None if labels is None else labels[a:b]
    with label("scaled_fp16_fused_epilogue"):
        if residual is not None:
            block = ops.row_reduce_finish(parts, shift, A, weight_scale, residual=residual[a:b],
                                          gate=gate, labels=lab)
            full = residual
        else:
            block = ops.row_reduce_finish(parts, shift, A, weight_scale, out_dtype)
            full = torch.empty((rows, n), dtype=out_dtype, device=payload.device)
    with label("scaled_fp16_gather"):
        return C.gather_row_blocks(block, full, comm)
