"""Scaled-FP16 row transport (mirror of patches/tilelang_transport_tradeoffs.py and
patches/tilelang_transport_p2.py) on B200.

  encode:  P -> f16(f32(P) * 2^-shift)         (fused into the row GEMM epilogue)
  collect: fp16 SUM over ranks                  ('allreduce': NCCL all_reduce, or
                                                 'rowblock': all_to_all + fixed-order sum)
  finish:  restored = int(f32(S) * 2^shift); y = (restored * A) * W   (+ gated residual)

and the packed INT8 scheme 'int8_gather' (tilelang_transport_tradeoffs.py:40-88,
tilelang_transport_p2.py:28-42): per 128-column group an fp32 scale max|P|/127 and
INT8 codes, gathered, then restored = rint(sum_w q_w * s_w) in rank order.

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
    if scheme == "int8_gather":
        return ops.pack8(partial)
    if scheme != "fp16":
        raise ValueError(scheme)
    return ops.fp16_encode(partial, shift_for(local_k, world_size))


def collect(payload: torch.Tensor, scheme: str, comm) -> torch.Tensor:
    """NCCL fp16 SUM, or the all-gather of the packed INT8 payloads in rank order
    ([world * rows, pitch] uint8) (tilelang_transport_p2.py:57-62)."""
    world = C.world_of(comm)
    if scheme == "int8_gather":
        if world == 1:
            return payload
        gathered = torch.empty((payload.shape[0] * world, payload.shape[1]), dtype=torch.uint8,
                               device=payload.device)
        comm.all_gather_into_tensor(gathered, payload.contiguous())
        return gathered
    if scheme != "fp16":
        raise ValueError(scheme)
    if world > 1:
        comm.all_reduce(payload, op=comm.ReduceOp.SUM)
    return payload


def finish(payload, activation_scale, weight_scale, scheme, local_k, world_size: int = 2,
           out_dtype=torch.float32):
    """Decode + FP32 dequant of a reduced payload (tilelang_transport_p2.py:65-69); for
    'int8_gather' the gathered payloads are reconstructed in rank order first."""
    if scheme == "int8_gather":
        rows = activation_scale.shape[0]
        width = weight_scale.numel()
        parts = payload.reshape(-1, rows, payload.shape[-1])
        return ops.unpack8_finish(parts, width, activation_scale, weight_scale, out_dtype)
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
    if scheme == "int8_gather":
        with label("pack_INT8_with_scales"):
            payload = ops.pack8(partial)
        gathered = collect(payload, scheme, comm)
        with label("reconstruct_INT8_rank_order"):
            return ops.unpack8_finish(gathered.reshape(world, partial.shape[0], -1),
                                      partial.shape[1], out_dtype=torch.int32)
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
    if transport not in ("rowblock", "p2p", "nvls"):
        # 'p2p' / 'nvls' reach here only for the forms the peer kernels do not cover (no
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


def int8_row_exchange(q, weight, activation_scale, weight_scale, comm, transport: str = "p2p",
                      *, out_dtype=torch.float32, residual=None, gate=None, labels=None):
    """Row GEMM + the packed INT8 partial SUM ('int8_gather') + the row epilogue.

    The GEMM packs in its epilogue; the payloads are summed in rank order by
    p2p:       h3_peer_reduce_int8 / h3_peer_gather over NVLink peer memory (residual
               form, NCCL group);
    rowblock:  all_to_all of the packed row blocks, reconstruction + epilogue of the
               owned block, all_gather of the finished rows;
    allreduce: all_gather of the whole payloads and the reconstruction on every rank
               (the reference's form, tilelang_transport_p2.py:57-69)."""
    from . import peer as P
    world = C.world_of(comm)
    rows, width = q.shape[0], weight.shape[0]
    ws = weight_scale.reshape(-1)
    if (transport in ("p2p", "nvls") and world > 1 and residual is not None and residual.is_contiguous()
            and P.available(comm)):
        wsp = P.workspace(comm, q.device, width, rows)
        with label("int8_gemm_pack_int8"):
            ops.int8_gemm_row_pack8(q, weight, out=wsp.partial_u8(rows))
        with label("packed_int8_peer_reduce_gather"):
            return wsp.reduce_and_gather(rows, 0, activation_scale, ws, residual, gate, labels,
                                         packed=True)
    with label("int8_gemm_pack_int8"):
        payload = ops.int8_gemm_row_pack8(q, weight)
    if world > 1 and transport in ("rowblock", "p2p", "nvls"):
        with label("packed_int8_exchange"):
            parts, a, b = C.exchange_row_blocks(payload, comm)
        A = activation_scale.reshape(-1)[a:b]
        lab = None if labels is None else labels[a:b]
        with label("packed_int8_epilogue"):
            if residual is not None:
                block = ops.unpack8_finish(parts, width, A, ws, residual=residual[a:b], gate=gate,
                                           labels=lab)
                full = residual
            else:
                block = ops.unpack8_finish(parts, width, A, ws, out_dtype)
                full = torch.empty((rows, width), dtype=out_dtype, device=q.device)
        with label("packed_int8_gather"):
            return C.gather_row_blocks(block, full, comm)
    if transport not in ("rowblock", "p2p", "nvls", "allreduce"):
        raise ValueError("Unknown row transport")
    with label("packed_int8_all_gather"):
        gathered = collect(payload, "int8_gather", comm)
    parts = gathered.reshape(world, rows, -1)
    with label("packed_int8_epilogue"):
        if residual is not None:
            return ops.unpack8_finish(parts, width, activation_scale, ws, residual=residual,
                                      gate=gate, labels=labels)
        return ops.unpack8_finish(parts, width, activation_scale, ws, out_dtype)
