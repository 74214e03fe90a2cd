"""Quantisation-preserving primitives of the TP blocks (mirror of
patches/parallel_int8.py) on B200.

gather / packed_rows are layout helpers; int_mm and dequantize run the sm_100a
kernels (exact INT32 tcgen05 GEMM; ((acc * a) * w) + bias dequant).  row_linear is
the exact full-gather route used when a rank's K-shard does not own whole 256-groups
(parallel_int8.py:72-94): every rank gathers the complete row, quantises it with
one global row maximum, multiplies its own K-slice and the INT32 partials are summed.
"""
from __future__ import annotations

import torch

from . import comm as C
from . import ops


def gather(x, comm, dim):
    """All-gather along `dim` (parallel_int8.py:7-23 / optimized_tp.fixed_gather).
    Returns (full, start, length) of this rank's slice."""
    world = C.world_of(comm)
    if world == 1:
        return x, 0, x.shape[dim]
    if dim not in (-1, x.ndim - 1):
        raise ValueError("Only the feature dimension is gathered")
    x = x.contiguous()
    parts = [torch.empty_like(x) for _ in range(world)]
    comm.all_gather(parts, x)
    return torch.cat(parts, dim=-1), C.rank_of(comm) * x.shape[-1], x.shape[-1]


def int_mm(q, weight):
    """Exact INT32 q @ weight.T (parallel_int8.py:46-50 / optimized_tp.native_int_mm);
    any row count, no padding."""
    return ops.int8_gemm_i32(q.reshape(-1, q.shape[-1]), weight)


def dequantize(accumulator, activation_scale, weight_scale, dtype, bias=None):
    """y = ((f32(acc) * a) * w) [+ bias], then cast (parallel_int8.py:53-69)."""
    out_dtype = torch.float16 if dtype == torch.float16 else torch.float32
    y = ops.dequantize_i32(accumulator, activation_scale, weight_scale, out_dtype, bias)
    return y if y.dtype == dtype else y.to(dtype)


def packed_rows(weight, scale, rank, world_size, components):
    """Component-packed row shard of a column weight (parallel_int8.py:97-103):
    rank r owns rows [c*chunk + r*chunk/t, c*chunk + (r+1)*chunk/t) of every component c."""
    if weight.shape[0] % (components * world_size):
        raise ValueError("Packed components must divide evenly across ranks")
    chunks = weight.chunk(components, dim=0)
    scale_chunks = scale.chunk(components, dim=0)
    return (torch.cat([w.chunk(world_size, dim=0)[rank] for w in chunks], dim=0),
            torch.cat([s.chunk(world_size, dim=0)[rank] for s in scale_chunks], dim=0))


def row_linear(x, weight, weight_scale, comm, world_size, groupsize=256, input_act=None,
               bias=None, residual=None, residual_scale=None, *, division="rn"):
    """Exact full-gather route (parallel_int8.py:72-94) with the B200 quantiser."""
    if groupsize != 256:
        raise ValueError("Only regular ConvRot256 groups are supported")
    full, start, length = gather(x, comm, -1)
    if input_act == "swiglu":
        pieces = full.chunk(world_size, -1)
        full = torch.cat([p.chunk(2, -1)[0] for p in pieces] + [p.chunk(2, -1)[1] for p in pieces], -1)
        start //= 2
        length //= 2
        kind = "gateup_f16" if full.dtype == torch.float16 else None
        if kind is None:
            raise ValueError("[gate|up] input must be fp16")
    elif input_act is None:
        kind = "act_f32" if full.dtype == torch.float32 else "act_f16"
    else:
        raise ValueError("Unknown input activation")
    flat = full.reshape(-1, full.shape[-1]).contiguous()
    q, scale, _ = ops.swiglu_rotate_quantize_local(flat, kind, division)
    del full, flat
    partial = int_mm(q[:, start:start + length].contiguous(), weight)
    del q
    if world_size > 1:
        comm.all_reduce(partial, op=comm.ReduceOp.SUM)
    out = dequantize(partial, scale, weight_scale, x.dtype, bias).reshape(*x.shape[:-1], weight.shape[0])
    if residual is not None:
        out = torch.addcmul(residual, out.to(x.dtype), residual_scale)
    return out.to(x.dtype)
