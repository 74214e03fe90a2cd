"""Row quantizer and the O-projection global row quantisation (mirror of
patches/tilelang_row_quant.py) on B200.

quantize(): codes of rotated[:, start:start+width] under an external row maximum:
    scale = max(min(max, FLT_MAX) * f32(1/127), 1e-30)
    q = clamp(rint(x / scale), -128, 127)
division 'rn' (IEEE, the default, bit-exact with the CPU oracle) or 'fast' (the
reference's production __fdividef).

global_row_quantize(): the O-projection's local ConvRot of whole owned 256-groups,
MAX all-reduce of the row maxima, then quantisation (tilelang_row_quant.py:89-146,
the P0-C local-rotation variant, which is the only form that needs no padded
full-width GEMM once the rotation is a butterfly rather than a GEMM).  When a rank's
slice does not hold whole groups (the O projection at TP 8: 3072 / 8 = 384 columns),
the rows are gathered first, as the reference's exact full-gather route does
(parallel_int8.py:72-94): every rank rotates and quantises the complete row (one global
row maximum, no exchange of maxima) and keeps its own columns' codes - the same codes
the local route gives wherever both apply.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch

from . import comm as C
from . import ops


@contextmanager
def label(name: str):
    """NVTX range 'row_fusion/<name>' (tilelang_row_quant.py:14-18)."""
    torch.cuda.nvtx.range_push("row_fusion/" + name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def quantize(rotated: torch.Tensor, maximum: torch.Tensor, width: int | None = None,
             start: int = 0, division: str = "rn"):
    if rotated.ndim != 2 or rotated.dtype != torch.float32 or not rotated.is_contiguous():
        raise ValueError("Contiguous FP32 storage and matching global row maxima required")
    if maximum.numel() != rotated.shape[0] or maximum.dtype != torch.float32:
        raise ValueError("Contiguous FP32 storage and matching global row maxima required")
    return ops.row_quantize(rotated, maximum, width, start, division)


def global_row_quantize(x: torch.Tensor, comm, world_size: int | None = None, groupsize: int = 256,
                        input_act=None, *, division: str = "rn", consume_input: bool = False):
    """Local rotation of the owned groups + global row max + quantisation.
    x: fp16 or fp32 [..., Kl] (this rank's slice).  Returns (q int8 [M, Kl], scale [M, 1])."""
    if input_act is not None:
        raise ValueError("O-projection rows take no input activation")
    if groupsize != 256:
        raise ValueError("Whole regular ConvRot256 groups required")
    flat = x.reshape(-1, x.shape[-1])
    kind = "act_f32" if flat.dtype == torch.float32 else "act_f16"
    flat = flat.contiguous()
    world = C.world_of(comm) if world_size is None else world_size
    if flat.shape[-1] % groupsize:
        if world == 1 or (flat.shape[-1] * world) % groupsize:
            raise ValueError("ConvRot groups must remain wholly owned by a rank")
        return _gathered_row_quantize(flat, comm, world, kind, division)
    if world == 1:
        q, s, _ = ops.swiglu_rotate_quantize_local(flat, kind, division)
        if consume_input:
            x.set_()
        return q, s
    with label("local_maximum"):
        _, maximum = ops.swiglu_rotate_max(flat, kind, store=False)
    C.all_reduce_max(maximum, comm)
    with label("external_max_quantization"):
        q, s = ops.swiglu_rotate_quantize(flat, maximum, kind, division)
    if consume_input:
        x.set_()
    return q, s


def _gathered_row_quantize(flat: torch.Tensor, comm, world: int, kind: str, division: str):
    """Rows gathered over the group (rank order along the features), rotated and
    quantised whole on every rank; returns this rank's columns of the codes and the
    row scales."""
    width = flat.shape[-1]
    with label("gather_rows"):
        parts = [torch.empty_like(flat) for _ in range(world)]
        comm.all_gather(parts, flat)
        full = torch.cat(parts, dim=-1)
        del parts
    with label("full_row_quantization"):
        q, s, _ = ops.swiglu_rotate_quantize_local(full, kind, division)
    r = C.rank_of(comm)
    return q[:, r * width:(r + 1) * width].contiguous(), s
