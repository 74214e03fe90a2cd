"""Column projections (QKV / FC1) on B200 (mirror of patches/dit_column_linear.py).

column_linear: ConvRot256 + per-row INT8 quantisation of the fp16 input, then one
tcgen05 INT8 GEMM whose epilogue applies the ordered column dequant
    y = f16( f32(C) *rn (A_row *rn W_col) [+rn bias] )
(tilelang_column_epilogue.py:11-27) and stores fp16 once.  With swiglu=True the
[gate_r | up_r] accumulators of one output tile are paired in the same CTA and the
epilogue stores the FP32 SwiGLU activation of the FC2 producer instead
(tilelang_swiglu_quant.py:21-24 applied to the fp16-rounded gate/up values).
"""
from __future__ import annotations

import torch

from . import ops

BACKENDS = ("b200", "preallocated", "cuda_int8_tilelang")


def _prepare_activation(x, convrot, convrot_groupsize):
    """Rotation + row quantisation of the column input (dit_column_linear.py:13-21).
    Returns (codes int8 [M, K], row_scale fp32 [M, 1])."""
    if convrot and convrot_groupsize != 256:
        raise ValueError("Only regular ConvRot256 groups are supported")
    if convrot and x.shape[-1] % convrot_groupsize:
        raise ValueError("ConvRot group size must divide input features")
    flat = x.reshape(-1, x.shape[-1])
    if flat.dtype != torch.float16:
        flat = flat.to(torch.float16)
    return ops.column_quantize(flat.contiguous(), convrot)


def _check(x, weight, weight_scale):
    if x.shape[-1] != weight.shape[-1]:
        raise ValueError("Input and weight inner dimensions must match")
    if weight.dtype != torch.int8 or weight.ndim != 2:
        raise ValueError("INT8 [N, K] weight required")
    ws = weight_scale.to(device=x.device, dtype=torch.float32).reshape(-1)
    if ws.numel() not in (1, weight.shape[0]):
        raise ValueError("INT8 weight scale must be scalar or per-output-channel")
    return weight.to(device=x.device).contiguous(), ws.contiguous()


def column_linear(x, weight, weight_scale, *, convrot=True, convrot_groupsize=256,
                  out_dtype=torch.float16, backend="b200", p0_a1=False, bias=None,
                  swiglu=False, swiglu_dtype=torch.float32):
    """ColumnParallel INT8 linear of one rank (dit_column_linear.py:99-125).

    Returns fp16 [..., N] (or, with swiglu=True, the SwiGLU activation
    [..., N/2] in swiglu_dtype).  p0_a1 (a T4 CUTLASS route) is accepted and ignored."""
    if backend not in BACKENDS:
        raise ValueError("Unknown column linear backend")
    if out_dtype != torch.float16:
        raise ValueError("The B200 column path stores fp16 (the DiT activation dtype)")
    weight, ws = _check(x, weight, weight_scale)
    shape = x.shape
    codes, row_scale = _prepare_activation(x, convrot, convrot_groupsize)
    b = None if bias is None else bias.to(device=x.device, dtype=torch.float32).reshape(-1)
    if swiglu:
        if ws.numel() != weight.shape[0]:
            ws = ws.expand(weight.shape[0]).contiguous()
        out = ops.int8_gemm_swiglu(codes, weight, row_scale, ws, b, swiglu_dtype)
        return out.reshape(*shape[:-1], weight.shape[0] // 2)
    out = ops.int8_gemm_column(codes, weight, row_scale, ws, b)
    return out.reshape(*shape[:-1], weight.shape[0])


def column_linear_quantized(codes, row_scale, weight, weight_scale, *, bias=None, swiglu=False,
                            swiglu_dtype=torch.float32):
    """The GEMM + ordered epilogue of column_linear on activation codes that were
    already produced (e.g. by the fused modulated-norm producer)."""
    weight, ws = _check(codes, weight, weight_scale)
    b = None if bias is None else bias.to(device=codes.device, dtype=torch.float32).reshape(-1)
    if swiglu:
        if ws.numel() != weight.shape[0]:
            ws = ws.expand(weight.shape[0]).contiguous()
        return ops.int8_gemm_swiglu(codes, weight, row_scale, ws, b, swiglu_dtype)
    return ops.int8_gemm_column(codes, weight, row_scale, ws, b)


def shared_column_linears(x, projections, *, convrot=True, convrot_groupsize=256):
    """One rotation + quantisation shared by several projections of the same input
    (dit_column_linear.py:70-96); one GEMM per projection."""
    if torch.is_grad_enabled() or type(x) is not torch.Tensor:
        return None
    codes, row_scale = _prepare_activation(x, convrot, convrot_groupsize)
    outputs = []
    for weight, weight_scale in projections:
        weight, ws = _check(x, weight, weight_scale)
        out = ops.int8_gemm_column(codes, weight, row_scale, ws)
        outputs.append(out.reshape(*x.shape[:-1], weight.shape[0]))
    return tuple(outputs)
