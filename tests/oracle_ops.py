"""Test infrastructure: a CPU stand-in for h3tp.ops built on the oracle.

Host-side orchestration (sharding, collectives, row-block exchange, dispatch) is
tested on CPU ranks (gloo) by swapping h3tp.ops' kernel wrappers for these functions,
which compute the same values with the oracle's restatement of the reference
arithmetic.  The product never imports this module; install() is called only from
tests.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

_F = {torch.float32: "f32", torch.float16: "f16"}


def _n(t):
    return t.detach().cpu().contiguous().numpy()


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def transport_shift(full_k):
    return O.transport_shift(int(full_k))


def column_quantize(x, convrot=True):
    q, s = O.column_quantize(_n(x), convrot)
    return _t(q), _t(s).reshape(-1, 1)


def int8_gemm_i32(q, w):
    return _t(O.int8_gemm(_n(q), _n(w)))


def int8_gemm_column(q, w, row_scale, weight_scale, bias=None):
    C = O.int8_gemm(_n(q), _n(w))
    return _t(O.column_epilogue(C, _n(row_scale), _n(weight_scale), None if bias is None else _n(bias)))


def int8_gemm_swiglu(q, w, row_scale, weight_scale, bias=None, out_dtype=torch.float32):
    C = O.int8_gemm(_n(q), _n(w))
    return _t(O.swiglu_epilogue(C, _n(row_scale), _n(weight_scale),
                                None if bias is None else _n(bias), _F[out_dtype]))


_KIND = {"gateup_f16": "gateup_f16", "act_f32": "act_f32", "act_f16": "act_f16"}


def swiglu_rotate_max(x, kind="gateup_f16", store=True):
    R, m = O.fc2_rotate(_n(x), _KIND[kind])
    return (_t(R) if store else None), _t(m).reshape(-1, 1)


def swiglu_rotate_quantize(x, row_max, kind="gateup_f16", division="rn"):
    assert division == "rn"
    R, _ = O.fc2_rotate(_n(x), _KIND[kind])
    q, s = O.row_quantize(R, _n(row_max).ravel())
    return _t(q), _t(s).reshape(-1, 1)


def swiglu_rotate_quantize_local(x, kind="gateup_f16", division="rn"):
    assert division == "rn"
    R, m = O.fc2_rotate(_n(x), _KIND[kind])
    q, s = O.row_quantize(R, m)
    return _t(q), _t(s).reshape(-1, 1), _t(m).reshape(-1, 1)


def row_quantize(rotated, row_max, width=None, start=0, division="rn"):
    q, s = O.row_quantize(_n(rotated), _n(row_max).ravel(), start, width)
    return _t(q), _t(s).reshape(-1, 1)


def int8_gemm_row_encode(q, w, shift):
    return _t(O.fp16_encode(O.int8_gemm(_n(q), _n(w)), shift))


def _residual_out(residual, res_np):
    residual.copy_(_t(res_np))
    return residual


def int8_gemm_row_dequant(q, w, row_scale, weight_scale, out_dtype=torch.float32,
                          residual=None, gate=None, labels=None):
    C = O.int8_gemm(_n(q), _n(w))
    if residual is not None:
        res = _n(residual).copy()
        O.dequantize_i32(C, _n(row_scale), _n(weight_scale), out="residual", residual=res,
                         gate=None if gate is None else _n(gate),
                         labels=None if labels is None else _n(labels))
        return _residual_out(residual, res)
    return _t(O.dequantize_i32(C, _n(row_scale), _n(weight_scale), out=_F[out_dtype]))


def fp16_encode(partial, shift):
    return _t(O.fp16_encode(_n(partial), shift))


def fp16_decode(payload, shift):
    return _t(O.fp16_decode(_n(payload), shift))


def row_reduce_finish(parts, shift, row_scale, weight_scale, out_dtype=torch.float32,
                      residual=None, gate=None, labels=None):
    p = _n(parts)
    if p.ndim == 2:
        p = p[None]
    if residual is not None:
        res = _n(residual).copy()
        O.row_reduce_finish(p, shift, _n(row_scale), _n(weight_scale), out="residual",
                            residual=res, gate=None if gate is None else _n(gate),
                            labels=None if labels is None else _n(labels))
        return _residual_out(residual, res)
    return _t(O.row_reduce_finish(p, shift, _n(row_scale), _n(weight_scale), out=_F[out_dtype]))


def dequantize_i32(acc, row_scale, weight_scale, out_dtype=torch.float32, bias=None):
    return _t(O.dequantize_i32(_n(acc), _n(row_scale), _n(weight_scale),
                               bias=None if bias is None else _n(bias), out=_F[out_dtype]))


def int8_gemm_row_pack8(q, w, out=None):
    r = _t(O.pack8(O.int8_gemm(_n(q), _n(w))))
    if out is not None:
        out.copy_(r)
        return out
    return r


def pack8(partial):
    return _t(O.pack8(_n(partial)))


def unpack8_finish(parts, width, row_scale=None, weight_scale=None, out_dtype=torch.float32,
                   residual=None, gate=None, labels=None):
    p = _n(parts)
    if p.ndim == 2:
        p = p[None]
    restored = O.unpack8_restore(p, width)
    if out_dtype == torch.int32 and residual is None:
        return _t(restored)
    if residual is not None:
        res = _n(residual).copy()
        O.dequantize_i32(restored, _n(row_scale), _n(weight_scale), out="residual", residual=res,
                         gate=None if gate is None else _n(gate),
                         labels=None if labels is None else _n(labels))
        return _residual_out(residual, res)
    return _t(O.dequantize_i32(restored, _n(row_scale), _n(weight_scale), out=_F[out_dtype]))


def gated_add(residual, branch, gate=None, labels=None):
    res = _n(residual).copy()
    O.gated_add(_n(branch).astype(np.float32), res, None if gate is None else _n(gate),
                None if labels is None else _n(labels))
    return _residual_out(residual, res)


NAMES = ["transport_shift", "column_quantize", "int8_gemm_i32", "int8_gemm_column",
         "int8_gemm_swiglu", "swiglu_rotate_max", "swiglu_rotate_quantize",
         "swiglu_rotate_quantize_local", "row_quantize", "int8_gemm_row_encode",
         "int8_gemm_row_dequant", "fp16_encode", "fp16_decode", "row_reduce_finish",
         "dequantize_i32", "gated_add", "int8_gemm_row_pack8", "pack8", "unpack8_finish"]


def install():
    """Replaces h3tp.ops' kernel wrappers by the oracle versions (tests only)."""
    from h3tp import ops
    g = globals()
    for name in NAMES:
        setattr(ops, name, g[name])
