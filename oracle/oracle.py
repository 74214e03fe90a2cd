"""ORACLE - TEST INFRASTRUCTURE ONLY.

numpy front end of the CPU restatement in h3_oracle.c of the reference's INT8 linear
path arithmetic (chinokikiss/minimax-h3-2xt4, patches/).  Only tests/, the smoke
check in __graft_entry__.py and bench.py's cpu_baseline / reference arm use it, and
only as the checker or the timed CPU baseline; the product never imports it.

Each function cites the reference lines it restates.  Arrays are numpy; fp16 data is
passed as numpy.float16 (bit-compatible with torch.float16).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import build as _build

_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        F = ctypes.c_float
        L.h3o_half_to_float.argtypes = [ctypes.c_uint16]
        L.h3o_half_to_float.restype = F
        L.h3o_float_to_half.argtypes = [F]
        L.h3o_float_to_half.restype = ctypes.c_uint16
        L.h3o_expf.argtypes = [F]
        L.h3o_expf.restype = F
        L.h3o_swiglu.argtypes = [F, F]
        L.h3o_swiglu.restype = F
        L.h3o_convrot256.argtypes = [P]
        L.h3o_fc2_rotate.argtypes = [P, I, I64, I64, P, P]
        L.h3o_row_quantize.argtypes = [P, I64, I64, I64, I64, P, P, P]
        L.h3o_column_quantize.argtypes = [P, I64, I64, I, P, P]
        L.h3o_int8_gemm.argtypes = [P, P, I64, I64, I64, P]
        L.h3o_column_epilogue.argtypes = [P, I64, I64, P, P, I64, P, P]
        L.h3o_swiglu_epilogue.argtypes = [P, I64, I64, P, P, P, I, P]
        L.h3o_fp16_encode.argtypes = [P, I64, I, P]
        L.h3o_fp16_decode.argtypes = [P, I64, I, P]
        L.h3o_row_reduce_finish.argtypes = [P, I, I64, I64, I64, I, P, P, I, P, P, P, P]
        L.h3o_dequantize_i32.argtypes = [P, I64, I64, P, P, I64, P, I, P, P, P, P]
        L.h3o_gated_add.argtypes = [P, I64, I64, P, P, P]
        L.h3o_transport_shift.argtypes = [I64]
        L.h3o_pack8.argtypes = [P, I64, I64, P]
        L.h3o_modulated_norm.argtypes = [P, I64, I64, P, F, P, P, P, P]
        L.h3o_rsqrt_rn.argtypes = [F]
        L.h3o_rsqrt_rn.restype = F
        L.h3o_unpack8_restore.argtypes = [P, I, I64, I64, I64, P]
        L.h3o_transport_shift.restype = I
        _LIB = L
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------------------
# scalar helpers
# ----------------------------------------------------------------------------
def expf(x: np.ndarray) -> np.ndarray:
    """Exponential of the SwiGLU denominator (the path's documented stand-in for CUDA
    expf at tilelang_swiglu_quant.py:22)."""
    L = lib()
    x = _c(x, np.float32).ravel()
    return np.array([L.h3o_expf(float(v)) for v in x], dtype=np.float32)


def convrot256(v: np.ndarray) -> np.ndarray:
    """Regular ConvRot256 of one group: tilelang_swiglu_quant.py:26-36,46."""
    a = _c(v, np.float32).copy()
    assert a.shape == (256,)
    lib().h3o_convrot256(_p(a))
    return a


def transport_shift(full_k: int) -> int:
    """shift_for (tilelang_transport_tradeoffs.py:20-22) on the full reduction length."""
    return int(lib().h3o_transport_shift(int(full_k)))


# ----------------------------------------------------------------------------
# FC2 producer and quantizers
# ----------------------------------------------------------------------------
KIND = {"gateup_f16": 0, "act_f32": 1, "act_f16": 2}


def fc2_rotate(x: np.ndarray, kind: str = "gateup_f16"):
    """fused_kernel phase 'stored' (tilelang_swiglu_quant.py:37-51) + row maximum
    (:86).  Returns (rotated fp32 [rows, width], row_max fp32 [rows])."""
    k = KIND[kind]
    x = _c(x, np.float16 if k != 1 else np.float32)
    rows = x.shape[0]
    width = x.shape[1] // 2 if k == 0 else x.shape[1]
    R = np.empty((rows, width), np.float32)
    m = np.empty((rows,), np.float32)
    lib().h3o_fc2_rotate(_p(x), k, rows, width, _p(R), _p(m))
    return R, m


def row_quantize(X: np.ndarray, row_max: np.ndarray, start: int = 0, width: int | None = None):
    """Row quantizer, division 'rn' (tilelang_row_quant.py:27-46)."""
    X = _c(X, np.float32)
    rows, stride = X.shape
    width = stride - start if width is None else width
    q = np.empty((rows, width), np.int8)
    s = np.empty((rows,), np.float32)
    lib().h3o_row_quantize(_p(X), rows, width, stride, start, _p(_c(row_max, np.float32)), _p(q), _p(s))
    return q, s


def column_quantize(x: np.ndarray, convrot: bool = True):
    """Column activation preparation (dit_column_linear.py:13-21) as this path defines
    it: rotated = f16(H256 x), then the row quantizer with the row's own maximum."""
    x = _c(x, np.float16)
    rows, k = x.shape
    q = np.empty((rows, k), np.int8)
    s = np.empty((rows,), np.float32)
    lib().h3o_column_quantize(_p(x), rows, k, int(bool(convrot)), _p(q), _p(s))
    return q, s


def int8_gemm_loop(A: np.ndarray, W: np.ndarray) -> np.ndarray:
    """Exact INT32 GEMM, C = A @ W.T, as a plain C loop (the oracle's own statement)."""
    A = _c(A, np.int8)
    W = _c(W, np.int8)
    M, K = A.shape
    N = W.shape[0]
    assert W.shape[1] == K
    C = np.empty((M, N), np.int32)
    lib().h3o_int8_gemm(_p(A), _p(W), M, N, K, _p(C))
    return C


def int8_gemm(A: np.ndarray, W: np.ndarray) -> np.ndarray:
    """Exact INT32 GEMM, C = A @ W.T.  Large products run through torch._int_mm on the
    CPU, which is what the reference's own parallel_int8.int_mm calls there
    (patches/parallel_int8.py:46-50); small ones through the C loop.  The two agree bit
    for bit (tests/test_oracle_golden.py pins both against the reference's int_mm)."""
    A = _c(A, np.int8)
    W = _c(W, np.int8)
    M, K = A.shape
    N = W.shape[0]
    assert W.shape[1] == K
    if M * N * K < (1 << 24):
        return int8_gemm_loop(A, W)
    import torch
    return torch._int_mm(torch.from_numpy(A), torch.from_numpy(W).t()).numpy()


# ----------------------------------------------------------------------------
# epilogues and transport
# ----------------------------------------------------------------------------
def column_epilogue(C, row_scale, weight_scale, bias=None) -> np.ndarray:
    """tilelang_column_epilogue.py:11-27 (+ bias after the product)."""
    C = _c(C, np.int32)
    M, N = C.shape
    w = _c(weight_scale, np.float32).ravel()
    Y = np.empty((M, N), np.float16)
    lib().h3o_column_epilogue(_p(C), M, N, _p(_c(row_scale, np.float32).ravel()), _p(w), w.size,
                              _p(None if bias is None else _c(bias, np.float32).ravel()), _p(Y))
    return Y


def swiglu_epilogue(C, row_scale, weight_scale, bias=None, out="f32") -> np.ndarray:
    """FC1 [gate|up] column epilogue followed by the FC2 producer's FP32 SwiGLU."""
    C = _c(C, np.int32)
    M, N2 = C.shape
    Nh = N2 // 2
    Y = np.empty((M, Nh), np.float32 if out == "f32" else np.float16)
    lib().h3o_swiglu_epilogue(_p(C), M, Nh, _p(_c(row_scale, np.float32).ravel()),
                              _p(_c(weight_scale, np.float32).ravel()),
                              _p(None if bias is None else _c(bias, np.float32).ravel()),
                              0 if out == "f32" else 1, _p(Y))
    return Y


def fp16_encode(P, shift: int) -> np.ndarray:
    P = _c(P, np.int32)
    Y = np.empty(P.shape, np.float16)
    lib().h3o_fp16_encode(_p(P), P.size, int(shift), _p(Y))
    return Y


def fp16_decode(Y, shift: int) -> np.ndarray:
    Y = _c(Y, np.float16)
    P = np.empty(Y.shape, np.int32)
    lib().h3o_fp16_decode(_p(Y), Y.size, int(shift), _p(P))
    return P


def modulated_norm(x, weight, eps, shift, scale, labels=None) -> np.ndarray:
    """Modulated RMSNorm of the fused column producer (tilelang_dit_fusion.py:11-37
    order of operations, correctly rounded rsqrt, the kernel's fixed sum order):
    fp16 [rows, width] -> fp16 h."""
    x = _c(x, np.float16)
    rows, width = x.shape
    h = np.empty_like(x)
    lib().h3o_modulated_norm(_p(x), rows, width, _p(_c(weight, np.float32).ravel()),
                             float(np.float32(eps)), _p(_c(shift, np.float32)),
                             _p(_c(scale, np.float32)),
                             _p(None if labels is None else _c(labels, np.int32)), _p(h))
    return h


def rsqrt_rn(v: float) -> float:
    return float(lib().h3o_rsqrt_rn(float(v)))


def pack8(P) -> np.ndarray:
    """'int8_gather' pack of an INT32 partial (tilelang_transport_tradeoffs.py:40-62):
    uint8 [rows, groups * 132], per group 128 codes then the fp32 scale's bytes."""
    P = _c(P, np.int32)
    rows, width = P.shape
    assert width % 128 == 0
    out = np.empty((rows, width // 128 * 132), np.uint8)
    lib().h3o_pack8(_p(P), rows, width, _p(out))
    return out


def unpack8_restore(parts, width: int) -> np.ndarray:
    """Rank-order reconstruction of packed payloads [world, rows, groups * 132] into the
    restored INT32 sum (tilelang_transport_p2.py:28-42, tp2_tradeoffs.py:73-78)."""
    parts = _c(parts, np.uint8)
    world, rows, pitch = parts.shape
    assert pitch == width // 128 * 132
    out = np.empty((rows, width), np.int32)
    lib().h3o_unpack8_restore(_p(parts), world, rows * pitch, rows, width, _p(out))
    return out


OUT = {"f32": 0, "f16": 1, "residual": 2}


def row_reduce_finish(parts, shift, row_scale, weight_scale, out="f32", residual=None,
                      gate=None, labels=None):
    """Rank-order fp32 sum of fp16 partials, one fp16 rounding, then the fused
    decode + dequant epilogue (tilelang_transport_p2.py:15-47) and optionally the
    gated residual (tilelang_dit_fusion.py:57-77, applied to `residual` in place).
    parts: fp16 [world, rows, width]."""
    parts = _c(parts, np.float16)
    world, rows, width = parts.shape
    o = OUT[out]
    Y = None
    if o == 0:
        Y = np.empty((rows, width), np.float32)
    elif o == 1:
        Y = np.empty((rows, width), np.float16)
    else:
        assert residual is not None and residual.dtype == np.float16 and residual.flags.c_contiguous
    lib().h3o_row_reduce_finish(
        _p(parts), world, rows * width, rows, width, int(shift),
        _p(_c(row_scale, np.float32).ravel()), _p(_c(weight_scale, np.float32).ravel()), o, _p(Y),
        _p(residual) if o == 2 else None,
        _p(None if gate is None else _c(gate, np.float32)),
        _p(None if labels is None else _c(labels, np.int32)))
    return residual if o == 2 else Y


def dequantize_i32(acc, row_scale, weight_scale, bias=None, out="f32", residual=None,
                   gate=None, labels=None):
    """parallel_int8.dequantize CPU branch (parallel_int8.py:66-69)."""
    acc = _c(acc, np.int32)
    rows, width = acc.shape
    o = OUT[out]
    w = _c(weight_scale, np.float32).ravel()
    Y = None
    if o == 0:
        Y = np.empty((rows, width), np.float32)
    elif o == 1:
        Y = np.empty((rows, width), np.float16)
    lib().h3o_dequantize_i32(
        _p(acc), rows, width, _p(_c(row_scale, np.float32).ravel()), _p(w), w.size,
        _p(None if bias is None else _c(bias, np.float32).ravel()), o, _p(Y),
        _p(residual) if o == 2 else None,
        _p(None if gate is None else _c(gate, np.float32)),
        _p(None if labels is None else _c(labels, np.int32)))
    return residual if o == 2 else Y


def gated_add(y, residual, gate=None, labels=None):
    """X = f16(fma(f16(y), G[label], X)) in place on `residual` (fp16, contiguous)."""
    y = _c(y, np.float32)
    rows, width = y.shape
    assert residual.dtype == np.float16 and residual.flags.c_contiguous and residual.shape == y.shape
    lib().h3o_gated_add(_p(y), rows, width, _p(residual),
                        _p(None if gate is None else _c(gate, np.float32)),
                        _p(None if labels is None else _c(labels, np.int32)))
    return residual


# ----------------------------------------------------------------------------
# composite chains (the whole operator, as the reference runs it)
# ----------------------------------------------------------------------------
def packed_rows(weight, scale, rank, world_size, components):
    """parallel_int8.packed_rows (parallel_int8.py:97-103)."""
    if weight.shape[0] % (components * world_size):
        raise ValueError("Packed components must divide evenly across ranks")
    wc = np.split(weight, components, axis=0)
    sc = np.split(scale, components, axis=0)
    return (np.concatenate([np.split(w, world_size, axis=0)[rank] for w in wc], 0),
            np.concatenate([np.split(s, world_size, axis=0)[rank] for s in sc], 0))


def column_linear(x, weight, weight_scale, convrot=True, bias=None):
    """ColumnParallelLinearINT8.forward on one rank (tp_dit.py:69-96): prepare, exact
    INT32 GEMM, ordered epilogue -> fp16 [M, Nl]."""
    q, s = column_quantize(x, convrot)
    C = int8_gemm(q, weight)
    return column_epilogue(C, s, weight_scale, bias), (q, s, C)


def fc2_fused_stored(xs, weights, weight_scale, out="f32", residual=None, gate=None,
                     labels=None, kind="gateup_f16"):
    """RowParallel FC2 `fused_stored` over `world` ranks (tilelang_swiglu_quant.py:
    67-128 with the scaled-FP16 transport).  xs[r]: rank r's input; weights[r]: its
    [N, Kl] shard.  world == 1 takes the exact INT32 route (no transport)."""
    world = len(xs)
    rots, maxes = zip(*[fc2_rotate(x, kind) for x in xs])
    gmax = np.maximum.reduce(list(maxes))                      # all_reduce MAX
    qs = [row_quantize(R, gmax) for R in rots]
    partials = [int8_gemm(q, w) for (q, _), w in zip(qs, weights)]
    scale = qs[0][1]
    if world == 1:
        return dequantize_i32(partials[0], scale, weight_scale, out=out, residual=residual,
                              gate=gate, labels=labels), qs, partials
    local_k = qs[0][0].shape[1]
    shift = transport_shift(local_k * world)
    enc = np.stack([fp16_encode(p, shift) for p in partials])
    y = row_reduce_finish(enc, shift, scale, weight_scale, out=out, residual=residual,
                          gate=gate, labels=labels)
    return y, qs, partials


# ----------------------------------------------------------------------------
# compositions of whole blocks at TP = world (the arithmetic of every rank, combined
# the way the collectives combine it); inputs and outputs are numpy arrays
# ----------------------------------------------------------------------------
def mlp_block(x, h, w1, s1, w2, s2, world, gate=None, labels=None, payload="fp16"):
    """TPDiTMLPINT8.forward at TP = world (tp_dit.py:347-366): FC1 on rank shards
    (packed_rows, components [gate | up]) with the FP32 SwiGLU, FC2 over contiguous K
    blocks with the global row maximum, scaled-fp16 partials summed in rank order (or,
    payload 'int8_gather', the packed INT8 group-128 payloads), gated residual.
    Returns the updated residual (x is not modified)."""
    ref = np.array(x, dtype=np.float16, copy=True)
    s2 = np.asarray(s2, np.float32).ravel()
    q, a = column_quantize(h, True)
    kl = w2.shape[1] // world
    acts, w2s = [], []
    for r in range(world):
        w1r, s1r = packed_rows(w1, s1, r, world, 2)
        acts.append(swiglu_epilogue(int8_gemm(q, w1r), a, np.asarray(s1r).ravel()))
        w2s.append(np.ascontiguousarray(w2[:, r * kl:(r + 1) * kl]))
    if payload == "fp16" or world == 1:
        fc2_fused_stored(acts, w2s, s2, out="residual", residual=ref, gate=gate, labels=labels,
                         kind="act_f32")
        return ref
    rots = [fc2_rotate(v, "act_f32") for v in acts]
    gmax = np.max(np.stack([m for _, m in rots]), 0)
    qs = [row_quantize(R, gmax) for R, _ in rots]
    packed = np.stack([pack8(int8_gemm(qq, w)) for (qq, _), w in zip(qs, w2s)])
    restored = unpack8_restore(packed, w2.shape[0])
    dequantize_i32(restored, qs[0][1], s2, out="residual", residual=ref, gate=gate, labels=labels)
    return ref


def o_projection(x, attn, wo, so, world, gate=None, labels=None):
    """RowParallel O projection with the gated residual at TP = world: attn [M, K] is the
    full attention output (rank r holds columns [r K/t, (r+1) K/t)).  The rows are
    rotated per 256-group and quantised with one global row maximum (whether each rank
    rotates its own whole groups or, when its slice splits a group, the gathered rows,
    the codes are the same); each rank multiplies its columns' codes; TP 1 dequantises
    the exact INT32 sum, TP > 1 sums the scaled-fp16 partials in rank order.  Returns
    the updated residual."""
    ref = np.array(x, dtype=np.float16, copy=True)
    so = np.asarray(so, np.float32).ravel()
    R, m = fc2_rotate(np.ascontiguousarray(attn, np.float16), "act_f16")
    q, a = row_quantize(R, m)
    K = attn.shape[1]
    kl = K // world
    parts = [int8_gemm(np.ascontiguousarray(q[:, r * kl:(r + 1) * kl]),
                       np.ascontiguousarray(wo[:, r * kl:(r + 1) * kl])) for r in range(world)]
    if world == 1:
        dequantize_i32(parts[0], a, so, out="residual", residual=ref, gate=gate, labels=labels)
        return ref
    shift = transport_shift(K)
    enc = np.stack([fp16_encode(p, shift) for p in parts])
    row_reduce_finish(enc, shift, a, so, out="residual", residual=ref, gate=gate, labels=labels)
    return ref


def linear_block(x, wqkv, sqkv, wo, so, w1, s1, w2, s2, world, gate_msa=None, gate_mlp=None,
                 labels=None):
    """TPDiTLinearBlockINT8.forward at TP = world: QKV column projection (components
    q | k | v), the V third as the attention output, O projection + gated residual,
    then the MLP block on the updated residual (its own input, the norm being the
    identity).  Returns the final residual."""
    hidden = x.shape[1]
    inner = hidden // world
    q, a = column_quantize(x, True)
    attn = []
    for r in range(world):
        wr, sr = packed_rows(wqkv, sqkv, r, world, 3)
        qkv = column_epilogue(int8_gemm(q, wr), a, np.asarray(sr).ravel())
        attn.append(qkv[:, 2 * inner:3 * inner])
    x1 = o_projection(x, np.concatenate(attn, 1), wo, so, world, gate_msa, labels)
    return mlp_block(x1, x1, w1, s1, w2, s2, world, gate_mlp, labels)
