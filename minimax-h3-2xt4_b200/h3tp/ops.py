"""torch front end of the C ABI: validates tensors, allocates outputs on the input's
device, and enqueues the sm_100a kernels on the current CUDA stream.

Every function here launches native kernels; none has a CPU path.  Scales follow
the reference's shapes: activation scales [M, 1] fp32, weight scales [N, 1] fp32.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N


def launch_count() -> int:
    """Kernels enqueued so far by this process (one per native call)."""
    return N.launch_count()


def sm_clock_probe(out: torch.Tensor, ns: int, stream: torch.cuda.Stream) -> None:
    """Enqueues the SM clock probe on `stream`: a 32-thread kernel that sleeps `ns`
    nanoseconds and writes [elapsed ns, SM cycles] into `out` (int64 [2], on the GPU),
    so that cycles / ns is the SM clock while other kernels ran beside it."""
    out = _need(out, torch.int64, "out", 1)
    if out.numel() != 2:
        raise ValueError("out must hold 2 int64 values")
    N.call("h3_sm_clock_probe", int(ns), out.data_ptr(), stream.cuda_stream)


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(t: torch.Tensor, dtype, name: str, ndim: int | None = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name}: CUDA tensor required (the INT8 path has no CPU fallback)")
    if t.dtype != dtype:
        raise ValueError(f"{name}: {dtype} required, got {t.dtype}")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name}: {ndim}-D tensor required")
    return t.contiguous()


def _vec(t: torch.Tensor, n: int, name: str) -> torch.Tensor:
    t = _need(t, torch.float32, name)
    if t.numel() != n:
        raise ValueError(f"{name}: {n} values required, got {t.numel()}")
    return t.reshape(-1)


INPUT_KINDS = {"gateup_f16": N.IN_GATEUP_F16, "act_f32": N.IN_ACT_F32, "act_f16": N.IN_ACT_F16}
DIVISIONS = {"rn": N.DIV_RN, "fast": N.DIV_FAST}


def _out(out, shape, dtype, device, name):
    """A caller-provided output buffer (contiguous, exact shape / dtype / device), or a
    fresh one."""
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    if (out.dtype != dtype or tuple(out.shape) != tuple(shape) or not out.is_contiguous()
            or out.device != device):
        raise ValueError(f"{name}: contiguous {dtype} {tuple(shape)} buffer on {device} required")
    return out


def _producer_input(x: torch.Tensor, kind: str):
    k = INPUT_KINDS[kind]
    x = _need(x, torch.float32 if k == N.IN_ACT_F32 else torch.float16, "x", 2)
    width = x.shape[1] // 2 if k == N.IN_GATEUP_F16 else x.shape[1]
    return x, k, x.shape[0], width


# ----------------------------------------------------------------------------
# column path
# ----------------------------------------------------------------------------
def column_quantize(x: torch.Tensor, convrot: bool = True, out_q=None, out_scale=None):
    """Rotation (optional) + per-row INT8 quantisation of the column input.
    Returns (q int8 [M, K], scale fp32 [M, 1])."""
    x = _need(x, torch.float16, "x", 2)
    M, K = x.shape
    q = _out(out_q, (M, K), torch.int8, x.device, "out_q")
    s = _out(out_scale, (M, 1), torch.float32, x.device, "out_scale")
    N.call("h3_column_quantize", x.data_ptr(), M, K, int(bool(convrot)), q.data_ptr(),
           s.data_ptr(), _stream(x))
    return q, s


def modulated_norm_quantize(x, weight, eps: float, shift, scale, labels=None, convrot=True,
                            quantize=True, want_h=False):
    """Modulated RMSNorm (tilelang_dit_fusion.py:11-37) fused with the column
    activation quantiser: x fp16 [M, K] -> (codes int8 [M, K], row_scale fp32 [M, 1],
    h fp16 [M, K] or None).  quantize=False returns (None, None, h)."""
    x = _need(x, torch.float16, "x", 2)
    M, K = x.shape
    w = _vec(weight, K, "norm weight")
    shift = _need(shift, torch.float32, "shift", 2)
    scale = _need(scale, torch.float32, "scale", 2)
    if shift.shape != scale.shape or shift.shape[1] != K:
        raise ValueError("shift / scale tables must be [modulation_rows, K]")
    lab = None
    if labels is not None:
        lab = _need(labels, torch.int32, "labels", 1)
        if lab.numel() != M:
            raise ValueError("one label per row required")
    elif shift.shape[0] != 1:
        raise ValueError("labels required for a multi-row modulation table")
    q = s = h = None
    if quantize:
        q = torch.empty((M, K), dtype=torch.int8, device=x.device)
        s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    if want_h or not quantize:
        h = torch.empty((M, K), dtype=torch.float16, device=x.device)
    N.call("h3_modulated_norm_quantize", x.data_ptr(), M, K, w.data_ptr(), float(eps),
           shift.data_ptr(), scale.data_ptr(), shift.shape[0], _ptr(lab), int(bool(convrot)),
           _ptr(q), _ptr(s), _ptr(h), _stream(x))
    return q, s, h


def int8_gemm_i32(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Exact INT32 q @ w.T on the tensor cores (tcgen05 kind::i8)."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    out = torch.empty((M, w.shape[0]), dtype=torch.int32, device=q.device)
    N.call("h3_int8_gemm_i32", q.data_ptr(), w.data_ptr(), M, w.shape[0], K, out.data_ptr(),
           _stream(q))
    return out


def int8_gemm_column(q, w, row_scale, weight_scale, bias=None) -> torch.Tensor:
    """INT8 GEMM + ordered column epilogue, fp16 [M, N]."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    Nn = w.shape[0]
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    a = _vec(row_scale, M, "row_scale")
    ws = _need(weight_scale, torch.float32, "weight_scale").reshape(-1)
    if ws.numel() not in (1, Nn):
        raise ValueError("INT8 weight scale must be scalar or per-output-channel")
    b = None if bias is None else _vec(bias, Nn, "bias")
    out = torch.empty((M, Nn), dtype=torch.float16, device=q.device)
    N.call("h3_int8_gemm_column", q.data_ptr(), w.data_ptr(), M, Nn, K, a.data_ptr(),
           ws.data_ptr(), ws.numel(), _ptr(b), out.data_ptr(), _stream(q))
    return out


def int8_gemm_swiglu(q, w, row_scale, weight_scale, bias=None, out_dtype=torch.float32, out=None):
    """FC1 GEMM with the FP32 SwiGLU epilogue; w is [gate_r | up_r]; output
    [M, w.shape[0] // 2] in out_dtype (fp32 keeps the reference's bits)."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    Np = w.shape[0]
    if w.shape[1] != K or Np % 2:
        raise ValueError("SwiGLU weight must be [2*n, K] with matching K")
    a = _vec(row_scale, M, "row_scale")
    ws = _vec(weight_scale, Np, "weight_scale")
    b = None if bias is None else _vec(bias, Np, "bias")
    kind = {torch.float32: N.OUT_F32, torch.float16: N.OUT_F16}[out_dtype]
    out = _out(out, (M, Np // 2), out_dtype, q.device, "out")
    N.call("h3_int8_gemm_swiglu", q.data_ptr(), w.data_ptr(), M, Np, K, a.data_ptr(),
           ws.data_ptr(), _ptr(b), kind, out.data_ptr(), _stream(q))
    return out


def column_dequantize(acc, row_scale, weight_scale) -> torch.Tensor:
    """tilelang_column_epilogue.dequantize: f16(C * (A * W))."""
    acc = _need(acc, torch.int32, "accumulator", 2)
    M, Nn = acc.shape
    a = _vec(row_scale, M, "row_scale")
    ws = _need(weight_scale, torch.float32, "weight_scale").reshape(-1)
    if ws.numel() not in (1, Nn):
        raise ValueError("Scalar or channel scale required")
    out = torch.empty((M, Nn), dtype=torch.float16, device=acc.device)
    N.call("h3_column_dequantize", acc.data_ptr(), M, Nn, a.data_ptr(), ws.data_ptr(),
           ws.numel(), out.data_ptr(), _stream(acc))
    return out


# ----------------------------------------------------------------------------
# FC2 producer
# ----------------------------------------------------------------------------
def swiglu_rotate_max(x, kind="gateup_f16", store=True):
    """Phase 'stored' (store=True) or 'maximum'.  Returns (rotated fp32 or None,
    row_max fp32 [M, 1])."""
    x, k, M, W = _producer_input(x, kind)
    rot = torch.empty((M, W), dtype=torch.float32, device=x.device) if store else None
    m = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    N.call("h3_swiglu_rotate_max", x.data_ptr(), k, M, W, _ptr(rot), m.data_ptr(), _stream(x))
    return rot, m


def swiglu_rotate_quantize(x, row_max, kind="gateup_f16", division="rn"):
    """Phase 'recompute': codes of the rotated activation under the reduced row max."""
    x, k, M, W = _producer_input(x, kind)
    m = _vec(row_max, M, "row_max")
    q = torch.empty((M, W), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    N.call("h3_swiglu_rotate_quantize", x.data_ptr(), k, M, W, m.data_ptr(),
           DIVISIONS[division], q.data_ptr(), s.data_ptr(), _stream(x))
    return q, s


def swiglu_rotate_quantize_local(x, kind="gateup_f16", division="rn"):
    """TP=1 single pass.  Returns (q, scale [M, 1], row_max [M, 1])."""
    x, k, M, W = _producer_input(x, kind)
    q = torch.empty((M, W), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    m = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    N.call("h3_swiglu_rotate_quantize_local", x.data_ptr(), k, M, W, DIVISIONS[division],
           q.data_ptr(), s.data_ptr(), m.data_ptr(), _stream(x))
    return q, s, m


PEER_PRODUCER_MAX_WIDTH = 16384  # H3_PEER_PRODUCER_MAX_WIDTH


def swiglu_rotate_quantize_peer(x, bases, world: int, rank: int, slots_off: int, epoch: int,
                                kind="gateup_f16", division="rn", want_max=False, out_q=None,
                                out_scale=None):
    """TP>1 single pass (h3_swiglu_rotate_quantize_peer): the row maxima are exchanged
    with the other ranks over peer memory inside the kernel.  Returns (q, scale [M, 1],
    row_max [M, 1] of the global maxima or None)."""
    x, k, M, W = _producer_input(x, kind)
    q = _out(out_q, (M, W), torch.int8, x.device, "out_q")
    s = _out(out_scale, (M, 1), torch.float32, x.device, "out_scale")
    m = torch.empty((M, 1), dtype=torch.float32, device=x.device) if want_max else None
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_swiglu_rotate_quantize_peer", x.data_ptr(), k, M, W, arr, world, rank,
           int(slots_off), int(epoch), DIVISIONS[division], q.data_ptr(), s.data_ptr(), _ptr(m),
           _stream(x))
    return q, s, m


def row_quantize(rotated, row_max, width=None, start=0, division="rn"):
    """tilelang_row_quant.quantize: codes of rotated[:, start:start+width]."""
    rotated = _need(rotated, torch.float32, "rotated", 2)
    M, stride = rotated.shape
    width = stride - start if width is None else int(width)
    m = _vec(row_max, M, "row_max")
    q = torch.empty((M, width), dtype=torch.int8, device=rotated.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=rotated.device)
    N.call("h3_row_quantize", rotated.data_ptr(), M, width, stride, int(start), m.data_ptr(),
           DIVISIONS[division], q.data_ptr(), s.data_ptr(), _stream(rotated))
    return q, s


# ----------------------------------------------------------------------------
# row path
# ----------------------------------------------------------------------------
def transport_shift(full_k: int) -> int:
    return int(N.load().h3_transport_shift(int(full_k)))


def int8_gemm_row_encode(q, w, shift: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """INT8 GEMM + scaled-FP16 encode: f16(acc * 2^-shift), [M, N].  `out` (contiguous
    fp16 [M, N], e.g. a peer-mapped transport buffer) receives the payload if given."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    if out is None:
        out = torch.empty((M, w.shape[0]), dtype=torch.float16, device=q.device)
    elif (out.dtype != torch.float16 or tuple(out.shape) != (M, w.shape[0])
          or not out.is_contiguous() or out.device != q.device):
        raise ValueError("out must be a contiguous fp16 [M, N] tensor on the input's device")
    N.call("h3_int8_gemm_row_encode", q.data_ptr(), w.data_ptr(), M, w.shape[0], K, int(shift),
           out.data_ptr(), _stream(q))
    return out


def int8_gemm_row_encode_push(q, w, shift: int, bases, world: int, rank: int,
                              partial_off: int) -> None:
    """INT8 GEMM + scaled-FP16 encode with every output row stored into the peer-mapped
    buffer of the rank that owns it (h3_int8_gemm_row_encode_push): the reduce-scatter
    of the partials fused into the GEMM epilogue."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_int8_gemm_row_encode_push", q.data_ptr(), w.data_ptr(), M, w.shape[0], K,
           int(shift), arr, world, rank, int(partial_off), _stream(q))


def _gate_args(residual, gate, labels, M, Nn):
    if residual is None:
        return None, None, 0, None
    residual = _need(residual, torch.float16, "residual", 2)
    if residual.shape != (M, Nn):
        raise ValueError("residual shape mismatch")
    if gate is None:
        return residual, None, 0, None
    gate = _need(gate, torch.float32, "gate", 2)
    if gate.shape[1] != Nn:
        raise ValueError("gate table width mismatch")
    lab = None
    if labels is not None:
        lab = _need(labels, torch.int32, "labels", 1)
        if lab.numel() != M:
            raise ValueError("one label per row required")
    elif gate.shape[0] != 1:
        raise ValueError("labels required for a multi-row gate table")
    return residual, gate, gate.shape[0], lab


def int8_gemm_row_dequant(q, w, row_scale, weight_scale, out_dtype=torch.float32,
                          residual=None, gate=None, labels=None):
    """TP=1 row GEMM, exact INT32 + fused dequant.  With `residual` the gated residual
    is updated in place and returned; otherwise a new [M, N] tensor in out_dtype."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    Nn = w.shape[0]
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    a = _vec(row_scale, M, "row_scale")
    ws = _vec(weight_scale, Nn, "weight_scale")
    if residual is not None:
        if not residual.is_contiguous():
            raise ValueError("residual must be contiguous (updated in place)")
        res, g, grows, lab = _gate_args(residual, gate, labels, M, Nn)
        N.call("h3_int8_gemm_row_dequant", q.data_ptr(), w.data_ptr(), M, Nn, K, a.data_ptr(),
               ws.data_ptr(), N.OUT_RESIDUAL, None, res.data_ptr(), _ptr(g), grows, _ptr(lab),
               _stream(q))
        return residual
    kind = {torch.float32: N.OUT_F32, torch.float16: N.OUT_F16}[out_dtype]
    out = torch.empty((M, Nn), dtype=out_dtype, device=q.device)
    N.call("h3_int8_gemm_row_dequant", q.data_ptr(), w.data_ptr(), M, Nn, K, a.data_ptr(),
           ws.data_ptr(), kind, out.data_ptr(), None, None, 0, None, _stream(q))
    return out


def fp16_encode(partial: torch.Tensor, shift: int) -> torch.Tensor:
    p = _need(partial, torch.int32, "partial")
    out = torch.empty(p.shape, dtype=torch.float16, device=p.device)
    N.call("h3_fp16_encode", p.data_ptr(), p.numel(), int(shift), out.data_ptr(), _stream(p))
    return out


def fp16_decode(payload: torch.Tensor, shift: int) -> torch.Tensor:
    y = _need(payload, torch.float16, "payload")
    out = torch.empty(y.shape, dtype=torch.int32, device=y.device)
    N.call("h3_fp16_decode", y.data_ptr(), y.numel(), int(shift), out.data_ptr(), _stream(y))
    return out


def row_reduce_finish(parts, shift, row_scale, weight_scale, out_dtype=torch.float32,
                      residual=None, gate=None, labels=None):
    """parts: fp16 [world, rows, N] (or [rows, N] for an already reduced payload).
    Fixed-order fp32 sum + one fp16 rounding, decode, dequant, then store or gated
    residual update (residual updated in place and returned)."""
    parts = _need(parts, torch.float16, "parts")
    if parts.ndim == 2:
        parts = parts.unsqueeze(0)
    world, M, Nn = parts.shape
    a = _vec(row_scale, M, "row_scale")
    ws = _vec(weight_scale, Nn, "weight_scale")
    if residual is not None:
        if not residual.is_contiguous():
            raise ValueError("residual must be contiguous (updated in place)")
        res, g, grows, lab = _gate_args(residual, gate, labels, M, Nn)
        N.call("h3_row_reduce_finish", parts.data_ptr(), world, M * Nn, M, Nn, int(shift),
               a.data_ptr(), ws.data_ptr(), N.OUT_RESIDUAL, None, res.data_ptr(), _ptr(g),
               grows, _ptr(lab), _stream(parts))
        return residual
    kind = {torch.float32: N.OUT_F32, torch.float16: N.OUT_F16}[out_dtype]
    out = torch.empty((M, Nn), dtype=out_dtype, device=parts.device)
    N.call("h3_row_reduce_finish", parts.data_ptr(), world, M * Nn, M, Nn, int(shift),
           a.data_ptr(), ws.data_ptr(), kind, out.data_ptr(), None, None, 0, None,
           _stream(parts))
    return out


# ----------------------------------------------------------------------------
# packed INT8 transport ('int8_gather')
# ----------------------------------------------------------------------------
def pack8_pitch(width: int) -> int:
    """Bytes per row of a packed payload: 128 codes + 4 scale bytes per 128 columns."""
    if width % 128:
        raise ValueError("Whole group128 outputs required")
    return width // 128 * 132


def int8_gemm_row_pack8(q, w, out: torch.Tensor | None = None) -> torch.Tensor:
    """INT8 GEMM with the group-128 INT8 pack fused: uint8 [M, N/128*132]."""
    q = _need(q, torch.int8, "q", 2)
    w = _need(w, torch.int8, "weight", 2)
    M, K = q.shape
    if w.shape[1] != K:
        raise ValueError("Input and weight inner dimensions must match")
    pitch = pack8_pitch(w.shape[0])
    if out is None:
        out = torch.empty((M, pitch), dtype=torch.uint8, device=q.device)
    elif (out.dtype != torch.uint8 or tuple(out.shape) != (M, pitch) or not out.is_contiguous()
          or out.device != q.device):
        raise ValueError("out must be a contiguous uint8 [M, N/128*132] tensor on q's device")
    N.call("h3_int8_gemm_row_pack8", q.data_ptr(), w.data_ptr(), M, w.shape[0], K,
           out.data_ptr(), _stream(q))
    return out


def pack8(partial) -> torch.Tensor:
    """Group-128 INT8 pack of an INT32 partial (pack_int8): uint8 [rows, width/128*132]."""
    p = _need(partial, torch.int32, "partial", 2)
    rows, width = p.shape
    out = torch.empty((rows, pack8_pitch(width)), dtype=torch.uint8, device=p.device)
    N.call("h3_pack8", p.data_ptr(), rows, width, out.data_ptr(), _stream(p))
    return out


def unpack8_finish(parts, width: int, row_scale=None, weight_scale=None, out_dtype=torch.float32,
                   residual=None, gate=None, labels=None):
    """parts: uint8 [world, rows, pitch] (or [rows, pitch]).  Rank-order reconstruction,
    then the row epilogue; out_dtype torch.int32 returns the restored sums."""
    parts = _need(parts, torch.uint8, "parts")
    if parts.ndim == 2:
        parts = parts.unsqueeze(0)
    world, M, pitch = parts.shape
    if pitch != pack8_pitch(width):
        raise ValueError("payload pitch does not match the width")
    if out_dtype == torch.int32 and residual is None:
        out = torch.empty((M, width), dtype=torch.int32, device=parts.device)
        N.call("h3_unpack8_finish", parts.data_ptr(), world, M * pitch, M, width, None, None,
               N.OUT_I32, out.data_ptr(), None, None, 0, None, _stream(parts))
        return out
    a = _vec(row_scale, M, "row_scale")
    ws = _vec(weight_scale, width, "weight_scale")
    if residual is not None:
        if not residual.is_contiguous():
            raise ValueError("residual must be contiguous (updated in place)")
        res, g, grows, lab = _gate_args(residual, gate, labels, M, width)
        N.call("h3_unpack8_finish", parts.data_ptr(), world, M * pitch, M, width, a.data_ptr(),
               ws.data_ptr(), N.OUT_RESIDUAL, None, res.data_ptr(), _ptr(g), grows, _ptr(lab),
               _stream(parts))
        return residual
    kind = {torch.float32: N.OUT_F32, torch.float16: N.OUT_F16}[out_dtype]
    out = torch.empty((M, width), dtype=out_dtype, device=parts.device)
    N.call("h3_unpack8_finish", parts.data_ptr(), world, M * pitch, M, width, a.data_ptr(),
           ws.data_ptr(), kind, out.data_ptr(), None, None, 0, None, _stream(parts))
    return out


def dequantize_i32(acc, row_scale, weight_scale, out_dtype=torch.float32, bias=None):
    """parallel_int8.dequantize order: ((acc * a) * w) + bias."""
    acc = _need(acc, torch.int32, "accumulator", 2)
    M, Nn = acc.shape
    a = _vec(row_scale, M, "activation_scale")
    ws = _need(weight_scale, torch.float32, "weight_scale").reshape(-1)
    if ws.numel() not in (1, Nn):
        raise ValueError("INT8 weight scale must be scalar or per-output-channel")
    b = None if bias is None else _vec(bias, Nn, "bias")
    kind = {torch.float32: N.OUT_F32, torch.float16: N.OUT_F16}[out_dtype]
    out = torch.empty((M, Nn), dtype=out_dtype, device=acc.device)
    N.call("h3_dequantize_i32", acc.data_ptr(), M, Nn, a.data_ptr(), ws.data_ptr(), ws.numel(),
           _ptr(b), kind, out.data_ptr(), _stream(acc))
    return out


def gated_add(residual, branch, gate=None, labels=None):
    """X = f16(fma(f16(branch), G[label], X)) in place (gate_kernel,
    tilelang_dit_fusion.py:39-53); branch fp32 or fp16 [M, N]; returns residual."""
    if not residual.is_contiguous():
        raise ValueError("residual must be contiguous (updated in place)")
    if branch.dtype not in (torch.float32, torch.float16):
        raise ValueError("branch must be fp32 or fp16")
    b = _need(branch, branch.dtype, "branch", 2)
    M, Nn = b.shape
    res, g, grows, lab = _gate_args(residual, gate, labels, M, Nn)
    kind = N.OUT_F32 if b.dtype == torch.float32 else N.OUT_F16
    N.call("h3_gated_add", b.data_ptr(), kind, M, Nn, res.data_ptr(), _ptr(g), grows, _ptr(lab),
           _stream(b))
    return residual


def peer_reduce(bases, world: int, rank: int, flags_off: int, partial_off: int, final_off: int,
                rows: int, width: int, shift: int, row_scale, weight_scale, residual,
                gate=None, labels=None, epoch: int = 1, multicast: int = 0, pushed: bool = False):
    """Reduce + fused gated-residual epilogue of this rank's row block from every rank's
    partial, finished rows stored into the peers' final areas (h3_peer_reduce).  With a
    non-zero `multicast` address of the same buffers the sum is taken in the NVSwitch
    and the finished rows are broadcast through it (h3_peer_reduce_nvls).  pushed: the
    partials were owner-routed by int8_gemm_row_encode_push (h3_peer_reduce_pushed)."""
    a = _vec(row_scale, rows, "row_scale")
    ws = _vec(weight_scale, width, "weight_scale")
    if not residual.is_contiguous():
        raise ValueError("residual must be contiguous (updated in place)")
    res, g, grows, lab = _gate_args(residual, gate, labels, rows, width)
    arr = (ctypes.c_void_p * world)(*bases)
    if multicast:
        N.call("h3_peer_reduce_nvls", arr, int(multicast), world, rank, flags_off, partial_off,
               final_off, rows, width, int(shift), a.data_ptr(), ws.data_ptr(), res.data_ptr(),
               _ptr(g), grows, _ptr(lab), int(epoch), _stream(res))
        return residual
    N.call("h3_peer_reduce_pushed" if pushed else "h3_peer_reduce", arr, world, rank, flags_off,
           partial_off, final_off, rows, width, int(shift), a.data_ptr(), ws.data_ptr(),
           res.data_ptr(), _ptr(g), grows, _ptr(lab), int(epoch), _stream(res))
    return residual


def peer_signal(bases, world: int, rank: int, flags_off: int, which: int, epoch: int,
                publish: bool, like: torch.Tensor) -> None:
    """h3_peer_signal on the stream of `like`'s device: optionally publish flag `which`
    (0 ready, 1 done) of this rank to every rank, then wait (bounded) for every peer's."""
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_peer_signal", arr, world, rank, int(flags_off), int(which), int(epoch),
           1 if publish else 0, _stream(like))


def peer_reduce_staged(bases, world: int, rank: int, flags_off: int, stage_off: int,
                       own_off: int, final_off: int, rows: int, width: int, shift: int,
                       row_scale, weight_scale, residual, gate=None, labels=None,
                       epoch: int = 1):
    """The reduce of the copy-engine exchange (h3_peer_reduce_staged): the peers' rows of
    this rank's block from the staging slots, its own rows at own_off, the finished rows
    into this rank's own final area."""
    a = _vec(row_scale, rows, "row_scale")
    ws = _vec(weight_scale, width, "weight_scale")
    if not residual.is_contiguous():
        raise ValueError("residual must be contiguous (updated in place)")
    res, g, grows, lab = _gate_args(residual, gate, labels, rows, width)
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_peer_reduce_staged", arr, world, rank, int(flags_off), int(stage_off),
           int(own_off), int(final_off), rows, width, int(shift), a.data_ptr(), ws.data_ptr(),
           res.data_ptr(), _ptr(g), grows, _ptr(lab), int(epoch), _stream(res))
    return residual


def copy_async(dst: int, src: int, nbytes: int, like: torch.Tensor) -> None:
    """cudaMemcpyAsync of nbytes between device addresses (either may be a peer's mapped
    buffer) on the stream of `like`'s device."""
    N.call("h3_copy_async", int(dst), int(src), int(nbytes), _stream(like))


def peer_reduce_int8(bases, world: int, rank: int, flags_off: int, partial_off: int,
                     final_off: int, rows: int, width: int, row_scale, weight_scale, residual,
                     gate=None, labels=None, epoch: int = 1):
    """peer_reduce for packed INT8 payloads (h3_peer_reduce_int8)."""
    a = _vec(row_scale, rows, "row_scale")
    ws = _vec(weight_scale, width, "weight_scale")
    if not residual.is_contiguous():
        raise ValueError("residual must be contiguous (updated in place)")
    res, g, grows, lab = _gate_args(residual, gate, labels, rows, width)
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_peer_reduce_int8", arr, world, rank, flags_off, partial_off, final_off, rows, width,
           a.data_ptr(), ws.data_ptr(), res.data_ptr(), _ptr(g), grows, _ptr(lab), int(epoch),
           _stream(res))
    return residual


def peer_gather(bases, world: int, rank: int, flags_off: int, final_off: int, rows: int,
                width: int, residual, epoch: int = 1):
    """Copies the peers' finished row blocks into `residual` (h3_peer_gather)."""
    res = _need(residual, torch.float16, "residual", 2)
    if res.data_ptr() != residual.data_ptr() or tuple(res.shape) != (rows, width):
        raise ValueError("residual must be a contiguous fp16 [rows, width] tensor")
    arr = (ctypes.c_void_p * world)(*bases)
    N.call("h3_peer_gather", arr, world, rank, flags_off, final_off, rows, width, res.data_ptr(),
           int(epoch), _stream(res))
    return residual


def expf_compare(x: torch.Tensor):
    """(h3_expf(x), CUDA expf(x)) evaluated on the device."""
    x = _need(x, torch.float32, "x")
    ours = torch.empty_like(x)
    ref = torch.empty_like(x)
    N.call("h3_expf_compare", x.data_ptr(), x.numel(), ours.data_ptr(), ref.data_ptr(), _stream(x))
    return ours, ref


def silu_compare(g: torch.Tensor):
    """(fast, ieee, cuda_expf) evaluations of g / (1 + exp(-g)) on the device."""
    g = _need(g, torch.float32, "g")
    fast = torch.empty_like(g)
    ieee = torch.empty_like(g)
    cuda = torch.empty_like(g)
    N.call("h3_silu_compare", g.data_ptr(), g.numel(), fast.data_ptr(), ieee.data_ptr(),
           cuda.data_ptr(), _stream(g))
    return fast, ieee, cuda


def quant_compare(x: torch.Tensor, scale: torch.Tensor):
    """(kernel codes, IEEE-division codes) of x / scale, elementwise."""
    x = _need(x, torch.float32, "x")
    scale = _need(scale, torch.float32, "scale")
    if scale.numel() != x.numel():
        raise ValueError("one scale per value")
    fast = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    ieee = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    N.call("h3_quant_compare", x.data_ptr(), scale.data_ptr(), x.numel(), fast.data_ptr(),
           ieee.data_ptr(), _stream(x))
    return fast, ieee
