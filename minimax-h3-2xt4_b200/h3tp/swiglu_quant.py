"""FC2 `fused_stored` row chain on B200 (mirror of patches/tilelang_swiglu_quant.py).

    FP32 SwiGLU -> regular ConvRot256 -> global per-row INT8 quant -> INT8 GEMM
    -> scaled-FP16 partial SUM -> fused FP32 dequant (+ gated residual)

Inputs accepted by prepare()/row_linear() (input_act='swiglu'):
  - fp16 [M, 2*Kl] = [gate_r | up_r], the FC1 column output (tp_dit.py:356);
  - fp32 [M, Kl]   = silu(f16 gate) * f16 up, already applied by the FC1 GEMM's
    SwiGLU epilogue (same bytes as the fp16 [gate|up], identical values);
  - fp16 [M, Kl]   post-SwiGLU activation (kind 'act_f16'; not the reference's
    rounding, for the literal "SwiGLU output" entry of the FC2 benchmark config).

Modes (the reference's fc2_quantizer values):
  fused_stored    rotate + store FP32, MAX all-reduce, quantise the stored values;
  fused_recompute rotate for the maximum only, MAX all-reduce, recompute + quantise
                  (identical codes, 9 instead of 13 bytes of HBM traffic per value).
At TP=1 both collapse into one kernel that rotates, reduces and quantises a whole row.
"""
from __future__ import annotations

import torch

from . import comm as C
from . import ops
from . import peer as P
from . import transport as T
from .row_quant import label

MODES = ("fused_stored", "fused_recompute")


def input_kind(x: torch.Tensor, local_k: int | None = None) -> tuple[str, int]:
    """Classifies an FC2 input; returns (kind, local_k)."""
    width = x.shape[-1]
    if x.dtype == torch.float32:
        if local_k is not None and width == 2 * local_k:
            raise ValueError("FP32 [gate|up] input: apply SwiGLU in the FC1 epilogue instead")
        return "act_f32", width
    if x.dtype != torch.float16:
        raise ValueError("FC2 input must be fp16 [gate|up] or the fp32 SwiGLU activation")
    if local_k is not None and width == local_k:
        return "act_f16", width
    if width % 2:
        raise ValueError("[gate|up] input needs an even width")
    return "gateup_f16", width // 2


def _checked_input(x: torch.Tensor, mode: str, local_k: int | None):
    """(kind, local_k) of a valid FC2 input; ValueError otherwise, raised on every rank
    before any collective (tilelang_swiglu_quant.py:16)."""
    if mode not in MODES:
        raise ValueError(mode)
    kind, kl = input_kind(x, local_k)
    if kl % 256 or kl == 0:
        raise ValueError("Whole regular ConvRot256 groups required")
    return kind, kl


def prepare(x: torch.Tensor, comm, mode: str = "fused_stored", *, consume_input: bool = False,
            division: str = "rn", local_k: int | None = None, peer_workspace=None):
    """SwiGLU + ConvRot + global row quantisation (tilelang_swiglu_quant.py:67-92).
    Returns (q int8 [M, Kl], scale fp32 [M, 1]).

    With `peer_workspace` (a peer.PeerWorkspace of this group) and TP>1, one kernel
    rotates, exchanges the row maxima with the other ranks over peer memory and
    quantises: the same codes as either mode, one pass over x."""
    kind, kl = _checked_input(x, mode, local_k)
    flat = x.reshape(-1, x.shape[-1]).contiguous()
    if C.world_of(comm) == 1:
        q, s, _ = ops.swiglu_rotate_quantize_local(flat, kind, division)
        if consume_input:
            x.set_()
        return q, s
    if peer_workspace is not None:
        q, s = peer_workspace.quantize_rows(flat, kind, division)
        if consume_input:
            x.set_()
        return q, s
    rotated, maximum = ops.swiglu_rotate_max(flat, kind, store=(mode == "fused_stored"))
    if consume_input and mode == "fused_stored":
        # The stored kernel was the last reader; release the caller's storage before
        # the quantiser allocates its outputs (tilelang_swiglu_quant.py:81-85).
        del flat
        x.set_()
    C.all_reduce_max(maximum, comm)
    if mode == "fused_recompute":
        q, s = ops.swiglu_rotate_quantize(flat, maximum, kind, division)
        if consume_input:
            x.set_()
        return q, s
    return ops.row_quantize(rotated, maximum, division=division)


def supported(x, weight, weight_scale, world_size, groupsize) -> bool:
    """Complete contract, checked before either rank enters a collective
    (tilelang_swiglu_quant.py:95-105), generalised to TP 1/2/4/8 on sm_100."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.numel() > 0):
        return False
    if not (isinstance(weight, torch.Tensor) and weight.ndim == 2 and weight.dtype == torch.int8):
        return False
    try:
        _, kl = input_kind(x, weight.shape[1])
    except ValueError:
        return False
    return (kl % 256 == 0 and kl == weight.shape[1] and groupsize == 256
            and world_size in (1, 2, 4, 8) and weight.device == x.device
            and weight_scale.dtype == torch.float32 and weight_scale.is_contiguous()
            and weight_scale.numel() == weight.shape[0] and weight_scale.device == x.device
            and torch.cuda.get_device_capability(x.device) == (10, 0))


def _finish_quantized(q, scale, weight, weight_scale, comm, scaled_transport=True,
                      transport="rowblock", *, residual=None, gate=None, labels=None,
                      out_dtype=torch.float32, finish_fn=None, payload="fp16"):
    """GEMM -> (transport) -> epilogue of the quantised row activation (shared by FC2
    and the O projection; tilelang_swiglu_quant.py:116-127, tilelang_transport_p2.py:
    240-249).  Returns [M, N] in out_dtype, or the residual updated in place."""
    world = C.world_of(comm)
    local_k = q.shape[-1]
    if world == 1 and finish_fn is None:
        # TP=1: exact INT32 accumulators dequantised in the GEMM epilogue, no transport.
        with label("int8_gemm_dequant"):
            if residual is not None:
                return ops.int8_gemm_row_dequant(q, weight, scale, weight_scale,
                                                 residual=residual, gate=gate, labels=labels)
            return ops.int8_gemm_row_dequant(q, weight, scale, weight_scale, out_dtype)
    if scaled_transport and payload == "int8_gather":
        if finish_fn is not None:
            raise ValueError("The fused row-gate callback takes the fp16 payload")
        return T.int8_row_exchange(q, weight, scale, weight_scale, comm, transport,
                                   out_dtype=out_dtype, residual=residual, gate=gate,
                                   labels=labels)
    if scaled_transport:
        shift = T.shift_for(local_k, world)
        if (transport in ("p2p", "nvls") and residual is not None and finish_fn is None
                and residual.is_contiguous() and residual.shape[-1] % 8 == 0 and P.available(comm)):
            # p2p, push form: the GEMM's encode epilogue stores each partial row into its
            # owner's peer-mapped buffer (the reduce-scatter rides on the GEMM), then the
            # owner's local reduce + gated residual, the finished rows stored into every
            # peer, and the gather (csrc/h3_gemm.cu, csrc/h3_peer.cu).  Pull form (and
            # nvls): the GEMM writes locally and the reduce reads the peers.
            rows = q.shape[0]
            ws = P.workspace(comm, q.device, weight.shape[0], rows)
            form = P.exchange_form(world) if transport == "p2p" else "pull"
            push = form == "push"
            with label("int8_gemm_scaled_fp16_encode"):
                if push:
                    ws.encode_push(q, weight, shift)
                else:
                    ops.int8_gemm_row_encode(q, weight, shift, out=ws.partial(rows))
            with label("scaled_fp16_peer_reduce_gather"):
                if form == "dma":
                    return ws.reduce_and_gather_dma(rows, shift, scale, weight_scale, residual,
                                                    gate, labels)
                return ws.reduce_and_gather(rows, shift, scale, weight_scale, residual, gate, labels,
                                            nvls=transport == "nvls", pushed=push)
        with label("int8_gemm_scaled_fp16_encode"):
            payload = ops.int8_gemm_row_encode(q, weight, shift)
        if finish_fn is not None:
            with label("scaled_fp16_sum"):
                payload = T.collect(payload, "fp16", comm)
            with label("scaled_fp16_fused_epilogue"):
                return finish_fn(payload, scale, weight_scale, local_k)
        return T.reduce_and_finish(payload, comm, shift, scale, weight_scale, transport=transport,
                                   out_dtype=out_dtype, residual=residual, gate=gate, labels=labels)
    with label("int8_gemm"):
        partial = ops.int8_gemm_i32(q, weight)
    with label("int32_sum"):
        if world > 1:
            comm.all_reduce(partial, op=comm.ReduceOp.SUM)
    with label("dequantize"):
        out = ops.dequantize_i32(partial, scale, weight_scale, torch.float32)
    if residual is not None:
        from .h3_tensor_flow import gated_add_fp32
        return gated_add_fp32(residual, out, gate, labels)
    return out if out_dtype == torch.float32 else out.to(out_dtype)


def row_linear(x, weight, weight_scale, comm, *, mode="fused_stored", scaled_transport=True,
               finish_fn=None, consume_input=False, p0_b=False, residual=None, gate=None,
               labels=None, transport="rowblock", division="rn", out_dtype=torch.float32,
               payload="fp16", peer_max=True):
    """FC2 row linear (tilelang_swiglu_quant.py:108-128).

    Returns FP32 [..., N] (the caller adds LoRA, then stores once), or with
    `residual` the gated residual updated in place.  finish_fn keeps the reference's
    callback form: it receives the all-reduced fp16 payload.
    p0_b (the T4 in-place storage trick) is accepted and ignored: on B200 the FP32
    SwiGLU lives in the FC1 epilogue's own output instead.
    With the p2p transport (residual form, NCCL group) the row maxima are exchanged in
    the producer kernel over the same peer workspace unless peer_max is False; the
    peer reduce that follows synchronises the ranks before the slots are reused."""
    if finish_fn is not None and not scaled_transport:
        raise ValueError("Fused row-gate requires scaled FP16 transport")
    shape = x.shape
    ws = None
    _checked_input(x, mode, weight.shape[1])  # before the workspace's collective steps
    if (peer_max and transport in ("p2p", "nvls") and scaled_transport and finish_fn is None
            and residual is not None and residual.is_contiguous()
            and (payload == "int8_gather" or residual.shape[-1] % 8 == 0)
            and C.world_of(comm) > 1 and weight.shape[1] <= ops.PEER_PRODUCER_MAX_WIDTH
            and P.available(comm)):
        ws = P.workspace(comm, x.device, weight.shape[0], x.numel() // x.shape[-1])
    with label("fp32_swiglu_convrot_quantize"):
        q, scale = prepare(x, comm, mode, consume_input=consume_input, division=division,
                           local_k=weight.shape[1], peer_workspace=ws)
    del x
    out = _finish_quantized(q, scale, weight, weight_scale.reshape(-1), comm, scaled_transport,
                            transport, residual=residual, gate=gate, labels=labels,
                            out_dtype=out_dtype, finish_fn=finish_fn, payload=payload)
    if residual is not None or finish_fn is not None:
        return out
    return out.reshape(*shape[:-1], weight.shape[0])
