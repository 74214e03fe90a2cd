"""Fused DiT row-gate epilogue on B200 (mirror of the row parts of
patches/tilelang_dit_fusion.py).

row_gated() runs a RowParallel projection (O or FC2) and writes its output straight
into the fp16 residual stream:
    X[r, c] = f16(fma(f32(f16(y[r, c])), Gate[label[r], c], f32(X[r, c])))
with y the dequantised FP32 row output (tilelang_dit_fusion.py:57-77).  It returns
None, before any collective, when the call cannot take the fused route, exactly like
the reference (tilelang_dit_fusion.py:153-168).
"""
from __future__ import annotations

import threading
from functools import lru_cache

import torch

from . import comm as C
from . import ops


def segment_key(rows, segments, modulation_rows=9):
    """Validated, hashable segments: [(a, b, row)] tiling [0, rows) exactly
    (tilelang_dit_fusion.py:93-100)."""
    key = tuple(tuple(s) for s in segments)
    cursor = 0
    for a, b, row in sorted(key):
        if (any(type(v) is not int for v in (a, b, row)) or a != cursor
                or not a < b <= rows or not 0 <= row < modulation_rows):
            return None
        cursor = b
    return key if cursor == rows else None


_label_lock = threading.RLock()


@lru_cache(maxsize=4)
def _labels(rows, segments, device):
    labels = torch.empty(rows, dtype=torch.int32)
    for a, b, row in segments:
        labels[a:b] = row
    labels = labels.to(device)
    ready = torch.cuda.Event()
    ready.record(torch.cuda.current_stream(device))
    return labels, ready


def _norm_supported(norm, x, shift, scale):
    return (isinstance(x, torch.Tensor) and x.is_cuda and x.ndim == 2 and x.shape[0] > 0
            and x.dtype == torch.float16 and x.shape[1] % 16 == 0 and x.shape[1] <= 32768
            and not getattr(norm, "layer_norm", False)
            and tuple(getattr(norm, "normalized_shape", ())) == (x.shape[1],)
            and getattr(norm, "weight", None) is not None
            and norm.weight.dtype == torch.float32 and norm.weight.device == x.device
            and shift.ndim == 2 and shift.shape == scale.shape and shift.shape[1] == x.shape[1]
            and shift.dtype == torch.float32 and scale.dtype == torch.float32
            and shift.device == x.device and scale.device == x.device)


def modulated_norm(norm, x, shift, scale, segments):
    """Fused modulated RMSNorm (tilelang_dit_fusion.py:127-134): fp16 h, or None when the
    fused kernel does not apply (the caller then runs its own path)."""
    if not _norm_supported(norm, x, shift, scale):
        return None
    labels = labels_for(x, segments, shift.shape[0])
    if labels is None:
        return None
    _, _, h = ops.modulated_norm_quantize(x, norm.weight, float(norm.eps), shift.contiguous(),
                                          scale.contiguous(), labels, quantize=False)
    return h


def modulated_norm_quantize(norm, x, shift, scale, segments, convrot=True):
    """The column input producer: modulated RMSNorm -> (ConvRot256) -> per-row INT8
    quantisation in one kernel, h never stored.  Returns (codes, row_scale), the
    operands of ColumnParallelLinearINT8.forward_quantized, or None."""
    if not _norm_supported(norm, x, shift, scale) or (convrot and x.shape[1] % 256):
        return None
    labels = labels_for(x, segments, shift.shape[0])
    if labels is None:
        return None
    q, s, _ = ops.modulated_norm_quantize(x, norm.weight, float(norm.eps), shift.contiguous(),
                                          scale.contiguous(), labels, convrot=convrot)
    return q, s


def labels_for(x, segments, modulation_rows=9):
    """Per-row modulation labels on x's device, cached (tilelang_dit_fusion.py:115-124)."""
    if segments is None:
        return None
    key = segment_key(x.shape[0], segments, modulation_rows)
    if key is None:
        return None
    with _label_lock:
        labels, ready = _labels(x.shape[0], key, str(x.device))
    stream = torch.cuda.current_stream(x.device)
    stream.wait_event(ready)
    labels.record_stream(stream)
    return labels


def _table(value, x, rows=None):
    return (value.ndim == 2 and value.shape[0] >= 1 and value.shape[1] == x.shape[1]
            and (rows is None or value.shape[0] == rows)
            and value.dtype == torch.float32 and value.device == x.device)


def supported(x) -> bool:
    return (not torch.is_grad_enabled() and x.is_cuda and x.ndim == 2 and x.shape[0] > 0
            and x.dtype == torch.float16 and x.is_contiguous()
            and torch.cuda.get_device_capability(x.device) == (10, 0))


def finish_row(payload, scale, weights, residual, gate, labels, local_k, world_size=2):
    """Decode + dequant + gated residual of an all-reduced payload
    (tilelang_dit_fusion.py:146-150)."""
    from .transport import shift_for
    return ops.row_reduce_finish(payload, shift_for(local_k, world_size), scale, weights,
                                 residual=residual, gate=gate, labels=labels)


def row_gated(module, value, residual, gate, segments, comm, input_act=None):
    """RowParallel projection fused into the gated residual; None when not fusable."""
    policy = getattr(module, "operator_policy", None)
    if (policy is None or not getattr(policy, "dit_fused_row_gate", False)
            or getattr(module, "lora_adapter", None) is not None or not supported(residual)
            or (gate is not None and not _table(gate, residual))
            or value.ndim != 2 or value.shape[0] != residual.shape[0]
            or value.device != residual.device or not value.is_contiguous()
            or not module.convrot or module.convrot_groupsize != 256):
        return None
    world = C.world_of(comm)
    if module.world_size != world:
        return None
    kl = module.weight.shape[1]
    if (input_act not in (None, "swiglu") or module.weight.dtype != torch.int8
            or module.weight.shape[0] != residual.shape[1]
            or module.weight_scale.numel() != residual.shape[1]
            or module.weight_scale.dtype != torch.float32 or kl % 256):
        return None
    labels = None
    if gate is not None:
        labels = labels_for(residual, segments, gate.shape[0])
        if labels is None:
            return None
        gate = gate.contiguous()
    ws = module.weight_scale.reshape(-1)
    transport = getattr(policy, "row_transport", "rowblock")
    payload = getattr(policy, "row_payload", "fp16")
    division = getattr(policy, "quant_division", "rn")
    scaled = policy.row_linear_backend in ("tilelang_scaled_fp16", "b200_scaled_fp16")
    if input_act == "swiglu":
        if policy.fc2_quantizer not in ("fused_stored", "fused_recompute"):
            return None
        from .swiglu_quant import row_linear
        consume = bool(getattr(module, "_vram_p0_3", False) and policy.fc2_quantizer == "fused_stored"
                       and not torch.is_grad_enabled() and type(value) is torch.Tensor)
        return row_linear(value, module.weight, ws, comm, mode=policy.fc2_quantizer,
                          scaled_transport=scaled, consume_input=consume, residual=residual,
                          gate=gate, labels=labels, transport=transport, division=division,
                          payload=payload,
                          peer_max=getattr(policy, "fc2_max_exchange", "peer") == "peer")
    if value.dtype not in (torch.float16, torch.float32) or value.shape[1] != kl:
        return None
    from .row_quant import global_row_quantize
    from .swiglu_quant import _finish_quantized
    q, scale = global_row_quantize(value, comm, world, 256, None, division=division)
    return _finish_quantized(q, scale, module.weight, ws, comm, scaled, transport,
                             residual=residual, gate=gate, labels=labels, payload=payload)
