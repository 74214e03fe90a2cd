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

from collections import OrderedDict

import numpy as np
import torch

from . import comm as C
from . import ops


def segment_key(rows, segments, modulation_rows=9):
    """The segment layout as a hashable, validated tuple, or None when it is not one.

    A layout is a list of (start, end, modulation_row) triples of plain ints that,
    taken in order of their starts, tile [0, rows) without gap or overlap, each with
    start < end and a modulation row in [0, modulation_rows) - the contract of the
    reference's segment check (tilelang_dit_fusion.py:93-100)."""
    triples = [tuple(seg) for seg in segments]
    if any(len(t) != 3 for t in triples):
        raise ValueError("segments are (start, end, modulation_row) triples")
    if any(type(v) is not int for t in triples for v in t):
        return None
    ordered = sorted(triples)
    bounds = [0] + [t[1] for t in ordered]
    if any(t[0] != b for t, b in zip(ordered, bounds)) or bounds[-1] != rows:
        return None
    if any(not (t[0] < t[1] and 0 <= t[2] < modulation_rows) for t in ordered):
        return None
    return tuple(triples)


class _LabelCache:
    """Per-row modulation labels (int32, one per row) on each device, built once per
    segment layout and kept in a small least-recently-used table per device.

    A label vector is built from the layout on the host, copied to the device and
    waited for before it is cached, so it is complete for every stream that reads it
    later; a reader on a stream other than the one that built it is recorded on the
    tensor, so the allocator keeps the memory until that stream's work is done even if
    the entry is evicted meanwhile."""

    def __init__(self, capacity: int = 8):
        self.capacity = capacity
        self.tables: dict = {}

    def get(self, device: torch.device, rows: int, key: tuple) -> torch.Tensor:
        table = self.tables.setdefault(device, OrderedDict())
        entry = table.get((rows, key))
        if entry is None:
            ordered = sorted(key)
            labels = np.repeat(np.array([t[2] for t in ordered], dtype=np.int32),
                               [t[1] - t[0] for t in ordered])
            with torch.cuda.device(device):
                built_on = torch.cuda.current_stream(device)
                tensor = torch.from_numpy(labels).to(device)
                built_on.synchronize()
            entry = (tensor, built_on)
            table[(rows, key)] = entry
            while len(table) > self.capacity:
                table.popitem(last=False)
        else:
            table.move_to_end((rows, key))
        tensor, built_on = entry
        reader = torch.cuda.current_stream(device)
        if reader != built_on:
            tensor.record_stream(reader)
        return tensor


_LABELS = _LabelCache()


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
    """Per-row modulation labels for x's rows on x's device, or None when `segments` is
    None or not a valid layout (tilelang_dit_fusion.py:107-124)."""
    if segments is None:
        return None
    key = segment_key(x.shape[0], segments, modulation_rows)
    if key is None:
        return None
    return _LABELS.get(x.device, x.shape[0], key)


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
            or module.weight_scale.dtype != torch.float32
            or (kl % 256 if input_act == "swiglu" else (kl * world) % 256)):
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
