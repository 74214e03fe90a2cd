"""Residual gauge of the FP16 DiT tensor flow (mirror of the parts of
patches/h3_tensor_flow.py that touch the INT8 linear path).

The residual stream is stored divided by 2**residual_exponent (512 by default), and
that divisor is folded once into the FP32 weight scales of the row projections
(out_proj, fc2) that write into it (h3_tensor_flow.py:82-127).  No INT8 weight is
requantised.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from . import ops


@dataclass(frozen=True)
class TensorFlowPolicy:
    mode: str = "fp16"
    residual_exponent: int = 9
    vision_residual_exponent: int = 0
    video_residual_exponent: int = 0

    def __post_init__(self):
        if self.mode not in ("legacy", "fp16", "bf16_reference"):
            raise ValueError("Unknown H3 tensor flow")
        for value in (self.residual_exponent, self.vision_residual_exponent,
                      self.video_residual_exponent):
            if type(value) is not int or not 0 <= value <= 12:
                raise ValueError("Residual exponent must be an integer in [0,12]")

    @property
    def enabled(self):
        return self.mode != "legacy"

    @property
    def dtype(self):
        return torch.bfloat16 if self.mode == "bf16_reference" else torch.float16

    @property
    def divisor(self):
        return float(2 ** self.residual_exponent)


def fold_linear(module, divisor: float) -> None:
    """weight_scale <- f32(weight_scale) / divisor (h3_tensor_flow.py:82-91)."""
    base = getattr(module, "base", module)
    if not hasattr(base, "weight_scale"):
        raise ValueError("Residual folding requires FP32 INT8 weight scales")
    base.weight_scale = nn.Parameter(base.weight_scale.detach().float() / divisor,
                                     requires_grad=False)
    bias = getattr(base, "bias", None)
    if bias is not None:
        base.bias = nn.Parameter(bias.detach() / divisor, requires_grad=False)


def prepare_tp(block, kind: str, policy: TensorFlowPolicy):
    """Folds the residual divisor into the row projections of a TP block
    (h3_tensor_flow.py:114-127, linear part)."""
    if not policy.enabled:
        return block
    if hasattr(block, "tensor_flow"):
        raise ValueError("Tensor flow already prepared")
    block.tensor_flow = policy
    names = ("o_proj", "down_proj") if kind == "te" else ("out_proj", "fc2")
    for name in names:
        if getattr(block, name, None) is not None:
            fold_linear(getattr(block, name), policy.divisor)
    return block


def gated_add(x, gate, branch, segments=None, *, labels=None, fused=True):
    """x <- f16(fma(f16(branch), gate[row], x)) in place (h3_tensor_flow.py:145-152;
    fused kernel tilelang_dit_fusion.py:39-53).  gate: fp32 [rows_mod, N] table or None
    (unit gate); segments [(a, b, row)] or labels [M] select the table row."""
    if gate is not None and labels is None:
        from .dit_fusion import labels_for
        labels = labels_for(x, segments, gate.shape[0])
        if labels is None:
            raise ValueError("segments must tile the rows exactly")
    return ops.gated_add(x, branch.reshape(x.shape), gate, labels)


def gated_add_fp32(residual, out, gate=None, labels=None):
    """Gated residual from an FP32 row output (rounded to fp16 first, as the row
    projection's .to(fp16) does, tp_dit.py:157)."""
    return ops.gated_add(residual, out.reshape(residual.shape).float().contiguous(), gate, labels)
