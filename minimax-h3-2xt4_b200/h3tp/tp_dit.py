"""Tensor-parallel INT8 linear modules of the DiT block (mirror of patches/tp_dit.py).

ColumnParallelLinearINT8 / RowParallelLinearINT8 keep the reference's constructor
arguments, parameters (int8 `weight`, fp32 `weight_scale` [., 1]), shard loaders and
forward signatures (tp_dit.py:25-162), so they drop into the same call sites.  All
arithmetic runs in libh3b200.so; collectives go through `self.comm` (torch.distributed
by default, the reference's `dist`).

TPDiTMLPINT8 and TPDiTLinearBlockINT8 chain the projections the way
TPDiTBlockINT8.forward does (tp_dit.py:260-368) minus attention and the norms, which
are outside this path: they exist to run and measure the linear set end to end.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import comm as C
from .parallel_int8 import packed_rows, row_linear


def default_comm():
    """torch.distributed when a process group is up, else None (single rank)."""
    return dist if dist.is_available() and dist.is_initialized() else None


def _check_device_error(x: torch.Tensor) -> None:
    """Raises if a kernel enqueued earlier on x's GPU recorded a failure (a bounded
    wait that gave up, a label out of range).  One read of host-mapped memory, no
    device synchronisation."""
    if x.is_cuda:
        from ._native import raise_on_device_error
        raise_on_device_error(x.device.index if x.device.index is not None
                              else torch.cuda.current_device(), "INT8 linear")


def run_int8_linear_forward(x, weight, weight_scale, convrot=True, convrot_groupsize=256,
                            out_dtype=torch.float16, backend="b200", p0_a1=False, **kw):
    from .dit_column_linear import column_linear
    return column_linear(x, weight, weight_scale, out_dtype=out_dtype, convrot=convrot,
                         convrot_groupsize=convrot_groupsize, backend=backend, p0_a1=p0_a1, **kw)


class ColumnParallelLinearINT8(nn.Module):
    """Column-parallel INT8 linear: output features split across TP ranks, no
    communication.  Input [S, in_features] fp16 -> output [S, out_features // world]
    fp16, the reference's layout (for FC1 the component-packed [gate_r | up_r]).

    Opt-in change of output: when the operator policy sets `fc1_swiglu_epilogue`
    (configure_block copies it into `_swiglu_epilogue`) and components == 2, FC1 returns
    the FP32 SwiGLU activation silu(f16 gate) * f16 up, shape [S, out_features // world
    // 2] and dtype float32 - the same bytes as the fp16 [gate|up] it replaces, and the
    same INT8 codes in FC2, whose producer then skips the SwiGLU.  Only callers that hand
    FC1's output straight to RowParallelLinearINT8(input_act='swiglu') should turn it on."""

    def __init__(self, in_features: int, out_features: int, rank: int = 0, world_size: int = 2,
                 convrot: bool = True, convrot_groupsize: int = 256,
                 device: Optional[torch.device] = None, components: int = 1):
        super().__init__()
        assert out_features % world_size == 0
        self.components = components
        self.in_features = in_features
        self.out_features_per_rank = out_features // world_size
        self.rank = rank
        self.world_size = world_size
        self.convrot = convrot
        self.convrot_groupsize = convrot_groupsize
        self.device = torch.device(device) if device is not None else torch.device("cuda", rank)
        self.weight = nn.Parameter(torch.empty(self.out_features_per_rank, in_features,
                                               dtype=torch.int8, device=self.device),
                                   requires_grad=False)
        self.weight_scale = nn.Parameter(torch.empty(self.out_features_per_rank, 1,
                                                     dtype=torch.float32, device=self.device),
                                         requires_grad=False)
        self.bias = None

    def load_shard_from_full(self, full_weight: torch.Tensor, full_scale: torch.Tensor):
        w, scale = packed_rows(full_weight, full_scale, self.rank, self.world_size, self.components)
        self.weight.data.copy_(w)
        self.weight_scale.data.copy_(scale.reshape(-1, 1))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _check_device_error(x)
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features)
        policy = getattr(self, "operator_policy", None)
        adapter = getattr(self, "lora_adapter", None)
        swiglu = bool(self.components == 2 and getattr(self, "_swiglu_epilogue", False)
                      and adapter is None)
        options = {}
        if policy is not None:
            options["backend"] = policy.column_linear_backend
        out = run_int8_linear_forward(x_2d, self.weight, self.weight_scale, convrot=self.convrot,
                                      convrot_groupsize=self.convrot_groupsize,
                                      out_dtype=torch.float16, swiglu=swiglu, bias=self.bias,
                                      **options)
        width = self.out_features_per_rank // 2 if swiglu else self.out_features_per_rank
        out = out.view(*orig_shape[:-1], width)
        return adapter.add_to(x, out) if adapter is not None else out

    def forward_quantized(self, codes: torch.Tensor, row_scale: torch.Tensor) -> torch.Tensor:
        """forward() on activation codes from the fused modulated-norm producer
        (h3tp.dit_fusion.modulated_norm_quantize); no LoRA (it needs the fp16 input)."""
        from .dit_column_linear import column_linear_quantized
        if getattr(self, "lora_adapter", None) is not None:
            raise ValueError("forward_quantized has no LoRA path: use forward(h)")
        swiglu = bool(self.components == 2 and getattr(self, "_swiglu_epilogue", False))
        return column_linear_quantized(codes, row_scale, self.weight, self.weight_scale,
                                       bias=self.bias, swiglu=swiglu)


class RowParallelLinearINT8(nn.Module):
    """Row-parallel INT8 linear: input features split across TP ranks, partial sums
    reduced across the group.  Input [S, in_features // world] -> output
    [S, out_features] (fp16), or the fp16 residual updated in place when `residual`
    is given."""

    def __init__(self, in_features: int, out_features: int, rank: int = 0, world_size: int = 2,
                 convrot: bool = True, convrot_groupsize: int = 256,
                 device: Optional[torch.device] = None):
        super().__init__()
        assert in_features % world_size == 0
        self.in_features_per_rank = in_features // world_size
        self.out_features = out_features
        self.rank = rank
        self.world_size = world_size
        self.convrot = convrot
        self.convrot_groupsize = convrot_groupsize
        self.device = torch.device(device) if device is not None else torch.device("cuda", rank)
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_rank,
                                               dtype=torch.int8, device=self.device),
                                   requires_grad=False)
        self.weight_scale = nn.Parameter(torch.empty(out_features, 1, dtype=torch.float32,
                                                     device=self.device),
                                         requires_grad=False)
        self.comm = None

    def load_shard_from_full(self, full_weight: torch.Tensor, full_scale: torch.Tensor):
        start = self.rank * self.in_features_per_rank
        end = start + self.in_features_per_rank
        self.weight.data.copy_(full_weight[:, start:end].to(self.device))
        self.weight_scale.data.copy_(full_scale.reshape(-1, 1).to(self.device))

    def _comm(self):
        comm = self.comm if self.comm is not None else default_comm()
        if self.world_size > 1 and C.world_of(comm) != self.world_size:
            raise RuntimeError("Row-parallel projection needs an initialised TP group of "
                               f"{self.world_size} ranks")
        return comm if self.world_size > 1 else None

    def forward(self, x: torch.Tensor, reduce_sum: bool = True, input_act=None, *,
                residual=None, gate=None, segments=None) -> torch.Tensor:
        if not reduce_sum and self.world_size > 1:
            raise ValueError("Quantization-preserving projection requires reduction")
        _check_device_error(x)
        comm = self._comm()
        if residual is not None:
            from .dit_fusion import row_gated
            fused = row_gated(self, x, residual, gate, segments, comm, input_act)
            if fused is not None:
                return fused
        from .h3_operator_policy import row_linear as dispatch_row
        out = dispatch_row(self, x, row_linear, comm, input_act)
        adapter = getattr(self, "lora_adapter", None)
        if adapter is not None:
            source = x.float() if out.dtype == torch.float32 else x
            out = adapter.add_to(source, out, comm=comm, input_act=input_act)
        target = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
        if residual is not None:
            from .h3_tensor_flow import gated_add_fp32
            labels = None
            if gate is not None:
                from .dit_fusion import labels_for
                labels = labels_for(residual, segments, gate.shape[0])
            return gated_add_fp32(residual, out, gate, labels)
        return out.to(target)


class TPDiTMLPINT8(nn.Module):
    """DiT MLP of one TP rank: FC1 (column, [gate|up]) -> FP32 SwiGLU -> ConvRot256
    -> global row quant -> FC2 (row) -> partial-sum reduction -> gated residual add
    (tp_dit.py:347-366)."""

    def __init__(self, hidden: int = 3072, ffn: int = 8192, rank: int = 0, world_size: int = 1,
                 device=None, policy=None, comm=None):
        super().__init__()
        from .h3_operator_policy import H3OperatorPolicy, configure_block
        self.fc1 = ColumnParallelLinearINT8(hidden, 2 * ffn, rank, world_size, components=2,
                                            device=device)
        self.fc2 = RowParallelLinearINT8(ffn, hidden, rank, world_size, device=device)
        self.fc2.comm = comm
        # FC1's output feeds FC2 only, so the FP32 SwiGLU epilogue is on unless the
        # caller's policy says otherwise
        configure_block(self, "dit", policy or H3OperatorPolicy(fc1_swiglu_epilogue=True))

    def forward(self, x: torch.Tensor, h: torch.Tensor, gate=None, segments=None) -> torch.Tensor:
        """x: fp16 residual [S, hidden] (updated in place); h: fp16 normed input."""
        fc1_out = self.fc1(h)
        return self.fc2(fc1_out, input_act="swiglu", residual=x, gate=gate, segments=segments)


class TPDiTLinearBlockINT8(nn.Module):
    """The four INT8 projections of one DiT block on one TP rank, chained with fp16
    residual adds: QKV (column) -> O (row, + residual) -> FC1 (column) -> FC2 (row,
    + residual).  Attention and the modulated norms are outside the INT8 linear path;
    here the norm is the identity and the attention output is the V third of QKV."""

    def __init__(self, hidden: int = 3072, ffn: int = 8192, rank: int = 0, world_size: int = 1,
                 device=None, policy=None, comm=None):
        super().__init__()
        from .h3_operator_policy import H3OperatorPolicy, configure_block
        self.hidden = hidden
        self.world_size = world_size
        self.qkv_proj = ColumnParallelLinearINT8(hidden, 3 * hidden, rank, world_size,
                                                 components=3, device=device)
        self.out_proj = RowParallelLinearINT8(hidden, hidden, rank, world_size, device=device)
        self.fc1 = ColumnParallelLinearINT8(hidden, 2 * ffn, rank, world_size, components=2,
                                            device=device)
        self.fc2 = RowParallelLinearINT8(ffn, hidden, rank, world_size, device=device)
        self.out_proj.comm = comm
        self.fc2.comm = comm
        configure_block(self, "dit", policy or H3OperatorPolicy(fc1_swiglu_epilogue=True))

    def forward(self, x: torch.Tensor, gate_msa=None, gate_mlp=None, segments=None) -> torch.Tensor:
        inner = self.hidden // self.world_size
        qkv = self.qkv_proj(x)
        attn_out = qkv[:, 2 * inner:3 * inner].contiguous()
        x = self.out_proj(attn_out, residual=x, gate=gate_msa, segments=segments)
        fc1_out = self.fc1(x)
        return self.fc2(fc1_out, input_act="swiglu", residual=x, gate=gate_mlp, segments=segments)
