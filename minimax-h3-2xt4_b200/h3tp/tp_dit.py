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
        return mlp_forward(self.fc1, self.fc2, x, h, gate, segments)

    def pipeline_chunks(self, x, h, gate=None) -> int:
        return mlp_pipeline_chunks(self.fc1, self.fc2, x, h, gate)

    def forward_pipelined(self, x, h, gate=None, segments=None, chunks: int = 4, timer=None):
        return mlp_forward_pipelined(self.fc1, self.fc2, x, h, gate, segments, chunks, timer)


def mlp_forward(fc1, fc2, x, h, gate=None, segments=None):
    """FC1 -> FC2 with the gated residual: pipelined over row chunks where
    mlp_pipeline_chunks allows it, else the plain module chain."""
    chunks = mlp_pipeline_chunks(fc1, fc2, x, h, gate)
    if chunks > 1:
        return mlp_forward_pipelined(fc1, fc2, x, h, gate, segments, chunks)
    fc1_out = fc1(h)
    return fc2(fc1_out, input_act="swiglu", residual=x, gate=gate, segments=segments)


def mlp_pipeline_chunks(fc1, fc2, x, h, gate=None) -> int:
    """Row chunks of the pipelined TP > 1 forward (1: the plain module chain).

    The pipelined form needs the peer-memory row transport (p2p or nvls) with the
    scaled-fp16 payload, the in-kernel maximum exchange, FC1's SwiGLU epilogue, no
    LoRA, an NCCL group, and fp16 contiguous [S, hidden] residual and input."""
    from . import ops, peer as P
    pol = getattr(fc2, "operator_policy", None)
    world = fc2.world_size
    if (pol is None or world == 1 or pol.mlp_pipeline_chunks == 1
            or pol.row_transport not in ("p2p", "nvls") or pol.row_payload != "fp16"
            or pol.fc2_max_exchange != "peer" or not pol.scaled_transport
            or pol.fc2_quantizer not in ("fused_stored", "fused_recompute")
            or not getattr(fc1, "_swiglu_epilogue", False)
            or getattr(fc1, "lora_adapter", None) is not None
            or getattr(fc2, "lora_adapter", None) is not None
            or torch.is_grad_enabled()):
        return 1
    hidden, kl = fc2.out_features, fc2.in_features_per_rank
    if (x.dtype != torch.float16 or h.dtype != torch.float16 or x.ndim != 2 or h.ndim != 2
            or x.shape != h.shape or x.shape[1] != hidden or not x.is_contiguous()
            or not h.is_contiguous() or not x.is_cuda or hidden % 8 or kl % 256
            or kl > ops.PEER_PRODUCER_MAX_WIDTH or (gate is not None and gate.ndim != 2)):
        return 1
    if not P.available(fc2._comm()):
        return 1
    rows = x.shape[0]
    chunks = pol.mlp_pipeline_chunks or (4 if rows >= 4 * 4096 else 2 if rows >= 2 * 2048 else 1)
    return max(1, min(chunks, rows // 256))


def mlp_forward_pipelined(fc1, fc2, x, h, gate=None, segments=None, chunks: int = 4,
                          timer=None):
    """The TP > 1 forward over row chunks, with the partial-sum exchange of one chunk
    overlapping the GEMMs of the next.

    Per chunk c: column quantise + FC1 GEMM with the SwiGLU epilogue (F_c), the FC2
    producer with the row maxima exchanged in the kernel (P_c), the FC2 GEMM writing
    its scaled-fp16 partial into the peer workspace (G_c), the reduce + gated
    residual of the rank's rows (R_c) and the gather of the other ranks' rows.  F and G
    run on the caller's stream; P and R, the only kernels that wait for other ranks,
    run on one exchange stream in the same order on every rank (P0, P1, R0, P2, R1,
    ..., R_{n-1}), so no two kernels that wait on other GPUs are ever in flight
    together on a GPU.  Issue order on the caller's stream is F0, F1, G0, F2, G1, ...:
    R_c, which is bound by NVLink and holds few SM resources, runs while the tensor
    cores work on F_{c+2} and G_{c+1}.  The bits are those of forward(): the same
    kernels on the same rows, the rows of a chunk reduced in rank order.
    `timer(name, chunk, start_or_end)` (optional) is called around each launch to
    record events on the stream it runs on."""
    from . import ops, peer as P, transport as T
    from .dit_fusion import labels_for
    dev = x.device
    rows, hidden = x.shape
    world = fc2.world_size
    kl = fc2.in_features_per_rank
    pol = fc2.operator_policy
    comm = fc2._comm()
    labels = None
    if gate is not None:
        labels = labels_for(x, segments, gate.shape[0])
        if labels is None:
            raise ValueError("gate given without a valid segment layout")
        gate = gate.contiguous()
    ws = P.workspace(comm, dev, hidden, rows)
    comp = torch.cuda.current_stream(dev)
    xs = _exchange_stream(dev)
    q1 = torch.empty((rows, hidden), dtype=torch.int8, device=dev)
    s1 = torch.empty((rows, 1), dtype=torch.float32, device=dev)
    act = torch.empty((rows, kl), dtype=torch.float32, device=dev)
    q2 = torch.empty((rows, kl), dtype=torch.int8, device=dev)
    s2 = torch.empty((rows, 1), dtype=torch.float32, device=dev)
    for t in (act, q2, s2, x) + tuple(v for v in (gate, labels) if v is not None):
        t.record_stream(xs)
    xs.wait_stream(comp)
    shift = T.shift_for(kl, world)
    w1s = fc1.weight_scale.reshape(-1)
    w2s = fc2.weight_scale.reshape(-1)
    nvls = pol.row_transport == "nvls"
    bounds = pipeline_bounds(rows, chunks)
    ev = {k: [torch.cuda.Event() for _ in bounds] for k in ("fc1", "prod", "fc2")}
    mark = timer or (lambda *a: None)

    def front(c):
        a, b = bounds[c]
        mark("column_quantize", c, 0)
        ops.column_quantize(h[a:b], True, out_q=q1[a:b], out_scale=s1[a:b])
        mark("column_quantize", c, 1)
        mark("fc1_gemm", c, 0)
        ops.int8_gemm_swiglu(q1[a:b], fc1.weight, s1[a:b], w1s, None, torch.float32,
                             out=act[a:b])
        mark("fc1_gemm", c, 1)
        ev["fc1"][c].record(comp)

    def producer(c):
        a, b = bounds[c]
        xs.wait_event(ev["fc1"][c])
        with torch.cuda.stream(xs):
            mark("peer_producer", c, 0)
            ws.quantize_rows_at(act[a:b], a, "act_f32", pol.quant_division, out_q=q2[a:b],
                                out_scale=s2[a:b])
            mark("peer_producer", c, 1)
        ev["prod"][c].record(xs)

    def back(c):
        a, b = bounds[c]
        comp.wait_event(ev["prod"][c])
        mark("fc2_gemm", c, 0)
        ops.int8_gemm_row_encode(q2[a:b], fc2.weight, shift, out=ws.partial_rows(a, b - a))
        mark("fc2_gemm", c, 1)
        ev["fc2"][c].record(comp)

    def exchange(c):
        a, b = bounds[c]
        xs.wait_event(ev["fc2"][c])
        with torch.cuda.stream(xs):
            mark("reduce_gather", c, 0)
            ws.reduce_rows(a, b - a, shift, s2[a:b], w2s, x[a:b], gate,
                           None if labels is None else labels[a:b], nvls=nvls)
            ws.gather_rows(a, b - a, x[a:b])
            mark("reduce_gather", c, 1)

    n = len(bounds)
    front(0)
    producer(0)
    for c in range(n):
        if c + 1 < n:
            front(c + 1)
            producer(c + 1)
        back(c)
        exchange(c)
    comp.wait_stream(xs)
    return x


def pipeline_bounds(rows: int, chunks: int) -> list[tuple[int, int]]:
    """Row ranges of the pipelined forward: about rows / chunks each, starting on
    256-row boundaries (whole GEMM tiles), the last one ragged; never empty."""
    per = -(-rows // max(1, chunks))
    per = max(256, -(-per // 256) * 256)
    return [(a, min(rows, a + per)) for a in range(0, rows, per)]


_EXCHANGE_STREAMS: dict = {}


def _exchange_stream(device) -> torch.cuda.Stream:
    """The stream that carries the cross-rank kernels of the pipelined forward (one per
    device, created on first use)."""
    device = torch.device(device)
    st = _EXCHANGE_STREAMS.get(device)
    if st is None:
        st = torch.cuda.Stream(device)
        _EXCHANGE_STREAMS[device] = st
    return st


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
        del qkv
        x = self.out_proj(attn_out, residual=x, gate=gate_msa, segments=segments)
        # FC1 reads the updated residual (the norm is the identity here): a copy, since
        # the MLP updates x in place
        return mlp_forward(self.fc1, self.fc2, x, x.clone(), gate_mlp, segments)
