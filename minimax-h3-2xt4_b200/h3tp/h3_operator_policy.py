"""Per-session operator selection (mirror of the linear-path parts of
patches/h3_operator_policy.py).

The reference's fields are kept with their names and value sets, and a `b200` value
is added to each backend field.  The T4-only values map onto the B200 kernels:
  row_linear_backend   'tilelang_scaled_fp16' / 'b200_scaled_fp16' -> scaled-FP16 transport
                       'tilelang_packed' / 'native' / 'b200_int32'  -> exact INT32 SUM
  fc2_quantizer        'fused_stored' / 'fused_recompute' -> B200 FC2 producer
                       'native' / 'owned_fp32' -> FP32 cast + full-gather exact route
  column_linear_backend 'preallocated' / 'cuda_int8_tilelang' / 'b200' -> B200 column GEMM
New B200 fields:
  row_transport   'p2p' (reduce + gather over NVLink peer memory, own kernels; the
                  default), 'rowblock' (NCCL all_to_all + fixed-order reduce + all_gather)
                  or 'allreduce' (NCCL fp16 SUM, the reference's form).  All three give
                  the same bits; 'p2p' needs a torch.distributed NCCL group and the
                  residual form of the row output, and uses 'rowblock' otherwise.
                  'nvls': 'p2p' with the fp16 partials summed inside the NVSwitch
                  (multimem.ld_reduce) and the finished rows broadcast through it
                  (multimem.st) where the group's symmetric memory has a multicast
                  address (else 'p2p'); the same bits as 'p2p' at TP 2, at TP 4/8 the
                  switch's summation order (rare last-bit differences of the fp16 sum)
  fc2_max_exchange 'peer' (default: under 'p2p' the FC2 producer exchanges its row
                  maxima over the peer workspace inside the kernel, one pass instead
                  of two and an NCCL MAX) or 'nccl' (the reference's MAX all-reduce
                  between the two passes).  Same codes either way.
  row_payload     'fp16' (the scaled-FP16 partials, default) or 'int8_gather' (the
                  reference's packed INT8 group-128 payload,
                  tilelang_transport_tradeoffs.py:40-88), with any row_transport
  quant_division  'rn' (IEEE, bit-exact with the CPU oracle) or 'fast' (__fdividef)
  mlp_pipeline_chunks  TPDiTMLPINT8 at TP > 1 on the peer transports: row chunks whose
                  partial-sum exchange overlaps the next chunks' GEMMs (1 = off, the
                  default; 0 = by size: 4 from 16384 rows, 2 from 4096).  Off by
                  default because it measured slower on B200: the persistent GEMM and
                  producer grids contend for the SMs (TP2, M = 32768: 1.63 ms a block
                  unpipelined, 1.77 ms at 2 chunks, 2.05 ms at 4)
  fc1_swiglu_epilogue  off (default): FC1 returns the reference's fp16 [S, 2*ffn/t]
                  [gate|up]; on: FC1 applies the FP32 SwiGLU in its GEMM epilogue and
                  returns fp32 [S, ffn/t] (same bytes, the same FC2 codes).  Turn it on
                  where FC1's output goes only to FC2 (TPDiTBlockINT8.forward,
                  tp_dit.py:356-360): FC2's producer then skips the SwiGLU
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from functools import lru_cache

import torch

ROW_BACKENDS = ("tilelang_packed", "tilelang_scaled_fp16", "native", "b200_scaled_fp16", "b200_int32")
FC2_QUANTIZERS = ("native", "owned_fp32", "fused_stored", "fused_recompute")
COLUMN_BACKENDS = ("preallocated", "cuda_int8_tilelang", "b200")


@dataclass(frozen=True)
class H3OperatorPolicy:
    row_linear_backend: str = "b200_scaled_fp16"
    fc2_quantizer: str = "fused_stored"
    column_linear_backend: str = "b200"
    dit_fused_gate: bool = True
    dit_fused_row_gate: bool = True
    dit_p0_2_lifetime: bool = True
    dit_p0_3_lifetime: bool = True
    dit_p0_b_inplace: bool = True
    dit_p0_a1_turing: bool = True
    dit_p0_c_local_rotation: bool = True
    row_transport: str = "p2p"
    row_payload: str = "fp16"
    fc2_max_exchange: str = "peer"
    quant_division: str = "rn"
    fc1_swiglu_epilogue: bool = False
    mlp_pipeline_chunks: int = 1

    def __post_init__(self):
        for name in ("dit_fused_gate", "dit_fused_row_gate", "dit_p0_2_lifetime",
                     "dit_p0_3_lifetime", "dit_p0_b_inplace", "dit_p0_a1_turing",
                     "dit_p0_c_local_rotation", "fc1_swiglu_epilogue"):
            if type(getattr(self, name)) is not bool:
                raise ValueError(name + " must be boolean")
        if self.row_linear_backend not in ROW_BACKENDS:
            raise ValueError("Unknown row-linear backend")
        if self.fc2_quantizer not in FC2_QUANTIZERS:
            raise ValueError("Unknown FC2 quantizer")
        if self.column_linear_backend not in COLUMN_BACKENDS:
            raise ValueError("Unknown column linear backend")
        if self.row_transport not in ("p2p", "nvls", "rowblock", "allreduce"):
            raise ValueError("Unknown row transport")
        if self.row_payload not in ("fp16", "int8_gather"):
            raise ValueError("Unknown row payload")
        if self.fc2_max_exchange not in ("peer", "nccl"):
            raise ValueError("Unknown FC2 maximum exchange")
        if self.quant_division not in ("rn", "fast"):
            raise ValueError("Unknown quantizer division")
        if type(self.mlp_pipeline_chunks) is not int or not 0 <= self.mlp_pipeline_chunks <= 64:
            raise ValueError("mlp_pipeline_chunks must be an int in [0, 64]")

    @property
    def scaled_transport(self) -> bool:
        return self.row_linear_backend in ("tilelang_scaled_fp16", "b200_scaled_fp16")


@lru_cache(maxsize=32)
def _fallback(name, device, capability):
    logging.warning("H3 %s: B200 path unavailable on %s (%s)", name, device, capability)


def configure_block(block, kind, policy):
    """Carries the policy onto a TP block's projections (h3_operator_policy.py:56-75)."""
    block.operator_policy = policy
    for name in (("o_proj", "down_proj") if kind == "te" else ("out_proj", "fc2")):
        if getattr(block, name, None) is not None:
            getattr(block, name).operator_policy = policy
    if kind == "dit":
        for name in ("qkv_proj", "fc1"):
            column = getattr(block, name, None)
            if column is not None:
                column.operator_policy = policy
                column._vram_p0_a1 = policy.dit_p0_a1_turing
        if getattr(block, "out_proj", None) is not None:
            block.out_proj._vram_p0_2 = policy.dit_p0_2_lifetime
            block.out_proj._vram_p0_c = policy.dit_p0_c_local_rotation
        if getattr(block, "fc2", None) is not None:
            block.fc2._vram_p0_3 = policy.dit_p0_3_lifetime
            block.fc2._vram_p0_b = policy.dit_p0_b_inplace
        if getattr(block, "fc1", None) is not None:
            block.fc1._vram_p0_3_producer = policy.dit_p0_3_lifetime
            block.fc1._swiglu_epilogue = policy.fc1_swiglu_epilogue
    return block


def row_linear(module, x, fallback, comm, input_act=None):
    """RowParallel dispatch (h3_operator_policy.py:213-237).  Returns FP32 [..., N]."""
    policy = getattr(module, "operator_policy", None) or H3OperatorPolicy()
    from . import swiglu_quant as quant
    division = policy.quant_division
    if (input_act == "swiglu" and policy.fc2_quantizer in ("fused_stored", "fused_recompute")
            and policy.row_linear_backend != "native"):
        if quant.supported(x, module.weight, module.weight_scale, module.world_size,
                           module.convrot_groupsize):
            return quant.row_linear(x, module.weight, module.weight_scale, comm,
                                    mode=policy.fc2_quantizer,
                                    scaled_transport=policy.scaled_transport,
                                    transport=policy.row_transport, division=division,
                                    payload=policy.row_payload,
                                    peer_max=policy.fc2_max_exchange == "peer")
        _fallback("FC2 fused quantizer", str(x.device), None)
    if (input_act is None and (x.shape[-1] * module.world_size) % 256 == 0
            and module.convrot_groupsize == 256):
        # O projection: local ConvRot of owned groups (or, for slices that split a group,
        # of the gathered rows), global row max, quantise.
        from .row_quant import global_row_quantize
        q, scale = global_row_quantize(x, comm, module.world_size, 256, None, division=division)
        out = quant._finish_quantized(q, scale, module.weight, module.weight_scale.reshape(-1),
                                      comm, policy.scaled_transport, policy.row_transport,
                                      payload=policy.row_payload)
        return out.reshape(*x.shape[:-1], module.weight.shape[0])
    args = (x, module.weight, module.weight_scale, comm, module.world_size,
            module.convrot_groupsize, input_act)
    return fallback(*args)


def row_linear_parts(module, gate, up, fallback, comm):
    """Separate gate/up inputs (h3_operator_policy.py:240-255): packed into the
    [gate | up] layout of the fused FC2 route."""
    if gate.shape != up.shape or gate.dtype != up.dtype or gate.device != up.device:
        raise ValueError("Matching gate/up required")
    return row_linear(module, torch.cat((gate, up), -1), fallback, comm, "swiglu")
