"""h3tp - B200-native (sm_100a) tensor-parallel W8A8 INT8 linear path.

Drop-in for the operator API of chinokikiss/minimax-h3-2xt4 `patches/` on this path:
ColumnParallelLinearINT8 / RowParallelLinearINT8 (tp_dit), column_linear
(dit_column_linear), the FC2 `fused_stored` row chain (swiglu_quant), the row
quantizer (row_quant), the scaled-FP16 transport (transport), the fused row-gate
epilogue (dit_fusion), the operator policy and the residual scale fold.

All arithmetic runs in libh3b200.so (hand-written sm_100a CUDA); this package only
validates, allocates and orchestrates (torch tensors, streams, torch.distributed).
"""
__version__ = "0.1.0"
