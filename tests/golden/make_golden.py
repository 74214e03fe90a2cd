"""Generates the golden vectors in tests/golden/ by running the reference's own code.

    python tests/golden/make_golden.py <minimax-h3-2xt4 checkout>

Only the reference's CPU-capable Python runs here (its TileLang kernels need an
sm_75/sm_120 GPU and its comfy_kitchen dependency is not installed): a stub
`comfy_kitchen` module is put in sys.modules so that the imports succeed, and only
functions whose CPU path never touches it are called:

  patches/parallel_int8.py         int_mm (torch._int_mm, CPU), dequantize (CPU
                                   branch, :66-69), packed_rows (:97-103)
  patches/tilelang_transport_tradeoffs.py  shift_for (:20-22)
  benchmarks/tp2_tradeoffs.py      transport_reference (:66-78), extracted from the
                                   module source because the module's own imports
                                   name retired files
  benchmarks/test_tp2_p2_epilogue.py  its five known-answer patterns (:15-38), built
                                   here on the CPU with the same seed and sizes, for
                                   both of its schemes ('fp16' and 'int8_gather')
  patches/h3_tensor_flow.py        fold_linear (:82-103), modulated_norm's torch
                                   path (:134-143)
  patches/tilelang_dit_fusion.py   segment_key (:93-100)

The reference is not needed at test time: the outputs are stored as .npz files next
to this script and the tests read those.
"""
from __future__ import annotations

import ast
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load_reference(root: Path):
    sys.path.insert(0, str(root))
    sys.modules.setdefault("comfy_kitchen", types.ModuleType("comfy_kitchen"))
    from patches import parallel_int8 as pi
    from patches import tilelang_transport_tradeoffs as transport
    from patches import h3_tensor_flow as flow
    from patches import tilelang_dit_fusion as fusion
    src = (root / "benchmarks" / "tp2_tradeoffs.py").read_text()
    fn = next(n for n in ast.parse(src).body
              if isinstance(n, ast.FunctionDef) and n.name == "transport_reference")
    ns = {"torch": torch, "transport": transport}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "tp2_tradeoffs.py", "exec"), ns)
    return pi, transport, flow, fusion, ns["transport_reference"]


def make(root: Path) -> None:
    pi, transport, flow, fusion, transport_reference = _load_reference(root)
    out = {}

    # --- shift_for on the TP2 local widths of the DiT and of the configs ----------------
    ks = np.array([256, 1024, 1536, 3584, 4096, 6400, 7168, 8192, 12800, 16384], np.int64)
    out["shift_local_k"] = ks
    out["shift_for"] = np.array([transport.shift_for(int(k)) for k in ks], np.int64)

    # --- int_mm: exact INT32 (rows padded to 32 inside) --------------------------------
    g = torch.Generator().manual_seed(11)
    q = torch.randint(-128, 128, (37, 512), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (96, 512), generator=g, dtype=torch.int8)
    out["int_mm_q"], out["int_mm_w"] = q.numpy(), w.numpy()
    out["int_mm_out"] = pi.int_mm(q, w).numpy()

    # --- dequantize CPU branch: ((acc * a) * w) [+ bias] -> dtype -----------------------
    acc = torch.randint(-2 ** 26, 2 ** 26, (23, 129), generator=g, dtype=torch.int32)
    a = (torch.rand((23, 1), generator=g) * 0.05).float()
    ws = (torch.rand((129, 1), generator=g) * 0.01).float()
    bias = torch.randn((129,), generator=g).float()
    out["deq_acc"], out["deq_a"], out["deq_w"], out["deq_bias"] = (
        acc.numpy(), a.numpy(), ws.numpy(), bias.numpy())
    out["deq_f32"] = pi.dequantize(acc, a, ws, torch.float32).numpy()
    out["deq_f16"] = pi.dequantize(acc, a, ws, torch.float16).numpy()
    out["deq_f32_bias"] = pi.dequantize(acc, a, ws, torch.float32, bias).numpy()

    # --- packed_rows: component-packed column shards -----------------------------------
    wfull = torch.arange(3 * 8 * 4, dtype=torch.int32).reshape(24, 4).to(torch.int8)
    sfull = torch.arange(24, dtype=torch.float32).reshape(24, 1)
    out["packed_w"], out["packed_s"] = wfull.numpy(), sfull.numpy()
    for world in (1, 2, 4):
        for rank in range(world):
            wr, sr = pi.packed_rows(wfull, sfull, rank, world, 3)
            out[f"packed_w_t{world}_r{rank}"] = wr.numpy()
            out[f"packed_s_t{world}_r{rank}"] = sr.numpy()

    # --- scaled-FP16 transport known-answer patterns (test_tp2_p2_epilogue.py:15-38) ----
    rows, width, k = 17, 256, 7168
    torch.manual_seed(744)
    for pattern in ("random", "zero", "bounds", "cancellation", "ties_outliers"):
        parts = torch.randint(-10000000, 10000000, (2, rows, width), dtype=torch.int32)
        if pattern == "zero":
            parts.zero_()
        if pattern == "bounds":
            parts.fill_(k * 128 * 128)
        if pattern == "cancellation":
            parts[1] = -parts[0] + 17
        if pattern == "ties_outliers":
            parts.zero_()
            parts[0, :, 0] = 16777217
            parts[1, :, 1] = -8388609
            parts[:, :, 2:10] = torch.tensor([1, -1, 3, -3, 127, -127, 65535, -65535], dtype=torch.int32)
        a = torch.rand(rows, 1) * .1
        wv = torch.rand(width) * .001
        independent = transport_reference(parts, "fp16", k)
        expected = (independent.float() * a) * wv
        native = pi.dequantize(independent, a, wv, torch.float32)
        assert torch.equal(native, expected)
        out[f"kat_{pattern}_parts"] = parts.numpy()
        out[f"kat_{pattern}_a"] = a.numpy()
        out[f"kat_{pattern}_w"] = wv.numpy()
        out[f"kat_{pattern}_reduced_i32"] = independent.numpy()
        out[f"kat_{pattern}_expected"] = expected.numpy()
        # the packed INT8 scheme of the same test (test_tp2_p2_epilogue.py:27-35)
        restored8 = transport_reference(parts, "int8_gather", k)
        out[f"kat_{pattern}_int8_restored"] = restored8.numpy()
        out[f"kat_{pattern}_int8_expected"] = ((restored8.float() * a) * wv).numpy()
    out["kat_k"] = np.array([k], np.int64)

    # --- row-order contract (test_fp16_fc2_experiment.py:10-30) -------------------------
    qc = torch.tensor([[1, -2, 3, 4]], dtype=torch.int8)
    wc = torch.tensor([[2, 3, -1, 4]], dtype=torch.int8)
    scale = torch.tensor([[.25]], dtype=torch.float32)
    wsc = torch.tensor([[.125]], dtype=torch.float32)
    out["order_expected"] = (((qc.int() @ wc.int().t()) * 2).float() * scale * wsc + 1.).half().numpy()

    # --- residual scale fold (h3_tensor_flow.py:82-91) ----------------------------------
    m = types.SimpleNamespace(weight=torch.zeros(4, 4, dtype=torch.int8),
                              weight_scale=torch.nn.Parameter(torch.tensor([[.3], [1e-3], [7.], [2.5e-5]]),
                                                              requires_grad=False), bias=None)
    before = m.weight_scale.detach().clone()
    flow.fold_linear(m, flow.TensorFlowPolicy().divisor)
    out["fold_before"], out["fold_after"] = before.numpy(), m.weight_scale.detach().numpy()
    out["fold_divisor"] = np.array([flow.TensorFlowPolicy().divisor], np.float64)

    # --- modulated RMSNorm, the reference's torch path (h3_tensor_flow.py:134-143) -------
    gn = torch.Generator().manual_seed(21)
    rows_n, width_n = 37, 1024
    xn = (torch.randn((rows_n, width_n), generator=gn) * 3).half()
    xn[5, :64] = 0  # a partly zero row
    norm = types.SimpleNamespace(normalized_shape=(width_n,),
                                 weight=(torch.rand(width_n, generator=gn) + .5).float(),
                                 eps=1e-6)
    shift_n = (torch.randn((3, width_n), generator=gn) * .1).float()
    scale_n = (torch.randn((3, width_n), generator=gn) * .1).float()
    segs = [(0, 10, 0), (10, 30, 2), (30, rows_n, 1)]
    out["norm_x"], out["norm_w"] = xn.numpy(), norm.weight.numpy()
    out["norm_shift"], out["norm_scale"] = shift_n.numpy(), scale_n.numpy()
    out["norm_eps"] = np.array([norm.eps], np.float64)
    out["norm_labels"] = np.concatenate([np.full(b - a, r, np.int32) for a, b, r in segs])
    out["norm_h"] = flow.modulated_norm(norm, xn, shift_n, scale_n, segs, fused=False).numpy()

    # --- segment validation (tilelang_dit_fusion.py:93-100) -----------------------------
    cases = [(10, [(0, 4, 1), (4, 10, 2)]), (10, [(0, 4, 1), (5, 10, 2)]),
             (10, [(0, 10, 9)]), (10, [(0, 10, 8)]), (6, [(3, 6, 0), (0, 3, 1)])]
    out["segment_ok"] = np.array([fusion.segment_key(r, s) is not None for r, s in cases])

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print("wrote", HERE / "reference_golden.npz", len(out), "arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout>")
    make(Path(sys.argv[1]))
