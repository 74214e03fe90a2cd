"""The CPU oracle (and the host-side layout helpers) against golden vectors produced by
running the reference's own code (tests/golden/make_golden.py): shift_for, int_mm,
the CPU dequantize branch, packed_rows, the scaled-FP16 transport known-answer
patterns of benchmarks/test_tp2_p2_epilogue.py, the FC2 row-order contract, the
residual scale fold and segment validation.  No GPU needed."""
from pathlib import Path

import numpy as np
import pytest
import torch

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_golden.npz")


def _eq(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert a.dtype == b.dtype, (a.dtype, b.dtype)
    v = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[a.itemsize]
    assert np.array_equal(a.view(v), b.view(v))


def test_transport_shift_matches_shift_for(oracle):
    # shift_for(local_k) at TP2 == the generalised shift on the full length 2*local_k
    for k, s in zip(G["shift_local_k"], G["shift_for"]):
        assert oracle.transport_shift(2 * int(k)) == int(s)


def test_int_mm_exact(oracle):
    _eq(oracle.int8_gemm(G["int_mm_q"], G["int_mm_w"]), G["int_mm_out"])
    _eq(oracle.int8_gemm_loop(G["int_mm_q"], G["int_mm_w"]), G["int_mm_out"])


def test_int8_gemm_routes_agree(oracle):
    """The C loop and the CPU int_mm route of the oracle's GEMM give the same INT32 bits,
    saturating operands included."""
    rng = np.random.default_rng(11)
    A = rng.integers(-128, 128, size=(300, 2048), dtype=np.int8)
    W = rng.integers(-127, 128, size=(96, 2048), dtype=np.int8)
    A[:4] = -128
    W[:3] = -127
    big = oracle.int8_gemm(A, W)  # above the size at which the int_mm route takes over
    _eq(big, oracle.int8_gemm_loop(A, W))


def test_dequantize_cpu_branch(oracle):
    acc, a, w, b = G["deq_acc"], G["deq_a"], G["deq_w"], G["deq_bias"]
    _eq(oracle.dequantize_i32(acc, a, w, out="f32"), G["deq_f32"])
    _eq(oracle.dequantize_i32(acc, a, w, out="f16"), G["deq_f16"])
    _eq(oracle.dequantize_i32(acc, a, w, bias=b, out="f32"), G["deq_f32_bias"])


@pytest.mark.parametrize("world", [1, 2, 4])
def test_packed_rows_layout(oracle, world):
    from h3tp.parallel_int8 import packed_rows
    w, s = G["packed_w"], G["packed_s"]
    for rank in range(world):
        wr, sr = oracle.packed_rows(w, s, rank, world, 3)
        _eq(wr, G[f"packed_w_t{world}_r{rank}"])
        _eq(sr, G[f"packed_s_t{world}_r{rank}"])
        wt, st = packed_rows(torch.from_numpy(w), torch.from_numpy(s), rank, world, 3)
        _eq(wt.numpy(), G[f"packed_w_t{world}_r{rank}"])
        _eq(st.numpy(), G[f"packed_s_t{world}_r{rank}"])


@pytest.mark.parametrize("pattern", ["random", "zero", "bounds", "cancellation", "ties_outliers"])
def test_scaled_fp16_transport_known_answers(oracle, pattern):
    """encode -> fp16 SUM (one RN addition at TP2) -> decode -> FP32 dequant, bitwise
    equal to the reference's independent transport_reference + eager dequant."""
    parts = G[f"kat_{pattern}_parts"]
    a, w = G[f"kat_{pattern}_a"], G[f"kat_{pattern}_w"]
    k = int(G["kat_k"][0])
    shift = oracle.transport_shift(2 * k)
    enc = np.stack([oracle.fp16_encode(p, shift) for p in parts])
    # the reduced INT32 the epilogue restores
    summed = (enc[0].astype(np.float32) + enc[1].astype(np.float32)).astype(np.float16)
    _eq(oracle.fp16_decode(summed, shift), G[f"kat_{pattern}_reduced_i32"])
    # the fused epilogue on the two partials
    _eq(oracle.row_reduce_finish(enc, shift, a, w, out="f32"), G[f"kat_{pattern}_expected"])


@pytest.mark.parametrize("pattern", ["random", "zero", "bounds", "cancellation", "ties_outliers"])
def test_packed_int8_transport_known_answers(oracle, pattern):
    """The 'int8_gather' scheme of the same test (test_tp2_p2_epilogue.py:27-35): per-rank
    group-128 pack, rank-order reconstruction, FP32 dequant, bitwise equal to the
    reference's transport_reference(parts, 'int8_gather') + eager dequant."""
    parts = G[f"kat_{pattern}_parts"]
    a, w = G[f"kat_{pattern}_a"], G[f"kat_{pattern}_w"]
    packed = np.stack([oracle.pack8(p) for p in parts])
    restored = oracle.unpack8_restore(packed, parts.shape[2])
    _eq(restored, G[f"kat_{pattern}_int8_restored"])
    _eq(oracle.dequantize_i32(restored, a, w, out="f32"), G[f"kat_{pattern}_int8_expected"])


def test_modulated_norm_vs_reference_torch_path(oracle):
    """The fused column producer's modulated RMSNorm against the reference's own torch
    path (h3_tensor_flow.modulated_norm, F.rms_norm + segment modulation): the same
    operations in a different summation order and with a correctly rounded rsqrt, so
    the fp16 outputs agree to within one ulp, nearly all bit for bit."""
    h = oracle.modulated_norm(G["norm_x"], G["norm_w"], G["norm_eps"][0], G["norm_shift"],
                              G["norm_scale"], G["norm_labels"])
    ref = G["norm_h"]
    assert np.array_equal(np.sign(h.astype(np.float32)), np.sign(ref.astype(np.float32)))
    d = np.abs(h.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    assert d.max() <= 1
    assert (d == 0).mean() >= 0.999


def test_oracle_rsqrt_is_correctly_rounded(oracle):
    from decimal import Decimal, getcontext
    getcontext().prec = 60
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.uniform(1e-6, 1e4, 500).astype(np.float32),
                           np.float32([1, 2, 4, 0.25, 3, 1e-38, 3e38, 1.5e-45])])
    for v in vals:
        y = np.float32(oracle.rsqrt_rn(float(v)))
        t = 1 / Decimal(float(v)).sqrt()
        best = min((np.nextafter(y, np.float32(0)), y, np.nextafter(y, np.float32(np.inf))),
                   key=lambda c: abs(Decimal(float(c)) - t))
        assert best == y, v


def test_row_order_contract(oracle):
    """INT32 partial SUM, then f32 * scale * ws, then FP32 LoRA, then one fp16 store
    (benchmarks/test_fp16_fc2_experiment.py:10-30)."""
    q = np.array([[1, -2, 3, 4]], np.int8)
    w = np.array([[2, 3, -1, 4]], np.int8)
    partial = oracle.int8_gemm(q, w) * 2  # two ranks with identical partials
    y = oracle.dequantize_i32(partial, np.array([.25], np.float32), np.array([.125], np.float32))
    _eq((y + np.float32(1.0)).astype(np.float16), G["order_expected"])


def test_residual_scale_fold():
    from h3tp.h3_tensor_flow import TensorFlowPolicy, fold_linear
    m = torch.nn.Module()
    m.weight = torch.nn.Parameter(torch.zeros(4, 4, dtype=torch.int8), requires_grad=False)
    m.weight_scale = torch.nn.Parameter(torch.from_numpy(G["fold_before"].copy()), requires_grad=False)
    m.bias = None
    assert TensorFlowPolicy().divisor == float(G["fold_divisor"][0])
    fold_linear(m, TensorFlowPolicy().divisor)
    _eq(m.weight_scale.detach().numpy(), G["fold_after"])


def test_segment_validation():
    from h3tp.dit_fusion import segment_key
    cases = [(10, [(0, 4, 1), (4, 10, 2)]), (10, [(0, 4, 1), (5, 10, 2)]),
             (10, [(0, 10, 9)]), (10, [(0, 10, 8)]), (6, [(3, 6, 0), (0, 3, 1)])]
    got = np.array([segment_key(r, s) is not None for r, s in cases])
    assert np.array_equal(got, G["segment_ok"])
