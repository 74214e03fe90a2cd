"""Kernel-level parity of libh3b200.so against the CPU oracle (bit-exact).

Each test drives one C-ABI entry point through h3tp.ops on seeded inputs and compares
every output bit with the oracle's restatement of the reference arithmetic:
  - INT8 codes, INT32 accumulators and row scales: exact equality;
  - fp16/fp32 epilogue outputs: exact equality too (the kernels follow the
    reference's rounding order operation by operation).
Shapes include ragged M/N tails, K at the 16-byte minimum and widths that are single
or many ConvRot groups.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


def _gateup(rng, rows, width, heavy=True):
    g = rng.standard_normal((rows, width)).astype(np.float32)
    u = rng.standard_normal((rows, width)).astype(np.float32)
    if heavy:
        g[::7] *= rng.standard_t(3, size=(len(g[::7]), width)).astype(np.float32)
        g[0, 0] = 1000.0  # reference outlier pattern (preview_fp32_swiglu_fusion.py:15)
        u[0, min(512, width - 1)] = 1000.0
    return np.concatenate([g, u], 1).astype(np.float16)


def _bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (a.shape, b.shape, a.dtype, b.dtype)
    va = a.view(np.uint8 if a.itemsize == 1 else {2: np.uint16, 4: np.uint32}[a.itemsize])
    vb = b.view(va.dtype)
    diff = va != vb
    if a.dtype.kind == "f":
        # NaN payloads are not part of the contract: the CPU oracle produces x86's
        # default NaN, the GPU its canonical one; a NaN must still meet a NaN.
        diff &= ~(np.isnan(a) & np.isnan(b))
    bad = np.flatnonzero(diff)
    assert bad.size == 0, f"{bad.size} of {a.size} differ; first at {np.unravel_index(bad[0], a.shape)}: {a.flat[bad[0]]} vs {b.flat[bad[0]]}"


# ----------------------------------------------------------------------------
# exponential
# ----------------------------------------------------------------------------
def test_expf_matches_oracle_on_all_fp16_inputs(cuda_device, oracle):
    from h3tp import ops
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    h = h[np.isfinite(h)]
    rng = np.random.default_rng(0)
    extra = np.concatenate([rng.uniform(-110, 95, 200000), rng.standard_normal(100000) * 4]).astype(np.float32)
    x = np.concatenate([-h, extra]).astype(np.float32)
    ours, cuda = ops.expf_compare(_t(x, cuda_device))
    _bits_equal(_np(ours), oracle.expf(x))


def test_expf_disagreement_with_cuda_expf_is_reported(cuda_device, oracle):
    """The path's exponential differs from CUDA's expf (which the reference calls) on
    a small fraction of inputs; measured here over every finite fp16 gate value."""
    from h3tp import ops
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    x = -h[np.isfinite(h)]
    ours, cuda = ops.expf_compare(_t(x, cuda_device))
    ours, cuda = _np(ours), _np(cuda)
    differ = np.count_nonzero(ours.view(np.uint32) != cuda.view(np.uint32))
    frac = differ / x.size
    print(f"h3_expf vs CUDA expf on {x.size} fp16 inputs: {differ} differ ({frac:.4%})")
    ulp = np.abs(ours.view(np.int32).astype(np.int64) - cuda.view(np.int32).astype(np.int64))
    fin = np.isfinite(ours) & np.isfinite(cuda) & (ours > 1e-37)
    assert ulp[fin].max() <= 4, "CUDA expf is documented within a few ulp"


def test_code_disagreement_vs_cuda_expf_swiglu(cuda_device, oracle):
    """Effect of the exponential on the INT8 codes: the reference's SwiGLU with CUDA
    expf, rotated and quantised by the oracle, against the path's codes."""
    from h3tp import ops
    rng = np.random.default_rng(31)
    x = _gateup(rng, 256, 4096)
    g = x[:, :4096].astype(np.float32)
    u = x[:, 4096:].astype(np.float32)
    _, _, silu_cuda = ops.silu_compare(_t(g.ravel(), cuda_device))
    act_cuda = (_np(silu_cuda).reshape(g.shape) * u).astype(np.float32)  # RN product, as the kernel
    R_c, m_c = oracle.fc2_rotate(act_cuda, "act_f32")
    q_c, _ = oracle.row_quantize(R_c, m_c)
    q, _, _ = ops.swiglu_rotate_quantize_local(_t(x, cuda_device), "gateup_f16")
    d = _np(q).astype(np.int32) - q_c.astype(np.int32)
    rate = np.count_nonzero(d) / d.size
    print(f"INT8 code disagreement vs CUDA-expf SwiGLU: {np.count_nonzero(d)} of {d.size} ({rate:.6%})")
    assert np.abs(d).max() <= 1 and rate < 1e-3


def test_silu_fast_path_is_bit_identical_on_all_fp16_gates(cuda_device, oracle):
    from h3tp import ops
    g = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    fast, ieee, _ = ops.silu_compare(_t(g, cuda_device))
    fast, ieee = _np(fast), _np(ieee)
    nan = np.isnan(g)
    assert np.isnan(fast[nan]).all() and np.isnan(ieee[nan]).all()
    _bits_equal(fast[~nan], ieee[~nan])
    fin = np.isfinite(g)
    ref = np.array([oracle.lib().h3o_swiglu(float(v), 1.0) for v in g[fin]], np.float32)
    _bits_equal(fast[fin], ref)


def test_quantizer_division_identity(cuda_device):
    """The kernels' code path (Markstein-corrected quotient from a per-row reciprocal,
    magic-number rounding) equals IEEE division + rintf + clamp on tens of millions of
    (x, scale) pairs, including exact half-way quotients and non-finite inputs."""
    from h3tp import ops
    g = torch.Generator(device=cuda_device).manual_seed(5)
    n = 1 << 24
    for trial in range(4):
        e = torch.rand(n, device=cuda_device, generator=g) * 200 - 100
        scale = torch.exp2(e).float()
        x = (torch.rand(n, device=cuda_device, generator=g) * 262 - 131) * scale
        fast, ieee = ops.quant_compare(x.float(), scale)
        assert torch.equal(fast, ieee), int((fast != ieee).sum())
    # exact ties (k + 1/2) * 2^e and their neighbours, scale a power of two
    k = torch.arange(-130, 131, device=cuda_device, dtype=torch.float32)
    es = torch.arange(-60, 61, device=cuda_device, dtype=torch.float32)
    scale = torch.exp2(es)[:, None].expand(-1, k.numel()).reshape(-1).contiguous()
    x = ((k + 0.5)[None, :] * torch.exp2(es)[:, None]).reshape(-1).contiguous()
    for xx in (x, torch.nextafter(x, torch.full_like(x, float("inf"))),
               torch.nextafter(x, torch.full_like(x, -float("inf")))):
        fast, ieee = ops.quant_compare(xx, scale)
        assert torch.equal(fast, ieee)
    special = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), float("nan"), 1e-45, -3e38, 3e38],
                           device=cuda_device)
    for s_ in (1e-30, 1.0, 3e38 / 127):
        fast, ieee = ops.quant_compare(special, torch.full_like(special, s_))
        assert torch.equal(fast, ieee), (s_, fast.tolist(), ieee.tolist())


# ----------------------------------------------------------------------------
# FC2 producer
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("rows,width", [(1, 256), (17, 512), (33, 1024), (5, 7168), (3, 8192), (2, 24576)])
@pytest.mark.parametrize("kind", ["gateup_f16", "act_f32", "act_f16"])
def test_fc2_producer_bit_exact(cuda_device, oracle, rows, width, kind):
    from h3tp import ops
    rng = np.random.default_rng(rows * 131 + width)
    if kind == "gateup_f16":
        x = _gateup(rng, rows, width)
    elif kind == "act_f32":
        x = (rng.standard_normal((rows, width)) * 0.7).astype(np.float32)
    else:
        x = (rng.standard_normal((rows, width)) * 0.7).astype(np.float16)
    R_ref, m_ref = oracle.fc2_rotate(x, kind)
    xd = _t(x, cuda_device)
    rot, m = ops.swiglu_rotate_max(xd, kind, store=True)
    _bits_equal(_np(rot), R_ref)
    _bits_equal(_np(m).ravel(), m_ref)
    rot2, m2 = ops.swiglu_rotate_max(xd, kind, store=False)
    assert rot2 is None
    _bits_equal(_np(m2).ravel(), m_ref)
    # global max across two emulated ranks: scale the maximum up for half the rows
    gmax = m_ref.copy()
    gmax[::2] *= 1.5
    q_ref, s_ref = oracle.row_quantize(R_ref, gmax)
    q, s = ops.swiglu_rotate_quantize(xd, _t(gmax, cuda_device), kind)
    _bits_equal(_np(q), q_ref)
    _bits_equal(_np(s).ravel(), s_ref)
    q3, s3 = ops.row_quantize(rot, _t(gmax, cuda_device))
    _bits_equal(_np(q3), q_ref)
    _bits_equal(_np(s3).ravel(), s_ref)
    ql_ref, sl_ref = oracle.row_quantize(R_ref, m_ref)
    ql, sl, ml = ops.swiglu_rotate_quantize_local(xd, kind)
    _bits_equal(_np(ql), ql_ref)
    _bits_equal(_np(sl).ravel(), sl_ref)
    _bits_equal(_np(ml).ravel(), m_ref)


def _special_rows(rng, rows, width, dtype):
    """Rows with a NaN, +inf, -inf, all zeros, signed zeros and tiny values, the largest
    finite value, and values on both sides of the packed paths' limits."""
    x = (rng.standard_normal((rows, width)) * 0.7).astype(np.float32)
    big = 65504.0 if dtype == np.float16 else 3e38
    tiny = 6e-8 if dtype == np.float16 else 1e-40
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    x[2, 9] = -np.inf
    x[3, :] = 0.0
    x[4, :] = tiny
    x[4, ::3] = -0.0
    x[5, 11] = big
    x[6, :16] = [100, -100, 89, -89, 88, -88, 88.0625, -88.0625, 17, -17, 1000, -1000,
                 65504, -65504, 0, -0.0]
    return x.astype(dtype)


@pytest.mark.parametrize("kind", ["gateup_f16", "act_f32", "act_f16"])
def test_fc2_producer_special_rows(cuda_device, oracle, kind):
    """NaN / infinity rows take the scalar quantiser, |gate| > 88 the scalar SiLU; all
    three producer forms stay bit-exact with the oracle."""
    from h3tp import ops
    rng = np.random.default_rng(23)
    rows, width = 8, 1024
    if kind == "gateup_f16":
        g = _special_rows(rng, rows, width, np.float16)
        u = (rng.standard_normal((rows, width)) * 0.7).astype(np.float16)
        x = np.concatenate([g, u], 1)
    else:
        x = _special_rows(rng, rows, width, np.float32 if kind == "act_f32" else np.float16)
    R_ref, m_ref = oracle.fc2_rotate(x, kind)
    xd = _t(x, cuda_device)
    rot, m = ops.swiglu_rotate_max(xd, kind, store=True)
    _bits_equal(_np(rot), R_ref)
    _bits_equal(_np(m).ravel(), m_ref)
    ql_ref, sl_ref = oracle.row_quantize(R_ref, m_ref)
    ql, sl, ml = ops.swiglu_rotate_quantize_local(xd, kind)
    _bits_equal(_np(ql), ql_ref)
    _bits_equal(_np(sl).ravel(), sl_ref)
    _bits_equal(_np(ml).ravel(), m_ref)
    q, s = ops.swiglu_rotate_quantize(xd, m, kind)
    _bits_equal(_np(q), ql_ref)
    _bits_equal(_np(s).ravel(), sl_ref)


@pytest.mark.parametrize("convrot", [True, False])
def test_column_quantize_special_rows(cuda_device, oracle, convrot):
    from h3tp import ops
    x = _special_rows(np.random.default_rng(29), 8, 3072, np.float16)
    q_ref, s_ref = oracle.column_quantize(x, convrot)
    q, s = ops.column_quantize(_t(x, cuda_device), convrot)
    _bits_equal(_np(q), q_ref)
    _bits_equal(_np(s).ravel(), s_ref)


# ----------------------------------------------------------------------------
# fused modulated RMSNorm -> ConvRot -> quant (the column input producer)
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("rows,width,convrot", [(37, 1024, True), (9, 3072, True),
                                                (5, 5376, True), (7, 1040, False)])
def test_modulated_norm_quantize_bit_exact(cuda_device, oracle, rows, width, convrot):
    from h3tp import ops
    rng = np.random.default_rng(rows + width)
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float16)
    x[0, : width // 3] = 0
    w = (rng.uniform(0.5, 1.5, width)).astype(np.float32)
    shift = (rng.standard_normal((3, width)) * .1).astype(np.float32)
    scale = (rng.standard_normal((3, width)) * .1).astype(np.float32)
    labels = rng.integers(0, 3, rows).astype(np.int32)
    h_ref = oracle.modulated_norm(x, w, 1e-6, shift, scale, labels)
    q_ref, s_ref = oracle.column_quantize(h_ref, convrot)
    q, s, h = ops.modulated_norm_quantize(_t(x, cuda_device), _t(w, cuda_device), 1e-6,
                                          _t(shift, cuda_device), _t(scale, cuda_device),
                                          _t(labels, cuda_device), convrot=convrot, want_h=True)
    _bits_equal(_np(h), h_ref)
    _bits_equal(_np(q), q_ref)
    _bits_equal(_np(s).ravel(), s_ref)
    _, _, h2 = ops.modulated_norm_quantize(_t(x, cuda_device), _t(w, cuda_device), 1e-6,
                                           _t(shift, cuda_device), _t(scale, cuda_device),
                                           _t(labels, cuda_device), quantize=False)
    _bits_equal(_np(h2), h_ref)


def test_modulated_norm_against_reference_golden(cuda_device):
    """The reference's own torch path (h3_tensor_flow.modulated_norm, tests/golden):
    within one fp16 ulp, nearly all bit for bit (different sum order, correctly
    rounded rsqrt)."""
    from h3tp import ops
    G = np.load(Path(__file__).parent / "golden" / "reference_golden.npz")
    _, _, h = ops.modulated_norm_quantize(
        _t(G["norm_x"], cuda_device), _t(G["norm_w"], cuda_device), float(G["norm_eps"][0]),
        _t(G["norm_shift"], cuda_device), _t(G["norm_scale"], cuda_device),
        _t(G["norm_labels"], cuda_device), quantize=False)
    d = np.abs(_np(h).view(np.int16).astype(np.int32) - G["norm_h"].view(np.int16).astype(np.int32))
    assert d.max() <= 1 and (d == 0).mean() >= 0.999


def test_row_quantize_owned_slice(cuda_device, oracle):
    from h3tp import ops
    rng = np.random.default_rng(5)
    X = rng.standard_normal((9, 1024)).astype(np.float32)
    m = np.abs(X).max(1).astype(np.float32) * 1.25
    q_ref, s_ref = oracle.row_quantize(X, m, start=256, width=512)
    q, s = ops.row_quantize(_t(X, cuda_device), _t(m, cuda_device), width=512, start=256)
    _bits_equal(_np(q), q_ref)
    _bits_equal(_np(s).ravel(), s_ref)


def test_fast_division_disagreement_is_small(cuda_device, oracle):
    """The reference's production quantizer divides with __fdividef; the path uses
    IEEE division (bit-exact with the oracle).  The fast variant must disagree on a
    tiny fraction of codes, by one step at most."""
    from h3tp import ops
    rng = np.random.default_rng(11)
    x = _gateup(rng, 64, 4096)
    xd = _t(x, cuda_device)
    q_rn, _, m = ops.swiglu_rotate_quantize_local(xd, "gateup_f16", "rn")
    q_fast, _ = ops.swiglu_rotate_quantize(xd, m, "gateup_f16", "fast")
    d = (_np(q_rn).astype(np.int32) - _np(q_fast).astype(np.int32))
    assert np.abs(d).max() <= 1
    assert np.count_nonzero(d) / d.size < 1e-3


# ----------------------------------------------------------------------------
# column activation quantizer
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("rows,k,convrot", [(1, 256, True), (19, 3072, True), (7, 5120, True),
                                            (4, 16384, True), (19, 3072, False), (3, 48, False)])
def test_column_quantize_bit_exact(cuda_device, oracle, rows, k, convrot):
    from h3tp import ops
    rng = np.random.default_rng(rows + k)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    cols = rng.permutation(k)[: max(1, k // 100)]
    x[:, cols] *= 20.0  # 1% outlier columns
    x = x.astype(np.float16)
    q_ref, s_ref = oracle.column_quantize(x, convrot)
    q, s = ops.column_quantize(_t(x, cuda_device), convrot)
    _bits_equal(_np(q), q_ref)
    _bits_equal(_np(s).ravel(), s_ref)


# ----------------------------------------------------------------------------
# tcgen05 INT8 GEMM + fused epilogues
# ----------------------------------------------------------------------------
GEMM_SHAPES = [(1, 256, 128), (17, 200, 16), (128, 256, 256), (300, 512, 3072),
               (129, 384, 1040), (256, 1024, 8192), (64, 3072, 1024)]


def _operands(rng, M, N, K):
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    return A, W


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_i32_exact(cuda_device, oracle, M, N, K):
    from h3tp import ops
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A, W = _operands(rng, M, N, K)
    C = ops.int8_gemm_i32(_t(A, cuda_device), _t(W, cuda_device))
    _bits_equal(_np(C), oracle.int8_gemm(A, W))


def test_gemm_i32_extremes(cuda_device, oracle):
    """Saturating operands: every product -128*-127 or 127*127 (largest sums)."""
    from h3tp import ops
    M, N, K = 130, 260, 8192
    A = np.full((M, K), -128, np.int8)
    A[1::2] = 127
    W = np.full((N, K), -127, np.int8)
    W[::3] = 127
    C = ops.int8_gemm_i32(_t(A, cuda_device), _t(W, cuda_device))
    _bits_equal(_np(C), oracle.int8_gemm(A, W))


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("bias", [False, True])
def test_gemm_column_bit_exact(cuda_device, oracle, M, N, K, bias):
    from h3tp import ops
    rng = np.random.default_rng(M + N + K + bias)
    A, W = _operands(rng, M, N, K)
    a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    w = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32) if bias else None
    y = ops.int8_gemm_column(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device),
                             _t(w, cuda_device), None if b is None else _t(b, cuda_device))
    _bits_equal(_np(y), oracle.column_epilogue(oracle.int8_gemm(A, W), a, w, b))


def test_gemm_column_scalar_weight_scale(cuda_device, oracle):
    from h3tp import ops
    rng = np.random.default_rng(3)
    A, W = _operands(rng, 40, 96, 64)
    a = rng.uniform(1e-3, 5e-2, 40).astype(np.float32)
    w = np.array([0.004], np.float32)
    y = ops.int8_gemm_column(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device), _t(w, cuda_device))
    _bits_equal(_np(y), oracle.column_epilogue(oracle.int8_gemm(A, W), a, w))


@pytest.mark.parametrize("M,Nh,K", [(1, 128, 128), (33, 96, 256), (300, 256, 3072), (129, 384, 1024),
                                    (260, 100, 512), (200, 98, 256)])
@pytest.mark.parametrize("out", ["f32", "f16"])
@pytest.mark.parametrize("bias", [False, True])
def test_gemm_swiglu_bit_exact(cuda_device, oracle, M, Nh, K, out, bias):
    """Ragged rows (M = 129, 200, 260, 300 on CTA pairs) and ragged columns (Nh = 100,
    98: a partial 8-column chunk, a width that is not a multiple of 4)."""
    from h3tp import ops
    rng = np.random.default_rng(M + Nh + K)
    A, W = _operands(rng, M, 2 * Nh, K)
    a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    w = rng.uniform(1e-3, 1e-2, 2 * Nh).astype(np.float32)
    b = (rng.standard_normal(2 * Nh) * 0.02).astype(np.float32) if bias else None
    y = ops.int8_gemm_swiglu(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device),
                             _t(w, cuda_device), None if b is None else _t(b, cuda_device),
                             torch.float32 if out == "f32" else torch.float16)
    _bits_equal(_np(y), oracle.swiglu_epilogue(oracle.int8_gemm(A, W), a, w, b, out))


@pytest.mark.parametrize("M,N,K", [(17, 256, 7168), (300, 512, 1024), (5, 200, 2048)])
def test_gemm_row_encode_bit_exact(cuda_device, oracle, M, N, K):
    from h3tp import ops
    rng = np.random.default_rng(M + N)
    A, W = _operands(rng, M, N, K)
    shift = oracle.transport_shift(2 * K)
    y = ops.int8_gemm_row_encode(_t(A, cuda_device), _t(W, cuda_device), shift)
    _bits_equal(_np(y), oracle.fp16_encode(oracle.int8_gemm(A, W), shift))


@pytest.mark.parametrize("out", ["f32", "f16", "residual", "residual_nogate"])
def test_gemm_row_dequant_bit_exact(cuda_device, oracle, out):
    from h3tp import ops
    M, N, K = 150, 384, 2048
    rng = np.random.default_rng(21)
    A, W = _operands(rng, M, N, K)
    a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    w = (rng.uniform(1e-3, 1e-2, N) / 512).astype(np.float32)
    C = oracle.int8_gemm(A, W)
    Ad, Wd, ad, wd = (_t(v, cuda_device) for v in (A, W, a, w))
    if out in ("f32", "f16"):
        y = ops.int8_gemm_row_dequant(Ad, Wd, ad, wd, torch.float32 if out == "f32" else torch.float16)
        _bits_equal(_np(y), oracle.dequantize_i32(C, a, w, out=out))
        return
    X = rng.standard_normal((M, N)).astype(np.float16)
    gate = labels = None
    if out == "residual":
        gate = rng.standard_normal((9, N)).astype(np.float32)
        labels = rng.integers(0, 9, M).astype(np.int32)
    Xd = _t(X, cuda_device)
    ops.int8_gemm_row_dequant(Ad, Wd, ad, wd, residual=Xd,
                              gate=None if gate is None else _t(gate, cuda_device),
                              labels=None if labels is None else _t(labels, cuda_device))
    ref = X.copy()
    oracle.dequantize_i32(C, a, w, out="residual", residual=ref, gate=gate, labels=labels)
    _bits_equal(_np(Xd), ref)


# ----------------------------------------------------------------------------
# persistent multi-tile GEMM: every CTA (pair) walks many tiles, so both TMEM
# accumulator buffers, their phase flips, the shared-memory ring wrapping across tiles
# and the grouped raster are exercised.  The pair kernel runs 74 clusters on 256 x 256
# tiles (256 x 128 output columns for SwiGLU); the single-CTA kernel 148 CTAs.
# ----------------------------------------------------------------------------
def _scales(rng, n, lo=1e-3, hi=1e-2):
    return rng.uniform(lo, hi, n).astype(np.float32)


def test_gemm_multitile_swiglu(cuda_device, oracle):
    """FC1 shape class: M = 4096, 2 x 8192 packed rows -> 16 x 64 = 1024 pair tiles."""
    from h3tp import ops
    rng = np.random.default_rng(401)
    M, Nh, K = 4096, 8192, 512
    A, W = _operands(rng, M, 2 * Nh, K)
    a, w = _scales(rng, M, 1e-3, 5e-2), _scales(rng, 2 * Nh)
    y = ops.int8_gemm_swiglu(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device),
                             _t(w, cuda_device), None, torch.float32)
    _bits_equal(_np(y), oracle.swiglu_epilogue(oracle.int8_gemm(A, W), a, w, None, "f32"))


def test_gemm_multitile_column_m_raster_groups(cuda_device, oracle):
    """A = 16384 x 3072 (50 MB) is larger than the 32 MB L2 slab, so the raster keeps
    groups of 42 M-blocks resident (two groups); 64 x 48 = 3072 pair tiles; bias on."""
    from h3tp import ops
    rng = np.random.default_rng(402)
    M, N, K = 16384, 12288, 3072
    A, W = _operands(rng, M, N, K)
    a, w = _scales(rng, M, 1e-3, 5e-2), _scales(rng, N)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    y = ops.int8_gemm_column(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device),
                             _t(w, cuda_device), _t(b, cuda_device))
    got = _np(y)
    del y
    _bits_equal(got, oracle.column_epilogue(oracle.int8_gemm(A, W), a, w, b))


def test_gemm_multitile_row_encode_n_raster_groups(cuda_device, oracle):
    """W = 16384 x 3072 is the larger operand: groups of 42 N-blocks (two groups) sweep
    all 48 M-blocks; 3072 pair tiles with the scaled-FP16 encode."""
    from h3tp import ops
    rng = np.random.default_rng(403)
    M, N, K = 12288, 16384, 3072
    A, W = _operands(rng, M, N, K)
    shift = oracle.transport_shift(2 * K)
    y = ops.int8_gemm_row_encode(_t(A, cuda_device), _t(W, cuda_device), shift)
    got = _np(y)
    del y
    _bits_equal(got, oracle.fp16_encode(oracle.int8_gemm(A, W), shift))


def test_gemm_multitile_row_dequant_residual(cuda_device, oracle):
    """FC2 shape class: M = 8192, N = 3072 -> 32 x 12 = 384 pair tiles, gated residual
    with per-row labels."""
    from h3tp import ops
    rng = np.random.default_rng(404)
    M, N, K = 8192, 3072, 1024
    A, W = _operands(rng, M, N, K)
    a, w = _scales(rng, M, 1e-3, 5e-2), (_scales(rng, N) / 512).astype(np.float32)
    X = rng.standard_normal((M, N)).astype(np.float16)
    gate = rng.standard_normal((9, N)).astype(np.float32)
    labels = rng.integers(0, 9, M).astype(np.int32)
    Xd = _t(X, cuda_device)
    ops.int8_gemm_row_dequant(_t(A, cuda_device), _t(W, cuda_device), _t(a, cuda_device),
                              _t(w, cuda_device), residual=Xd, gate=_t(gate, cuda_device),
                              labels=_t(labels, cuda_device))
    ref = X.copy()
    oracle.dequantize_i32(oracle.int8_gemm(A, W), a, w, out="residual", residual=ref,
                          gate=gate, labels=labels)
    _bits_equal(_np(Xd), ref)


def test_gemm_multitile_pack8(cuda_device, oracle):
    """Packed INT8 group-128 payload on 384 pair tiles."""
    from h3tp import ops
    rng = np.random.default_rng(405)
    M, N, K = 8192, 3072, 512
    A, W = _operands(rng, M, N, K)
    y = ops.int8_gemm_row_pack8(_t(A, cuda_device), _t(W, cuda_device))
    _bits_equal(_np(y), oracle.pack8(oracle.int8_gemm(A, W)))


def test_gemm_multitile_single_cta_kernel(cuda_device, oracle):
    """M <= 128 runs the single-CTA kernel: N = 80000 gives 313 tiles (a ragged last
    one) over 148 CTAs, so every CTA takes two or three tiles."""
    from h3tp import ops
    rng = np.random.default_rng(406)
    M, N, K = 100, 80000, 256
    A, W = _operands(rng, M, N, K)
    C = ops.int8_gemm_i32(_t(A, cuda_device), _t(W, cuda_device))
    _bits_equal(_np(C), oracle.int8_gemm(A, W))


# ----------------------------------------------------------------------------
# transport codec and reduction epilogue
# ----------------------------------------------------------------------------
# ----------------------------------------------------------------------------
# packed INT8 transport ('int8_gather')
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("world,rows,width", [(1, 5, 128), (2, 33, 384), (4, 17, 3072)])
def test_pack8_unpack8_bit_exact(cuda_device, oracle, world, rows, width):
    from h3tp import ops
    rng = np.random.default_rng(world * 7 + rows)
    parts = rng.integers(-2 ** 27, 2 ** 27, size=(world, rows, width)).astype(np.int32)
    parts[0, 0, :128] = 0                      # an all-zero group: the 1e-8 scale floor
    parts[-1, -1, 5] = 2 ** 31 - 1             # extremes
    parts[-1, -1, 6] = -2 ** 31
    packed = np.stack([oracle.pack8(p) for p in parts])
    got = torch.stack([ops.pack8(_t(p, cuda_device)) for p in parts])
    _bits_equal(_np(got), packed)
    restored = oracle.unpack8_restore(packed, width)
    _bits_equal(_np(ops.unpack8_finish(got, width, out_dtype=torch.int32)), restored)
    a = rng.uniform(1e-6, 1e-4, rows).astype(np.float32)
    w = rng.uniform(1e-4, 1e-3, width).astype(np.float32)
    for out, dt in (("f32", torch.float32), ("f16", torch.float16)):
        y = ops.unpack8_finish(got, width, _t(a, cuda_device), _t(w, cuda_device), dt)
        _bits_equal(_np(y), oracle.dequantize_i32(restored, a, w, out=out))
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((3, width)).astype(np.float32)
    lab = rng.integers(0, 3, rows).astype(np.int32)
    ref = X.copy()
    oracle.dequantize_i32(restored, a, w, out="residual", residual=ref, gate=G, labels=lab)
    Xd = _t(X, cuda_device)
    ops.unpack8_finish(got, width, _t(a, cuda_device), _t(w, cuda_device), residual=Xd,
                       gate=_t(G, cuda_device), labels=_t(lab, cuda_device))
    _bits_equal(_np(Xd), ref)


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (77, 384, 1024), (300, 3072, 2048)])
def test_gemm_row_pack8_bit_exact(cuda_device, oracle, M, N, K):
    from h3tp import ops
    rng = np.random.default_rng(M + N)
    A, W = _operands(rng, M, N, K)
    got = ops.int8_gemm_row_pack8(_t(A, cuda_device), _t(W, cuda_device))
    _bits_equal(_np(got), oracle.pack8(oracle.int8_gemm(A, W)))


@pytest.mark.parametrize("pattern", ["random", "zero", "bounds", "cancellation", "ties_outliers"])
def test_packed_known_answers_on_gpu(cuda_device, pattern):
    """The reference's 'int8_gather' known-answer patterns (test_tp2_p2_epilogue.py:15-38,
    outputs of its own transport_reference stored in tests/golden) through the GPU pack,
    reconstruction and FP32 dequant."""
    from h3tp import ops
    G = np.load(Path(__file__).parent / "golden" / "reference_golden.npz")
    parts = G[f"kat_{pattern}_parts"]
    a, w = G[f"kat_{pattern}_a"], G[f"kat_{pattern}_w"]
    packed = torch.stack([ops.pack8(_t(p, cuda_device)) for p in parts])
    width = parts.shape[2]
    _bits_equal(_np(ops.unpack8_finish(packed, width, out_dtype=torch.int32)),
                G[f"kat_{pattern}_int8_restored"])
    y = ops.unpack8_finish(packed, width, _t(a, cuda_device), _t(w, cuda_device))
    _bits_equal(_np(y), G[f"kat_{pattern}_int8_expected"])


def test_fp16_codec_bit_exact(cuda_device, oracle):
    from h3tp import ops
    rng = np.random.default_rng(744)
    P = rng.integers(-10_000_000, 10_000_000, size=(17, 256), dtype=np.int32)
    P[0, :8] = [16777217, -8388609, 1, -1, 65535, -65535, 127, 0]
    for shift in (0, 10, 11, 12):
        y = ops.fp16_encode(_t(P, cuda_device), shift)
        _bits_equal(_np(y), oracle.fp16_encode(P, shift))
        back = ops.fp16_decode(y, shift)
        _bits_equal(_np(back), oracle.fp16_decode(_np(y), shift))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("out", ["f32", "f16", "residual"])
def test_row_reduce_finish_bit_exact(cuda_device, oracle, world, out):
    from h3tp import ops
    rng = np.random.default_rng(world * 10 + len(out))
    rows, width = 37, 264
    shift = oracle.transport_shift(world * 1024)
    parts = rng.standard_normal((world, rows, width)).astype(np.float16) * np.float16(100)
    a = rng.uniform(1e-3, 5e-2, rows).astype(np.float32)
    w = rng.uniform(1e-6, 1e-5, width).astype(np.float32)
    pd = _t(parts, cuda_device)
    if out != "residual":
        y = ops.row_reduce_finish(pd, shift, _t(a, cuda_device), _t(w, cuda_device),
                                  torch.float32 if out == "f32" else torch.float16)
        _bits_equal(_np(y), oracle.row_reduce_finish(parts, shift, a, w, out=out))
        return
    X = rng.standard_normal((rows, width)).astype(np.float16)
    gate = rng.standard_normal((3, width)).astype(np.float32)
    labels = (np.arange(rows) % 3).astype(np.int32)
    Xd = _t(X, cuda_device)
    ops.row_reduce_finish(pd, shift, _t(a, cuda_device), _t(w, cuda_device), residual=Xd,
                          gate=_t(gate, cuda_device), labels=_t(labels, cuda_device))
    ref = X.copy()
    oracle.row_reduce_finish(parts, shift, a, w, out="residual", residual=ref, gate=gate, labels=labels)
    _bits_equal(_np(Xd), ref)


def test_column_and_int32_dequantize(cuda_device, oracle):
    from h3tp import ops
    rng = np.random.default_rng(9)
    C = rng.integers(-2**26, 2**26, size=(23, 129), dtype=np.int32)
    a = rng.uniform(1e-3, 5e-2, 23).astype(np.float32)
    w = rng.uniform(1e-3, 1e-2, 129).astype(np.float32)
    b = rng.standard_normal(129).astype(np.float32)
    Cd, ad, wd, bd = (_t(v, cuda_device) for v in (C, a, w, b))
    _bits_equal(_np(ops.column_dequantize(Cd, ad, wd)), oracle.column_epilogue(C, a, w))
    _bits_equal(_np(ops.dequantize_i32(Cd, ad, wd, torch.float32, bd)),
                oracle.dequantize_i32(C, a, w, bias=b, out="f32"))
    _bits_equal(_np(ops.dequantize_i32(Cd, ad, wd, torch.float16)),
                oracle.dequantize_i32(C, a, w, out="f16"))


def test_sm_clock_probe(cuda_device):
    """h3_sm_clock_probe: it sleeps at least the requested time and reports the SM
    cycles of that interval; the clock they give lies in the part's range."""
    from h3tp import ops
    out = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    ops.sm_clock_probe(out, 2_000_000, torch.cuda.current_stream(cuda_device))
    torch.cuda.synchronize()
    ns, cycles = out.tolist()
    assert 2_000_000 <= ns < 200_000_000
    assert 200.0 < cycles / ns * 1e3 < 2500.0
    with pytest.raises(ValueError):
        ops.sm_clock_probe(out, 0, torch.cuda.current_stream(cuda_device))


def test_no_device_error_after_suite(cuda_device):
    from h3tp import _native
    torch.cuda.synchronize()
    assert _native.device_error(0) == 0
