"""Self-checks of the CPU oracle that do not need the reference run: the butterfly
restatement against the matrix definition of ConvRot256, IEEE fp16 conversion against
numpy, the exponential's accuracy, and the quantizer's defining property
(benchmarks/preview_fp32_swiglu_fusion.py:24-26: codes == round(rot/scale).clamp)."""
import numpy as np
import pytest


def _h256():
    # H256 = (H4 (x) H4 (x) H4 (x) H4) / 16, H4[d][k] = -1 iff d + k == 3
    # (tilelang_swiglu_quant.py:19-36; the regular, not Sylvester, Hadamard)
    h4 = np.ones((4, 4))
    for d in range(4):
        h4[d, 3 - d] = -1
    h = h4
    for _ in range(3):
        h = np.kron(h, h4)
    return h / 16.0


def test_butterfly_equals_regular_hadamard_matrix(oracle):
    H = _h256()
    assert np.allclose(H @ H.T, np.eye(256))  # orthonormal
    rng = np.random.default_rng(0)
    for _ in range(20):
        v = rng.standard_normal(256).astype(np.float32) * rng.uniform(0.01, 100)
        got = oracle.convrot256(v).astype(np.float64)
        # the butterfly index i = 64*d3 + 16*d2 + 4*d1 + d0 transforms digit 0 first;
        # in Kronecker order digit 0 is the last factor, so H acts on v directly.
        ref = H @ v.astype(np.float64)
        assert np.allclose(got, ref, rtol=1e-5, atol=1e-5 * np.abs(v).max())


def test_fp16_conversions_match_numpy(oracle):
    L = oracle.lib()
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = h.view(np.float16).astype(np.float32)
    fin = np.isfinite(f)
    mine = np.array([L.h3o_half_to_float(int(v)) for v in h[fin]], np.float32)
    assert np.array_equal(mine.view(np.uint32), f[fin].view(np.uint32))
    rng = np.random.default_rng(1)
    mids = (f[fin][:-1].astype(np.float64) + f[fin][1:].astype(np.float64)) / 2
    vals = np.concatenate([mids.astype(np.float32), rng.standard_normal(50000).astype(np.float32) * 3000,
                           np.array([65519.99, 65520, 65504, -65520, 5.96e-8, 2.98e-8, 2.9802322e-08], np.float32)])
    vals = vals[np.isfinite(vals)]
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    mine = np.array([L.h3o_float_to_half(float(v)) for v in vals], np.uint16)
    assert np.array_equal(mine, ref)


def test_exponential_accuracy(oracle):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    x = -h[np.isfinite(h)]
    e = oracle.expf(x)
    with np.errstate(over="ignore"):
        ex = np.exp(x.astype(np.float64))
        fe = ex.astype(np.float32)
    ok = np.isfinite(fe) & (fe > 1.2e-38)
    ulp = np.abs(e[ok].astype(np.float64) - ex[ok]) / np.spacing(fe[ok]).astype(np.float64)
    assert ulp.max() < 0.65
    assert (e[ok] == fe[ok]).mean() > 0.99
    assert np.all(e[~ok & (x > 0)] == np.inf) and np.all(e[~ok & (x < 0)] <= 1.2e-38)


@pytest.mark.parametrize("kind", ["gateup_f16", "act_f32", "act_f16"])
def test_codes_are_rounded_scaled_rotation(oracle, kind):
    """INT8 codes equal clamp(round_half_even(rotated / scale), -128, 127) of the
    oracle's own rotation, and scale = max(max|rot| * f32(1/127), 1e-30)."""
    rng = np.random.default_rng(2)
    w = 1024
    if kind == "gateup_f16":
        x = (rng.standard_normal((9, 2 * w)) * 4).astype(np.float16)
        x[0, 0] = 1000
        x[0, 512] = 1000
    elif kind == "act_f32":
        x = rng.standard_normal((9, w)).astype(np.float32)
    else:
        x = rng.standard_normal((9, w)).astype(np.float16)
    R, m = oracle.fc2_rotate(x, kind)
    assert np.array_equal(m, np.abs(R).max(1))
    q, s = oracle.row_quantize(R, m)
    scale = np.maximum(m * np.float32(1 / 127), np.float32(1e-30)).astype(np.float32)
    assert np.array_equal(s, scale)
    ref = np.clip(np.rint(R / scale[:, None]), -128, 127).astype(np.int8)
    assert np.array_equal(q, ref)


def test_column_quantize_without_rotation_is_absmax_127(oracle):
    """BASELINE config 1 quantiser: per-row absmax/127, round half to even, and the
    clamp never reaches -128 because |x| <= absmax."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 3072)).astype(np.float16)
    q, s = oracle.column_quantize(x, False)
    assert q.min() >= -127
    xf = x.astype(np.float32)
    scale = (np.abs(xf).max(1) * np.float32(1 / 127)).astype(np.float32)
    assert np.array_equal(s, scale)
    assert np.array_equal(q, np.clip(np.rint(xf / scale[:, None]), -128, 127).astype(np.int8))


def test_transport_shift_bound(oracle):
    """The shift keeps every rank's encoded partial and their sum finite in fp16."""
    for k in (1024, 3072, 8192, 16384):
        s = oracle.transport_shift(k)
        assert k * 127 * 128 / 2 ** s < 65504
        assert s == 0 or k * 127 * 127 / 2 ** (s - 1) > 60000
