"""The reference's own TileLang kernels, run on the B200 next to this library and the C
oracle: pins the oracle (and the B200 path) to the reference's arithmetic where the
reference itself can run.

oracle/tilelang_ref.py lowers the reference's kernel factories (unchanged, from the
reference checkout) to CUDA C++ and builds them for sm_100a into oracle/_ref/; this
file only loads that build (it is test infrastructure, never used by the product).
Kernels and what is pinned:
  fused_kernel 'stored' / 'maximum' (tilelang_swiglu_quant.py:12-51): rotated values
      and group maxima bit for bit on gates where exp cannot matter (gate >= 17, where
      1 + exp(-gate) rounds to 1, gate <= -89, where exp(-gate) overflows, and 0);
      on ordinary gates the reference calls CUDA expf and this path its own
      exponential, so the rotated values agree to a few ulps and the codes are
      counted, not required, to agree;
  fused_kernel 'recompute' (:52-64, '__fdividef'): codes and scales bit for bit
      against the fast-division mode;
  quantizer 'rn' / 'fast' (tilelang_row_quant.py:27-46), incl. an owned slice;
  fp16_codec, pack_int8, unpack_int8 (tilelang_transport_tradeoffs.py:26-88);
  epilogue 'fp16' / 'int8_gather' (tilelang_transport_p2.py:15-47);
  row_gate_kernel (tilelang_dit_fusion.py:57-77);
  column epilogue kernel (tilelang_column_epilogue.py:11-27);
  norm_kernel (tilelang_dit_fusion.py:11-37): the reference calls the approximate
      rsqrtf, this path a correctly rounded one; compared within one fp16 ulp.
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
_TORCH = {"float16": torch.float16, "float32": torch.float32, "int8": torch.int8,
          "int32": torch.int32, "uint8": torch.uint8}


class RefKernels:
    def __init__(self):
        man, lib = REF / "tilelang_ref.json", REF / "libh3ref_tilelang.so"
        if not (man.exists() and lib.exists()):
            pytest.skip("reference TileLang kernels not built (oracle/tilelang_ref.py needs "
                        "the reference checkout and TileLang)")
        self.manifest = json.loads(man.read_text())
        self.lib = ctypes.CDLL(str(lib))

    def params(self, name):
        return self.manifest[name]["params"]

    def run(self, name, dev, **given):
        """Launches ref_<name> with the given tensors (by the factory's parameter
        names); parameters not given are allocated zeroed.  Returns every parameter."""
        bufs, ptrs = {}, []
        for p in self.params(name):
            t = given.get(p["name"])
            if t is None:
                t = torch.zeros(p["shape"], dtype=_TORCH[p["dtype"]], device=dev)
            else:
                t = t.to(dev).contiguous()
                assert list(t.shape) == p["shape"] and t.dtype == _TORCH[p["dtype"]], \
                    (name, p, t.shape, t.dtype)
            bufs[p["name"]] = t
            ptrs.append(t.data_ptr())
        fn = getattr(self.lib, "ref_" + name)
        fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        fn.restype = ctypes.c_int
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        assert fn(arr, torch.cuda.current_stream(dev).cuda_stream) == 0, name
        torch.cuda.synchronize(dev)
        return bufs


@pytest.fixture(scope="module")
def ref():
    return RefKernels()


def _np(t):
    return t.detach().cpu().numpy()


def _bits_equal(a, b, what=""):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (what, a.shape, b.shape, a.dtype, b.dtype)
    v = {1: np.uint8, 2: np.uint16, 4: np.uint32}[a.itemsize]
    bad = np.flatnonzero(a.view(v) != b.view(v))
    assert bad.size == 0, f"{what}: {bad.size}/{a.size} differ, first {a.flat[bad[0]]} vs {b.flat[bad[0]]}"


def _exp_free_gateup(rng, rows, width):
    """[gate | up] fp16 whose SwiGLU does not depend on the exponential's last bits:
    gates are 0, >= 17 (1 + exp(-gate) rounds to 1) or <= -89 (exp(-gate) = inf)."""
    mag = rng.uniform(17.0, 900.0, (rows, width))
    pick = rng.integers(0, 8, (rows, width))
    gate = np.where(pick == 0, 0.0, np.where(pick < 5, mag, -mag - 72.0))
    up = rng.standard_normal((rows, width))
    up[::9] *= rng.standard_t(3, size=up[::9].shape)
    return np.concatenate([gate, up], 1).astype(np.float16)


def _ordinary_gateup(rng, rows, width):
    g = rng.standard_normal((rows, width)) * 1.5
    u = rng.standard_normal((rows, width))
    g[::7] *= rng.standard_t(3, size=g[::7].shape)
    return np.concatenate([g, u], 1).astype(np.float16)


# ----------------------------------------------------------------------------
# FC2 producer
# ----------------------------------------------------------------------------
def test_fc2_stored_rotation_bit_exact_on_exp_free_gates(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width = ref.params("fc2_stored")[1]["shape"]
    x = _exp_free_gateup(np.random.default_rng(71), rows, width)
    xd = torch.from_numpy(x).to(cuda_device)
    r = ref.run("fc2_stored", cuda_device, X=xd)
    R_ref, M_ref = _np(r["R"]), _np(r["M"])
    rot, m = ops.swiglu_rotate_max(xd, "gateup_f16", store=True)
    _bits_equal(_np(rot), R_ref, "rotated vs reference")
    _bits_equal(_np(m).ravel(), M_ref.max(1), "row max vs reference")
    R_o, m_o = oracle.fc2_rotate(x, "gateup_f16")
    _bits_equal(R_o, R_ref, "oracle rotated vs reference")
    _bits_equal(np.asarray(m_o).ravel(), M_ref.max(1), "oracle row max vs reference")
    # phase 'maximum' writes the same group maxima without the values
    r2 = ref.run("fc2_maximum", cuda_device, X=xd)
    _bits_equal(_np(r2["M"]), M_ref, "maximum phase")


def test_fc2_codes_rn_bit_exact_on_exp_free_gates(ref, cuda_device, oracle):
    """stored -> row max -> quantizer('rn') of the reference against the TP1 single pass."""
    from h3tp import ops
    rows, width = ref.params("fc2_stored")[1]["shape"]
    assert ref.params("quant_rn")[2]["shape"] == [rows, width]
    x = _exp_free_gateup(np.random.default_rng(72), rows, width)
    xd = torch.from_numpy(x).to(cuda_device)
    r = ref.run("fc2_stored", cuda_device, X=xd)
    gmax = r["M"].amax(1, keepdim=True).contiguous()
    rq = ref.run("quant_rn", cuda_device, X=r["R"], Maximum=gmax)
    q, s, m = ops.swiglu_rotate_quantize_local(xd, "gateup_f16", "rn")
    _bits_equal(_np(q), _np(rq["Q"]), "codes")
    _bits_equal(_np(s), _np(rq["Scale"]), "scales")
    qo, so = oracle.row_quantize(oracle.fc2_rotate(x, "gateup_f16")[0], _np(gmax).ravel())
    _bits_equal(qo, _np(rq["Q"]), "oracle codes")
    _bits_equal(np.asarray(so).ravel(), _np(rq["Scale"]).ravel(), "oracle scales")


def test_fc2_recompute_fast_division_bit_exact_on_exp_free_gates(ref, cuda_device):
    from h3tp import ops
    rows, width = ref.params("fc2_recompute")[2]["shape"]
    x = _exp_free_gateup(np.random.default_rng(73), rows, width)
    xd = torch.from_numpy(x).to(cuda_device)
    gmax = ref.run("fc2_maximum", cuda_device, X=xd)["M"].amax(1, keepdim=True).contiguous()
    r = ref.run("fc2_recompute", cuda_device, X=xd, M=gmax)
    q, s = ops.swiglu_rotate_quantize(xd, gmax, "gateup_f16", division="fast")
    _bits_equal(_np(q), _np(r["Q"]), "codes")
    _bits_equal(_np(s), _np(r["S"]), "scales")


def test_fc2_ordinary_gates_differ_only_by_the_exponential(ref, cuda_device):
    """Ordinary gates: the reference's CUDA expf against this path's exponential.  The
    rotated values stay within a few ulps and the INT8 codes (rn, same maxima) almost
    never move; the counts are printed for the record."""
    from h3tp import ops
    rows, width = ref.params("fc2_stored")[1]["shape"]
    x = _ordinary_gateup(np.random.default_rng(74), rows, width)
    xd = torch.from_numpy(x).to(cuda_device)
    r = ref.run("fc2_stored", cuda_device, X=xd)
    rot, m = ops.swiglu_rotate_max(xd, "gateup_f16", store=True)
    R_ref, R = _np(r["R"]).astype(np.float64), _np(rot).astype(np.float64)
    scale = np.abs(R_ref).max(1, keepdims=True)
    err = np.abs(R - R_ref) / np.maximum(scale, 1e-30)
    differ = float(np.mean(_np(rot).view(np.uint32) != _np(r["R"]).view(np.uint32)))
    assert err.max() < 1e-6, err.max()
    gmax = r["M"].amax(1, keepdim=True).contiguous()
    rq = ref.run("quant_rn", cuda_device, X=r["R"], Maximum=gmax)
    q, _ = ops.row_quantize(rot, gmax, division="rn")
    dq = np.abs(_np(q).astype(np.int32) - _np(rq["Q"]).astype(np.int32))
    print(f"\n[reference fc2, ordinary gates] rotated values bit-identical: {1 - differ:.4%}; "
          f"max error / row max {err.max():.2e}; codes moved: {int((dq > 0).sum())} of {dq.size}")
    assert dq.max() <= 1 and (dq > 0).mean() < 1e-4


# ----------------------------------------------------------------------------
# row quantiser
# ----------------------------------------------------------------------------
def _quant_input(rng, rows, stride, start, width):
    """FP32 rows of varied magnitude, a global maximum above the owned slice's own
    (as after the MAX exchange), near-ties x / scale = k + 0.5 under the scale the
    kernels derive, and an all-zero row (the 1e-30 floor)."""
    X = (rng.standard_normal((rows, stride)) * rng.uniform(0.01, 50.0, (rows, 1))).astype(np.float32)
    X[1] = 0.0
    gmax = (np.abs(X).max(1) * np.float32(1.5)).astype(np.float32)
    scale = np.maximum(np.minimum(gmax, np.float32(3.4028234663852886e38)) * np.float32(1.0 / 127.0),
                       np.float32(1e-30)).astype(np.float32)
    k = rng.integers(-126, 126, (rows, 16)).astype(np.float32) + np.float32(0.5)
    X[:, start:start + 16] = (k * scale[:, None]).astype(np.float32)
    X[1] = 0.0
    return X, gmax


@pytest.mark.parametrize("name,division", [("quant_rn", "rn"), ("quant_fast", "fast"),
                                           ("quant_rn_slice", "rn")])
def test_row_quantizer_bit_exact(ref, cuda_device, oracle, name, division):
    from h3tp import ops
    meta = ref.manifest[name]["args"]  # rows, width, stride, start, division
    rows, width, stride, start = meta[:4]
    X, gmax = _quant_input(np.random.default_rng(80 + start), rows, stride, start, width)
    Xd = torch.from_numpy(X).to(cuda_device)
    Md = torch.from_numpy(gmax.reshape(-1, 1)).to(cuda_device)
    r = ref.run(name, cuda_device, X=Xd, Maximum=Md)
    q, s = ops.row_quantize(Xd, Md, width=width, start=start, division=division)
    _bits_equal(_np(q), _np(r["Q"]), "codes")
    _bits_equal(_np(s), _np(r["Scale"]), "scales")
    if division == "rn":
        qo, so = oracle.row_quantize(X, gmax, start=start, width=width)
        _bits_equal(qo, _np(r["Q"]), "oracle codes")


# ----------------------------------------------------------------------------
# transport codecs and epilogues
# ----------------------------------------------------------------------------
def _partials(rng, rows, width, shift):
    lim = int(60000 * 2 ** shift / 2)
    P = rng.integers(-lim, lim, (rows, width)).astype(np.int32)
    P[0, :8] = [0, 1, -1, 2 ** shift, -(2 ** shift) + 1, lim - 1, -lim, 3 * 2 ** (shift - 1)]
    return P


def test_fp16_codec_bit_exact(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width, shift = ref.manifest["encode_fp16"]["args"][:3]
    P = _partials(np.random.default_rng(90), rows, width, shift)
    Pd = torch.from_numpy(P).to(cuda_device)
    enc = ref.run("encode_fp16", cuda_device, X=Pd)["Y"]
    _bits_equal(_np(ops.fp16_encode(Pd, shift)), _np(enc), "encode")
    _bits_equal(oracle.fp16_encode(P, shift), _np(enc), "oracle encode")
    dec = ref.run("decode_fp16", cuda_device, X=enc)["Y"]
    _bits_equal(_np(ops.fp16_decode(enc, shift)), _np(dec), "decode")
    _bits_equal(oracle.fp16_decode(_np(enc), shift), _np(dec), "oracle decode")


def test_packed_int8_pack_unpack_bit_exact(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width = ref.manifest["pack_int8"]["args"][:2]
    rng = np.random.default_rng(91)
    P0, P1 = (_partials(rng, rows, width, 12) for _ in range(2))
    P0[3] = 0  # an all-zero group: the 1e-8 scale floor
    packed = [ref.run("pack_int8", cuda_device, X=torch.from_numpy(P).to(cuda_device))["Packed"]
              for P in (P0, P1)]
    for P, pk in zip((P0, P1), packed):
        _bits_equal(_np(ops.pack8(torch.from_numpy(P).to(cuda_device))), _np(pk), "pack")
        _bits_equal(oracle.pack8(P), _np(pk), "oracle pack")
    both = torch.cat(packed, 0)
    restored = ref.run("unpack_int8", cuda_device, P=both)["Y"]
    mine = ops.unpack8_finish(both.reshape(2, rows, -1), width, out_dtype=torch.int32)
    _bits_equal(_np(mine), _np(restored), "unpack")
    _bits_equal(oracle.unpack8_restore(_np(both).reshape(2, rows, -1), width), _np(restored),
                "oracle unpack")


def _scales(rng, rows, width):
    a = rng.uniform(1e-3, 5e-2, (rows, 1)).astype(np.float32)
    w = (rng.uniform(1e-3, 1e-2, width) / 512).astype(np.float32)
    return a, w


def test_row_epilogue_fp16_bit_exact(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width, _, shift = ref.manifest["epilogue_fp16"]["args"]
    rng = np.random.default_rng(92)
    payload = oracle.fp16_encode(_partials(rng, rows, width, shift), shift)
    a, w = _scales(rng, rows, width)
    Pd, Ad, Wd = (torch.from_numpy(v).to(cuda_device) for v in (payload, a, w))
    y = ref.run("epilogue_fp16", cuda_device, P=Pd, A=Ad, W=Wd)["Y"]
    _bits_equal(_np(ops.row_reduce_finish(Pd, shift, Ad, Wd, torch.float32)), _np(y), "epilogue")
    _bits_equal(oracle.row_reduce_finish(payload[None], shift, a.ravel(), w, out="f32"), _np(y),
                "oracle epilogue")


def test_row_epilogue_packed_int8_bit_exact(ref, cuda_device):
    from h3tp import ops
    rows, width = ref.manifest["epilogue_int8"]["args"][:2]
    rng = np.random.default_rng(93)
    parts = [ops.pack8(torch.from_numpy(_partials(rng, rows, width, 12)).to(cuda_device))
             for _ in range(2)]
    both = torch.cat(parts, 0)
    a, w = _scales(rng, rows, width)
    Ad, Wd = torch.from_numpy(a).to(cuda_device), torch.from_numpy(w).to(cuda_device)
    y = ref.run("epilogue_int8", cuda_device, P=both, A=Ad, W=Wd)["Y"]
    mine = ops.unpack8_finish(both.reshape(2, rows, -1), width, Ad, Wd, torch.float32)
    _bits_equal(_np(mine), _np(y), "packed epilogue")


def test_row_gate_bit_exact(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width, mod_rows, shift = ref.manifest["row_gate"]["args"][:4]
    rng = np.random.default_rng(94)
    payload = oracle.fp16_encode(_partials(rng, rows, width, shift), shift)
    a, w = _scales(rng, rows, width)
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((mod_rows, width)).astype(np.float32)
    L = rng.integers(0, mod_rows, rows).astype(np.int32)
    dev = cuda_device
    r = ref.run("row_gate", dev, P=torch.from_numpy(payload), A=torch.from_numpy(a),
                W=torch.from_numpy(w), X=torch.from_numpy(X.copy()), Gate=torch.from_numpy(G),
                Labels=torch.from_numpy(L))
    mine = torch.from_numpy(X.copy()).to(dev)
    ops.row_reduce_finish(torch.from_numpy(payload).to(dev), shift, torch.from_numpy(a).to(dev),
                          torch.from_numpy(w).to(dev), residual=mine,
                          gate=torch.from_numpy(G).to(dev), labels=torch.from_numpy(L).to(dev))
    _bits_equal(_np(mine), _np(r["X"]), "row gate")
    ref_o = X.copy()
    oracle.row_reduce_finish(payload[None], shift, a.ravel(), w, out="residual", residual=ref_o,
                             gate=G, labels=L)
    _bits_equal(ref_o, _np(r["X"]), "oracle row gate")


def test_column_epilogue_bit_exact(ref, cuda_device, oracle):
    from h3tp import ops
    rows, width = ref.manifest["column_epilogue"]["args"][:2]
    rng = np.random.default_rng(95)
    C = rng.integers(-(1 << 24), 1 << 24, (rows, width)).astype(np.int32)
    a = rng.uniform(1e-3, 5e-2, (rows, 1)).astype(np.float32)
    w = rng.uniform(1e-3, 1e-2, width).astype(np.float32)
    Cd, Ad, Wd = (torch.from_numpy(v).to(cuda_device) for v in (C, a, w))
    y = ref.run("column_epilogue", cuda_device, C=Cd, A=Ad, W=Wd)["Y"]
    _bits_equal(_np(ops.column_dequantize(Cd, Ad, Wd)), _np(y), "column epilogue")
    _bits_equal(oracle.column_epilogue(C, a.ravel(), w), _np(y), "oracle column epilogue")


def test_modulated_norm_within_one_ulp_of_reference_kernel(ref, cuda_device):
    """The reference's norm kernel calls the approximate rsqrtf; this path rounds
    1/sqrt correctly.  Outputs agree within one fp16 ulp; the share of identical
    values is printed for the record."""
    from h3tp import ops
    rows, width, mod_rows, eps = ref.manifest["modulated_norm"]["args"][:4]
    rng = np.random.default_rng(96)
    x = (rng.standard_normal((rows, width)) * rng.uniform(0.1, 30, (rows, 1))).astype(np.float16)
    W = rng.uniform(0.5, 1.5, width).astype(np.float32)
    sh = (rng.standard_normal((mod_rows, width)) * 0.1).astype(np.float32)
    sc = (rng.standard_normal((mod_rows, width)) * 0.1).astype(np.float32)
    L = rng.integers(0, mod_rows, rows).astype(np.int32)
    dev = cuda_device
    t = {k: torch.from_numpy(v).to(dev) for k, v in
         dict(X=x, W=W, Shift=sh, Scale=sc, Labels=L).items()}
    y = _np(ref.run("modulated_norm", dev, **t)["Y"])
    _, _, h = ops.modulated_norm_quantize(t["X"], t["W"], eps, t["Shift"], t["Scale"], t["Labels"],
                                          quantize=False)
    h = _np(h)
    ulps = np.abs(h.view(np.int16).astype(np.int32) - y.view(np.int16).astype(np.int32))
    same = float((ulps == 0).mean())
    print(f"\n[reference norm kernel] bit-identical: {same:.4%}, max ulps {ulps.max()}")
    assert ulps.max() <= 1 and same > 0.99
