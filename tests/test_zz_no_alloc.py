"""h3_column_linear_noalloc: the column linear for callers that may not allocate device
memory (inside runtimes that budget every device byte through their own pool, on
paths that cannot take cudaMalloc's implicit synchronisation).

It is called directly through the C ABI and must reproduce, bit for bit, the result of
the existing two-call path (h3_column_quantize then h3_int8_gemm_column) on two calls
in a row with different shapes - the second call reuses the static scratch the first
one left behind - and must refuse a problem larger than its static scratch without
launching anything.  This file is collected last so a failure here cannot hide
another test."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H3_ERR_INVALID = 1


def _scratch_bytes() -> int:
    """H3_NOALLOC_SCRATCH_BYTES as the library's header defines it."""
    header = (Path(__file__).resolve().parents[1] / "include" / "h3b200.h").read_text()
    m = re.search(r"#define\s+H3_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", header)
    assert m, "H3_NOALLOC_SCRATCH_BYTES not found in include/h3b200.h"
    return int(m.group(1)) << int(m.group(2))


def _fits(m: int, k: int, limit: int) -> bool:
    """The header's size rule: 256 + roundup256(4 m) + m k <= limit."""
    return 256 + -(-4 * m // 256) * 256 + m * k <= limit


def _noalloc(x, w, ws, bias, convrot):
    from h3tp import _native
    lib = _native.load()
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.float16, device=x.device)
    st = lib.h3_column_linear_noalloc(
        x.data_ptr(), m, k, int(convrot), w.data_ptr(), n, ws.data_ptr(), ws.numel(),
        None if bias is None else bias.data_ptr(), out.data_ptr(),
        torch.cuda.current_stream(x.device).cuda_stream)
    return st, out


def _existing(x, w, ws, bias, convrot):
    from h3tp import ops
    q, a = ops.column_quantize(x, convrot)
    return ops.int8_gemm_column(q, w, a, ws, bias)


def _case(dev, seed, m, k, n, convrot, bias):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[:, rng.permutation(k)[: max(1, k // 100)]] *= 20
    x = torch.from_numpy(x.astype(np.float16)).to(dev)
    w = torch.from_numpy(rng.integers(-127, 128, size=(n, k), dtype=np.int8)).to(dev)
    ws = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=(n, 1)).astype(np.float32)).to(dev)
    b = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float32)).to(dev) if bias else None
    return x, w, ws, b


def test_noalloc_column_linear_matches_existing_path(cuda_device):
    from h3tp import _native
    lib = _native.load()
    cases = [(1, 300, 3072, 512, True, False),   # CTA-pair GEMM path, rotation
             (2, 77, 1024, 264, False, True)]    # single-CTA path, ragged N, bias
    for seed, m, k, n, convrot, bias in cases:
        x, w, ws, b = _case(cuda_device, seed, m, k, n, convrot, bias)
        st, got = _noalloc(x, w, ws, b, convrot)
        assert st == 0, lib.h3_status_string(st)
        ref = _existing(x, w, ws, b, convrot)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
        code = ctypes.c_int(-1)
        assert lib.h3_column_linear_noalloc_error(cuda_device.index or 0, ctypes.byref(code)) == 0
        assert code.value == 0


def test_noalloc_rejects_problems_beyond_the_static_scratch(cuda_device):
    from h3tp import _native
    lib = _native.load()
    limit = _scratch_bytes()
    k = 4096
    m_max = limit // k
    while not _fits(m_max, k, limit):
        m_max -= 1
    x = torch.zeros((m_max + 1, k), dtype=torch.float16, device=cuda_device)
    w = torch.zeros((256, k), dtype=torch.int8, device=cuda_device)
    ws = torch.ones((256, 1), dtype=torch.float32, device=cuda_device)
    # one row beyond the rule is refused, launching nothing
    st, out = _noalloc(x, w, ws, None, True)
    assert st == H3_ERR_INVALID
    # the largest problem inside the rule still runs
    st, out = _noalloc(x[:m_max], w, ws, None, True)
    assert st == 0, lib.h3_status_string(st)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
