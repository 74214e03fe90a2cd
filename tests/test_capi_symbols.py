"""The C-ABI library loads and exports every entry point include/h3b200.h declares
(no compute: this runs without a GPU)."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "h3b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(h3_[a-z0-9_]+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "h3_int8_gemm_i32" in names and "h3_row_reduce_finish" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    from h3tp import _native
    lib = _native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) <= set(_native.SIGNATURES), "ctypes signatures missing"
    assert lib.h3_abi_version() == 1
    assert lib.h3_status_string(1) == b"invalid argument or unsupported geometry"


def test_transport_shift_is_host_only():
    from h3tp import _native
    lib = _native.load()
    # shift_for(local_k) at TP2 (tilelang_transport_tradeoffs.py:20-22) on full K
    assert lib.h3_transport_shift(2 * 7168) == 12
    assert lib.h3_transport_shift(2 * 3584) == 11
    assert lib.h3_transport_shift(8192) == 12
    assert lib.h3_transport_shift(3072) == 10
