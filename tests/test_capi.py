"""CPU tests of the C ABI: the library loads, exports every symbol the public
headers declare, and its host-only entry points behave (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from rust_katago_b200 import _capi

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^KB_API\s+[\w\s\*]+?\b(kb_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_headers_declare_symbols():
    names = declared_symbols()
    assert len(names) >= 20
    assert "kb_last_error" in names and "kb_int8_gemm_i32" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_capi.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_every_declared_symbol():
    assert sorted(_capi.SIGNATURES) == declared_symbols()


def test_version_and_error_string():
    lib = _capi.load()
    assert lib.kb_version() >= 100
    assert isinstance(lib.kb_last_error(), bytes)


def test_host_weight_quantiser_matches_oracle(oracle):
    from rust_katago_b200 import int8

    rng = np.random.default_rng(5)
    for n, k in [(4, 8), (64, 200), (96, 768)]:
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        w[0] = 0.0
        q, s = int8.quantize_weights(w)
        oq, os_ = oracle.quantize_weights(w)
        assert (q == oq).all() and (s.view(np.uint32) == os_.view(np.uint32)).all()


def test_host_weight_quantiser_rejects_bad_input():
    from rust_katago_b200 import int8

    w = np.zeros((4, 8), np.float32)
    w[2, 3] = np.inf
    with pytest.raises(_capi.KbError, match="NaN or infinity"):
        int8.quantize_weights(w)
    with pytest.raises(_capi.KbError, match="invalid INT8 weight shape"):
        int8.quantize_weights(np.zeros((6, 8), np.float32))
