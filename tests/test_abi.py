"""CPU tests of the C-ABI boundary: the library loads, exports every entry point include/*.h declares, and rejects bad
arguments on the host with the documented status codes (no GPU needed: validation precedes any CUDA call)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from vllm_espalier_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(esp_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"esp_dense", "esp_dequant", "esp_had", "esp_last_error", "esp_device_status"} <= set(names)


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports(name):
    lib = C.CDLL(str(_lib.library_path()))
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_signatures_cover_header():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES), "every declared entry point has a ctypes signature"


def declared_arity():
    """name -> number of parameters of each declaration in include/*.h."""
    out = {}
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(esp_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
            params = m.group(2).strip()
            out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_signatures_match_header_arity():
    """Every ctypes signature has as many arguments as its C declaration: a mismatch would pass garbage through the
    ABI instead of failing."""
    arity = declared_arity()
    assert arity, "no declarations parsed"
    bad = {n: (k, len(_lib.SIGNATURES[n][1])) for n, k in arity.items() if len(_lib.SIGNATURES[n][1]) != k}
    assert not bad, f"header vs ctypes argument counts: {bad}"


def test_host_validation_without_gpu():
    lib = _lib.lib()
    assert lib.esp_version() >= 100
    # bad codebook / width
    rc = lib.esp_dequant(C.c_void_p(16), 64, 64, 8, 3, C.c_void_p(16), None)
    assert rc == _lib.ESP_ERR_UNSUPPORTED and b"codebook" in lib.esp_last_error()
    # bad shape
    rc = lib.esp_dequant(C.c_void_p(16), 60, 64, 8, 7, C.c_void_p(16), None)
    assert rc == _lib.ESP_ERR_INVALID
    # dense: too many rows, too many matrices, null pointers
    mats = (_lib.esp_matrix_t * 1)(_lib.esp_matrix_t(16, 16, 16, 128, 0))
    args = [C.c_void_p(16), 1, 256, 33, 256, mats, 1, 8, 7, C.c_void_p(16), 1, 128, C.c_void_p(16), 1 << 20,
            C.c_void_p(16), 1 << 24, C.c_void_p(16), 8, None]
    assert lib.esp_dense(*args) == _lib.ESP_ERR_INVALID and b"32 rows" in lib.esp_last_error()
    args[3] = 4
    args[6] = 5
    assert lib.esp_dense(*args) == _lib.ESP_ERR_INVALID
    args[6] = 1
    args[7] = 6          # E2M1 / int6 at 3 bits is compiled, int6 at k2 = 6 yes; use an uncompiled one
    args[8] = 3
    args[7] = 8
    assert lib.esp_dense(*args) == _lib.ESP_ERR_UNSUPPORTED
    args[7], args[8] = 8, 7
    args[17] = 0         # counters too small
    assert lib.esp_dense(*args) == _lib.ESP_ERR_SCRATCH
    assert lib.esp_dense(None, *args[1:]) == _lib.ESP_ERR_INVALID
    # the diagnostic wait checks its pointers before any launch
    assert lib.esp_wait_flag(None, 1, C.c_void_p(16), None) == _lib.ESP_ERR_INVALID
    assert lib.esp_wait_flag(C.c_void_p(16), 1, None, None) == _lib.ESP_ERR_INVALID
    assert b"null" in lib.esp_last_error()


def test_ext_surface_names():
    """The reference extension's function names that this library implements (experts.cpp:234-248)."""
    e = _lib._Ext
    for name in ("dense", "dequant", "had"):
        assert callable(getattr(e, name))
