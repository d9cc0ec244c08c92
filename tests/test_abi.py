"""C ABI checks that need no GPU: the library loads, exports every entry point the
header declares, and rejects bad arguments before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from flashmlp_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "flashmlp_b200.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fmlp_[a-z0-9_]+)\s*\(", text)))


def header_defines():
    return dict((m[0], int(m[1])) for m in re.findall(r"#define\s+(FMLP_[A-Z0-9_]+)\s+(\d+)", HEADER.read_text()))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 7
    for n in names:
        assert hasattr(L, n), f"{n} declared in {HEADER.name} but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_python_constants_match_header():
    d = header_defines()
    for k, v in d.items():
        if hasattr(_lib, k):
            assert getattr(_lib, k) == v, k
    assert d["FMLP_ACT_LEAKY_RELU"] == _lib.FMLP_ACT_LEAKY_RELU
    assert d["FMLP_DTYPE_BF16"] == _lib.FMLP_DTYPE_BF16


def test_error_strings_and_version():
    L = _lib.lib()
    assert L.fmlp_abi_version() == 100
    for code in range(0, 14):
        s = L.fmlp_error_string(code).decode()
        assert s and s != "unknown error"
    assert L.fmlp_error_string(99).decode() == "unknown error"


def test_argument_validation_without_device():
    L = _lib.lib()
    nul = ctypes.c_void_p(0)
    d = header_defines()
    # bad dtype, negative sizes, unsupported D / E are rejected before any CUDA call
    assert L.fmlp_fwd(nul, nul, nul, nul, 1, 128, 64, 64, 7, 0, nul) == d["FMLP_ERR_UNSUPPORTED_DTYPE"]
    assert L.fmlp_fwd(nul, nul, nul, nul, -1, 128, 64, 64, 1, 0, nul) == d["FMLP_ERR_INVALID_SHAPE"]
    assert L.fmlp_fwd(nul, nul, nul, nul, 1, 128, 72, 64, 1, 0, nul) == d["FMLP_ERR_UNSUPPORTED_D"]
    assert L.fmlp_fwd(nul, nul, nul, nul, 1, 128, 512, 64, 1, 0, nul) == d["FMLP_ERR_UNSUPPORTED_D"]
    assert L.fmlp_fwd(nul, nul, nul, nul, 1, 128, 64, 100, 1, 0, nul) == d["FMLP_ERR_UNSUPPORTED_E"]
    assert L.fmlp_bwd(nul, nul, nul, nul, nul, nul, nul, nul, 0, 1, 128, 272, 64, 1, 0, nul) == d["FMLP_ERR_UNSUPPORTED_D"]
    assert L.fmlp_sgd_update(nul, nul, -5, 0.1, 1, nul) == d["FMLP_ERR_INVALID_SHAPE"]
    assert L.fmlp_sgd_update(nul, nul, 5, 0.1, 3, nul) == d["FMLP_ERR_UNSUPPORTED_DTYPE"]
    assert L.fmlp_bwd_workspace_size(32, 65536, 128, 2048, 1) == 0  # no device here
    assert L.fmlp_bwd_workspace_size_min(32, 65536, 128, 2048, 1) == 0
    assert L.fmlp_bwd_plan(1, 128, 72, 64, 1, 0, None, None, None) == d["FMLP_ERR_UNSUPPORTED_D"]
    assert L.fmlp_bwd_plan(1, 128, 64, 100, 1, 0, None, None, None) == d["FMLP_ERR_UNSUPPORTED_E"]
    assert L.fmlp_bwd_noalloc(nul, nul, nul, nul, nul, nul, nul, 1, 128, 272, 64, 1, 0, nul) == d["FMLP_ERR_UNSUPPORTED_D"]


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libflashmlp_b200.so")
    with pytest.raises(ImportError, match="not built"):
        _lib.lib()


def test_fp8_forward_validation_without_device():
    """fmlp_fwd_fp8 rejects bad shapes, output dtypes and scales before any CUDA call."""
    L = _lib.lib()
    nul = ctypes.c_void_p(0)
    d = header_defines()
    ok_scales = (1.0, 1.0, 1.0, 1.0)
    def call(H, B, D, E, scales=ok_scales, out=1):
        return L.fmlp_fwd_fp8(nul, nul, nul, nul, H, B, D, E, *scales, 2, out, nul)
    assert call(-1, 128, 64, 128) == d["FMLP_ERR_INVALID_SHAPE"]
    assert call(1, 128, 64, 128, out=2) == d["FMLP_ERR_UNSUPPORTED_DTYPE"]  # fp32 output
    assert call(1, 128, 144, 128) == d["FMLP_ERR_UNSUPPORTED_D"]             # D > 128
    assert call(1, 128, 72, 128) == d["FMLP_ERR_UNSUPPORTED_D"]              # D % 16
    assert call(1, 128, 64, 136) == d["FMLP_ERR_UNSUPPORTED_E"]              # E % 16
    assert call(1, 128, 64, 128, (1.0, 0.0, 1.0, 1.0)) == d["FMLP_ERR_INVALID_SCALE"]
    assert call(1, 128, 64, 128, (1.0, 1.0, float("nan"), 1.0)) == d["FMLP_ERR_INVALID_SCALE"]
    assert call(1, 128, 64, 128, (1.0, 1.0, 1.0, float("inf"))) == d["FMLP_ERR_INVALID_SCALE"]
