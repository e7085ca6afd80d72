"""libxdna_b200.so loads on a machine without a GPU and exports the C ABI."""
import ctypes
import re
from pathlib import Path

import pytest

from xdna_train import _abi

HEADER = Path(__file__).resolve().parent.parent / "include" / "b2.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const char\*|b2_status|int|size_t)\s+(b2_\w+)\(", text, re.M)))


def test_header_declares_the_boundary():
    names = declared()
    for must in ("b2_conv3x3_fwd", "b2_conv3x3_dgrad", "b2_conv3x3_wgrad", "b2_gemm_bf16", "b2_fused_adam",
                 "b2_pack_rows_bf16", "b2_region_sqdiff_sum_bf16"):
        assert must in names


def test_every_declared_symbol_is_exported_and_bound():
    lib = ctypes.CDLL(str(_abi.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), name
        assert name in _abi.SIGNATURES, name


def test_argument_errors_need_no_gpu():
    L = _abi.lib()
    assert L.b2_abi_version() >= 1
    st = L.b2_pack_rows_bf16(None, 1, 1, 1, 1, 1, 1, 1, 1, 1, None, None)
    assert st == 1
    assert b"null pointer" in L.b2_last_error()
    st = L.b2_conv3x3_fwd(8, 8, None, 8, 1, 1, 1, 1, 0, 1, 1, 1, 1, 0, None)
    assert st == 1 and b"bad shape" in L.b2_last_error()
    with pytest.raises(_abi.B2Error):
        _abi.call("b2_region_relu_bf16", None, None, 5, None)


def _declared_arity():
    """Parameter count of every b2_* function declared in include/b2.h."""
    text = re.sub(r"/\*.*?\*/|//[^\n]*", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"(?:const char\*|b2_status|int|size_t)\s+(b2_\w+)\(([^;]*?)\)\s*;", text, re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_bindings_match_the_header_arity():
    arity = _declared_arity()
    assert set(arity) == set(declared())
    for name, n in arity.items():
        assert len(_abi.SIGNATURES[name]) == n, f"{name}: header declares {n} parameters, ctypes binds " \
                                                f"{len(_abi.SIGNATURES[name])}"
