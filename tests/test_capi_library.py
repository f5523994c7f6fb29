"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
entry point that include/rep_b200.h declares; the Python layer refuses CPU
tensors instead of falling back."""

import ctypes
import os
import re

import pytest

from conftest import REPO


def _declared():
    with open(os.path.join(REPO, "include", "rep_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(rb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header_symbols():
    from baidu_cti_grab_b200 import build

    path = build.build()
    lib = ctypes.CDLL(path)
    names = _declared()
    assert "rb_rep_gather_ln_quant" in names and "rb_w8a8_gemm" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from baidu_cti_grab_b200 import _lib

    names = set(_declared())
    bound = set(_lib.SIGNATURES) | {"rb_last_error"}
    assert names <= bound, names - bound


def test_cpu_tensors_are_refused():
    torch = pytest.importorskip("torch")
    from baidu_cti_grab_b200 import quantization, w8a8_triton_kernels as wk, device_ops

    x = torch.randn(4, 64)
    with pytest.raises(RuntimeError):
        quantization.quantize_rows_int8_triton(x)
    with pytest.raises(RuntimeError):
        wk.dynamic_per_token_quantize_activation(x)
    with pytest.raises(RuntimeError):
        device_ops.w8a8_gemm(torch.zeros(2, 16, dtype=torch.int8), torch.zeros(4, 16, dtype=torch.int8), None, None,
                             torch.zeros(2, 4, dtype=torch.int32))


def test_status_codes_map_to_exceptions():
    from baidu_cti_grab_b200 import _lib

    lib = _lib.load()
    # invalid arguments are rejected on the host before any device work
    rc = lib.rb_w8a8_gemm(None, 16, None, 16, 4, 4, 16, None, 0, 1, None, 0, None, 0, None, 4, 1, None)
    assert rc == _lib.RB_ERR_VALUE
    assert "null" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.call("rb_quant_static", None, 0, -1, None, 0, None, None)
    rc = lib.rb_rep_gather_ln_quant(None, 1, 10, 256, None, None, None, 28, 5, None, None, 1, 1e-5, 0, None, 0,
                                    None, 14336, None, None, None, None)
    assert rc in (_lib.RB_ERR_VALUE, _lib.RB_ERR_UNSUPPORTED)
