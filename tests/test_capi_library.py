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


def test_pool_scatter_rejects_bad_arguments_on_the_host():
    """rb_rep_gather_pool_scatter validates its destinations before any device
    work.  The pointers below are never dereferenced: every call fails a host
    check before the launch (a call that passed them all would launch a kernel on
    fake addresses, so none may)."""
    from baidu_cti_grab_b200 import _lib

    lib = _lib.load()
    S, N, ld = 2, 10, 1024
    fake = 1 << 20  # 1 MiB: aligned, never dereferenced
    vals = _lib.ptr_array([fake, fake])
    offs = _lib.ptr_array([fake, fake])
    nnz = _lib.i64_array([5, 5])
    cols = _lib.i32_array([0, 1])

    def call(dest, begin, num_dest, ld=ld, shift=0, cols=cols, nnz=nnz):
        rc = lib.rb_rep_gather_pool_scatter(fake, _lib.RB_BF16, 100, 512, vals, offs, nnz, cols, S, N,
                                            _lib.ptr_array(dest), _lib.i64_array(begin), num_dest, ld, shift, None)
        return rc, _lib.last_error()

    assert call([fake], [0, N], 0)[0] == _lib.RB_ERR_VALUE                       # no destination
    assert call([fake] * 9, list(range(10)), 9)[0] == _lib.RB_ERR_VALUE          # more than RB_MAX_DEST
    rc, msg = call([fake, fake], [0, 4, 9], 2)                                   # does not end at num_items
    assert rc == _lib.RB_ERR_VALUE and "dest_begin" in msg
    rc, msg = call([fake, fake], [0, 6, 4], 2)                                   # decreasing (and wrong end)
    assert rc == _lib.RB_ERR_VALUE
    rc, msg = call([fake + 16, fake], [0, 6, 10], 2)                             # bf16 rows need 32-byte alignment
    assert rc == _lib.RB_ERR_VALUE and "aligned" in msg
    rc, msg = call([fake, fake], [0, 6, 10], 2, ld=520)                          # ld breaks the row alignment
    assert rc == _lib.RB_ERR_VALUE
    rc, msg = call([fake, fake], [0, 6, 10], 2, cols=_lib.i32_array([0, 2]))    # slot 1 past ld
    assert rc == _lib.RB_ERR_VALUE and "col_slot" in msg
    rc, msg = call([fake, fake], [0, 6, 10], 2, shift=N)                         # item_shift out of range
    assert rc == _lib.RB_ERR_VALUE and "item_shift" in msg
    rc, msg = call([fake, fake], [0, 6, 10], 2, nnz=_lib.i64_array([5, -1]))    # negative nnz
    assert rc == _lib.RB_ERR_VALUE


def test_ipc_entry_points_reject_null_arguments():
    import ctypes

    from baidu_cti_grab_b200 import _lib

    lib = _lib.load()
    off = ctypes.c_int64(0)
    assert lib.rb_ipc_export(None, None, ctypes.byref(off)) == _lib.RB_ERR_VALUE
    ptr = ctypes.c_void_p(0)
    assert lib.rb_ipc_import(None, 0, ctypes.byref(ptr)) == _lib.RB_ERR_VALUE
    assert lib.rb_ipc_close(None, 0) == _lib.RB_ERR_VALUE


def test_table_row_count_above_int32_is_rejected():
    """Ids are clamped to [0, num_rows - 1] in 32 bits on the device, so every
    gather entry point refuses num_rows >= 2^31 on the host (a caller passing
    the table's element count instead of its rows would otherwise read outside
    the table).  The pointers are never dereferenced: each call fails the host
    check before any launch."""
    from baidu_cti_grab_b200 import _lib

    lib = _lib.load()
    fake = 1 << 20
    S, N = 2, 10
    vals, offs = _lib.ptr_array([fake, fake]), _lib.ptr_array([fake, fake])
    nnz, cols = _lib.i64_array([5, 5]), _lib.i32_array([0, 1])
    too_many = 1 << 31
    rc = lib.rb_rep_gather_ln_quant(fake, _lib.RB_BF16, too_many, 512, vals, offs, nnz, S, N, fake, fake,
                                    _lib.RB_BF16, 1e-5, 0, None, 0, fake, S * 512, fake, None, None, None)
    assert rc == _lib.RB_ERR_VALUE and "num_rows" in _lib.last_error()
    rc = lib.rb_rep_gather_pool(fake, _lib.RB_BF16, too_many, 512, vals, offs, nnz, cols, S, N, fake, S * 512,
                                None)
    assert rc == _lib.RB_ERR_VALUE and "num_rows" in _lib.last_error()
    rc = lib.rb_rep_gather_pool_scatter(fake, _lib.RB_BF16, too_many, 512, vals, offs, nnz, cols, S, N,
                                        _lib.ptr_array([fake]), _lib.i64_array([0, N]), 1, S * 512, 0, None)
    assert rc == _lib.RB_ERR_VALUE and "num_rows" in _lib.last_error()


def test_split_k_workspace_sizes():
    """rb_w8a8_gemm_workspace_size (host logic; without a GPU the library
    assumes a 148-SM B200): no workspace up to M = 256 (GEMV and the
    swapped-operand cluster kernel) or once the CTA-pair tiles cover more than
    half of the 74 pairs; K splits of the one-SM 128 x 256 tiles from M = 257,
    of the pairs' 256 x 256 tiles from M = 2048; and never more int32 than the
    20 MiB array of rb_w8a8_gemm_noalloc holds."""
    from baidu_cti_grab_b200 import _lib

    lib = _lib.load()
    K, N = 14336, 512

    def ws(M, n=N, k=K):
        return int(lib.rb_w8a8_gemm_workspace_size(M, n, k))

    for M in (1, 16, 17, 128, 256):
        assert ws(M) == 0, M
    assert ws(512) == 16 * 512 * N      # 8 one-SM tiles: 148 // 8 = 18 splits, capped at 16
    assert ws(1024) == 9 * 1024 * N     # 16 tiles: 148 // 16 = 9 splits
    assert ws(2048) == 4 * 2048 * N     # 16 pair tiles: 74 // 16 = 4 splits
    assert ws(4096) == 2 * 4096 * N     # 32 pair tiles: 2 splits
    assert ws(4608) == 2 * 4608 * N     # 36 pair tiles: still at most half of the pairs
    for M in (4609, 8192, 32768, 103917):
        assert ws(M) == 0, M
    assert ws(0) == 0 and ws(4096, k=15) == 0  # empty, or K not a multiple of 16
    scratch = 5 * 1024 * 1024
    worst = max(ws(M) for M in range(1, 8193))
    assert 0 < worst <= scratch
