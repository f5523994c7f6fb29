"""numpy front end of the CPU oracle (oracle/rep_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product package never
imports this module.

Functions mirror the reference pieces they restate (file:line in the C file's
header).  bfloat16 arrays are passed around as uint16 bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librep_oracle.so")

F32, BF16, F16, I32 = 0, 1, 2, 3
_DT = {"float32": F32, "bfloat16": BF16, "float16": F16}
MAX_SLOTS = 32  # the widest row the CUDA kernels take (32 slots x 512)

_lib = None


def build() -> str:
    """Compile the oracle shared library (make -C oracle)."""
    src = os.path.join(HERE, "rep_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.rbo_embedding_bag_sum.argtypes = [vp, i32, i64, i64, vp, i64, vp, i64, vp, i32]
        L.rbo_layernorm_stats_rows.argtypes = [vp, i64, i64, f32, vp, vp]
        L.rbo_layernorm_apply_rows.argtypes = [vp, i64, i64, vp, vp, vp, vp, i32, vp]
        L.rbo_quant_dynamic_v2.argtypes = [vp, i64, i64, vp, vp]
        L.rbo_quant_static_v2.argtypes = [vp, i64, f32, vp]
        L.rbo_quant_rows_v1.argtypes = [vp, i64, i64, vp, vp]
        L.rbo_gemm_i8_i32.argtypes = [vp, vp, i64, i64, i64, vp]
        L.rbo_scaled_epilogue.argtypes = [vp, i64, i64, vp, i32, vp, vp, i32, vp]
        L.rbo_rep_pool_stats.argtypes = [vp, i32, i64, vp, vp, vp, i64, i64, f32, vp, vp, vp, i32]
        L.rbo_rep_finish.argtypes = [vp, i32, i64, i64, vp, vp, vp, vp, i32, f32, vp, vp, vp, i32]
        L.rbo_round_to_dtype.argtypes = [vp, i64, i32, vp]
        L.rbo_dtype_to_f32.argtypes = [vp, i64, i32, vp]
        for fn in (L.rbo_embedding_bag_sum, L.rbo_layernorm_stats_rows, L.rbo_layernorm_apply_rows,
                   L.rbo_quant_dynamic_v2, L.rbo_quant_static_v2, L.rbo_quant_rows_v1, L.rbo_gemm_i8_i32,
                   L.rbo_scaled_epilogue, L.rbo_rep_pool_stats, L.rbo_rep_finish, L.rbo_round_to_dtype,
                   L.rbo_dtype_to_f32):
            fn.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------- dtypes
def bf16_bits_to_f32(u: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().rbo_round_to_dtype(_p(x), x.size, BF16, _p(out))
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` and widen back to fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "float32":
        return x.copy()
    bits = np.empty(x.shape, dtype=np.uint16)
    lib().rbo_round_to_dtype(_p(x), x.size, _DT[dtype], _p(bits))
    out = np.empty(x.shape, dtype=np.float32)
    lib().rbo_dtype_to_f32(_p(bits), x.size, _DT[dtype], _p(out))
    return out


# ------------------------------------------------------ embedding bag sum
def embedding_bag_sum(table: np.ndarray, table_dtype: str, values: np.ndarray, offsets: np.ndarray,
                      out_dtype: Optional[str] = None) -> np.ndarray:
    """models.py:27-33 for one slot.  Returns fp32 values rounded to out_dtype (default: table dtype)."""
    out_dtype = table_dtype if out_dtype is None else out_dtype
    table = np.ascontiguousarray(table)
    values = np.ascontiguousarray(values, dtype=np.int64)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    n = len(offsets) - 1
    dim = table.shape[1]
    out = np.empty((n, dim), dtype=np.float32)
    lib().rbo_embedding_bag_sum(_p(table), _DT[table_dtype], table.shape[0], dim, _p(values),
                                len(values), _p(offsets), n, _p(out), F32)
    return round_to(out, out_dtype)


# -------------------------------------------------------------- LayerNorm
def rsqrt_nearest(v: np.ndarray) -> np.ndarray:
    """Correctly rounded fp32 1/sqrt(v): the CPU-only stand-in for CUDA's rsqrtf,
    which ATen's LayerNorm calls and which differs from it by up to 2 ulp."""
    return (1.0 / np.sqrt(np.asarray(v, dtype=np.float64))).astype(np.float32)


def _rstd(var_eps: np.ndarray, rsqrt) -> np.ndarray:
    r = rsqrt_nearest(var_eps) if rsqrt is None else np.asarray(rsqrt(var_eps), dtype=np.float32)
    return np.ascontiguousarray(r.reshape(var_eps.shape), dtype=np.float32)


def layernorm_stats(x: np.ndarray, eps: float) -> Tuple[np.ndarray, np.ndarray]:
    """Per-row mean and fl(var + eps) of rows x[M, H] (H % 4 == 0) in ATen CUDA's order."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, h = x.shape
    if h % 4 != 0:
        raise ValueError(f"row width {h} is not a multiple of 4")
    mean = np.empty(m, dtype=np.float32)
    var_eps = np.empty(m, dtype=np.float32)
    lib().rbo_layernorm_stats_rows(_p(x), m, h, eps, _p(mean), _p(var_eps))
    return mean, var_eps


def layernorm_rows(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float,
                   out_dtype: str, rsqrt=None) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """nn.LayerNorm of rows x[M, H] (fp32 values of the row dtype) as ATen's CUDA
    kernel computes it.  ``rsqrt`` maps fl(var + eps) to rstd: pass the GPU's
    rsqrtf (e.g. torch.rsqrt on a CUDA tensor) for bit-exact parity; the default
    is the correctly rounded value.  Returns (y, mean, rstd)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    beta = np.ascontiguousarray(beta, dtype=np.float32)
    m, h = x.shape
    mean, var_eps = layernorm_stats(x, eps)
    rstd = _rstd(var_eps, rsqrt)
    y = np.empty_like(x)
    lib().rbo_layernorm_apply_rows(_p(x), m, h, _p(mean), _p(rstd), _p(gamma), _p(beta), _DT[out_dtype], _p(y))
    return y, mean, rstd


# ------------------------------------------------------------- quantisers
def quant_dynamic_v2(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """w8a8_triton_kernels.py:41-64 on fp32 values x[M, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    lib().rbo_quant_dynamic_v2(_p(x), m, k, _p(q), _p(s))
    return q, s


def quant_static_v2(x: np.ndarray, scale: float) -> np.ndarray:
    """w8a8_triton_kernels.py:23-38 (per-tensor static scale, already widened to fp32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.shape, dtype=np.int8)
    lib().rbo_quant_static_v2(_p(x), x.size, float(np.float32(scale)), _p(q))
    return q


def quant_rows_v1(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """kernels/quantization.py:6-35 on fp32 values x[M, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    lib().rbo_quant_rows_v1(_p(x), m, k, _p(q), _p(s))
    return q, s


# ------------------------------------------------------------------- GEMM
def gemm_i8_i32(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    """int32 C = A[M,K] @ B[N,K]^T.  Uses an fp64 matmul, which is exact here:
    every product is <= 2^14 and |C| <= 2^14 * K < 2^53 for K < 2^39."""
    a64 = np.asarray(a, dtype=np.float64)
    b64 = np.asarray(b_nk, dtype=np.float64)
    return (a64 @ b64.T).astype(np.int64).astype(np.int32)


def gemm_i8_i32_loops(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    """Same as gemm_i8_i32 with plain integer loops in C (small sizes only)."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b_nk, dtype=np.int8)
    m, k = a.shape
    n = b.shape[0]
    c = np.empty((m, n), dtype=np.int32)
    lib().rbo_gemm_i8_i32(_p(a), _p(b), m, n, k, _p(c))
    return c


def scaled_epilogue(acc: np.ndarray, sa: np.ndarray, sb: np.ndarray, bias: Optional[np.ndarray],
                    out_dtype: str, sa_per_row: bool = True) -> np.ndarray:
    """w8a8_triton_kernels.py:230-246: ((f32(acc)*sa)*sb)+bias per fp32 op, stored as out_dtype.
    Returns fp32 values of the out_dtype result."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    m, n = acc.shape
    sa = np.ascontiguousarray(sa, dtype=np.float32).reshape(-1)
    sb = np.ascontiguousarray(sb, dtype=np.float32).reshape(-1)
    out = np.empty((m, n), dtype=np.float32)
    bias_p = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        bias_p = _p(bias)
    lib().rbo_scaled_epilogue(_p(acc), m, n, _p(sa), int(sa_per_row), _p(sb), bias_p, F32, _p(out))
    return round_to(out, out_dtype)


# ------------------------------------------------------- whole RepEncoder
def rep_forward(table: np.ndarray, table_dtype: str, batch: Dict[object, object], gamma: np.ndarray,
                beta: np.ndarray, eps: float = 1e-5, act_mode: str = "dynamic",
                static_scale: float = 1.0, num_slots: Optional[int] = None,
                intermediates: bool = False, threads: int = 0, rsqrt=None):
    """gather -> pool -> concat -> LayerNorm -> int8 quant for a batch dict of numpy arrays.

    ``rsqrt`` maps each row's fl(var + eps) to rstd (see layernorm_rows).
    Returns (q int8[N,H], scale fp32[N]) and, with intermediates=True, also the
    pooled and LayerNorm rows (fp32 values of the row dtype)."""
    if num_slots is None:
        num_slots = max(k for k in batch if isinstance(k, int))
    if not 1 <= num_slots <= MAX_SLOTS:
        raise ValueError(f"num_slots must be in [1, {MAX_SLOTS}], got {num_slots}")
    table = np.ascontiguousarray(table)
    vals = [np.ascontiguousarray(batch[s][0], dtype=np.int64) for s in range(1, num_slots + 1)]
    offs = [np.ascontiguousarray(batch[s][1], dtype=np.int64) for s in range(1, num_slots + 1)]
    n = len(offs[0]) - 1
    h = num_slots * 512
    vp = (ctypes.c_void_p * num_slots)(*[v.ctypes.data for v in vals])
    op = (ctypes.c_void_p * num_slots)(*[o.ctypes.data for o in offs])
    nnz = np.array([len(v) for v in vals], dtype=np.int64)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    beta = np.ascontiguousarray(beta, dtype=np.float32)
    q = np.empty((n, h), dtype=np.int8)
    scale = np.zeros(n, dtype=np.float32)
    pooled = np.empty((n, h), dtype=np.float32)
    mean = np.empty(n, dtype=np.float32)
    var_eps = np.empty(n, dtype=np.float32)
    ln = np.empty((n, h), dtype=np.float32) if intermediates else None
    if threads <= 0:
        threads = max(1, min(os.cpu_count() or 1, 64))
    L = lib()
    L.rbo_rep_pool_stats(_p(table), _DT[table_dtype], table.shape[0], vp, op, _p(nnz), num_slots, n, eps,
                         _p(pooled), _p(mean), _p(var_eps), threads)
    rstd = _rstd(var_eps, rsqrt)
    L.rbo_rep_finish(_p(pooled), _DT[table_dtype], num_slots, n, _p(mean), _p(rstd), _p(gamma), _p(beta),
                     0 if act_mode == "dynamic" else 1, float(np.float32(static_scale)), _p(q), _p(scale),
                     _p(ln) if intermediates else None, threads)
    if intermediates:
        return q, scale, pooled, ln
    return q, scale
