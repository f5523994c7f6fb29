"""torch-facing wrappers of the C ABI: validate tensors, pass device pointers
and the current stream, allocate outputs with torch's caching allocator.

These are the only functions in the package that call into librep_b200.so;
the reference-shaped modules (w8a8_triton_kernels, quantization,
rep_encoder_fusion, rep_encoder) are built on them.
"""

from __future__ import annotations

import ctypes
import weakref
from typing import Dict, Optional, Sequence, Tuple

import torch

from . import _lib as L

_DT = {
    torch.float32: L.RB_F32,
    torch.bfloat16: L.RB_BF16,
    torch.float16: L.RB_F16,
    torch.int32: L.RB_I32,
    torch.int8: L.RB_I8,
}


def rb_dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def require_cuda(name: str, *tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name} expects CUDA tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: tensors on different devices ({dev} vs {t.device})")
    if dev is None:
        raise RuntimeError(f"{name} expects CUDA tensors")
    return dev


# --------------------------------------------------------------- RepEncoder
_DERIVED: dict = {}


def cached_derived(src: torch.Tensor, tag: str, make):
    """``make(src)`` computed once per (tensor object, tag) and reused while the
    tensor is alive and unmodified (same storage pointer and version counter).
    Entries die with their source tensor, so a new tensor that happens to
    reuse a freed address never sees a stale value."""
    key = (id(src), tag)
    sig = (src.data_ptr(), src._version, src.dtype, tuple(src.shape), tuple(src.stride()), src.device)
    hit = _DERIVED.get(key)
    if hit is not None:
        ref, hsig, value = hit
        if ref() is src and hsig == sig:
            return value
    value = make(src)
    try:
        ref = weakref.ref(src, lambda _r, k=key: _DERIVED.pop(k, None))
    except TypeError:
        return value
    _DERIVED[key] = (ref, sig, value)
    return value


def _affine_param(t: torch.Tensor) -> torch.Tensor:
    """A LayerNorm parameter as the kernels read it: bf16, fp16 or fp32,
    contiguous (other dtypes are widened to fp32 once and cached).  16-bit
    parameters are read as they are: half the bytes of an fp32 copy."""
    if t.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return t.contiguous()
    return cached_derived(t, "affine_f32", lambda x: x.detach().float().contiguous())


def rep_gather_ln_quant(table: torch.Tensor, slot_values: Sequence[torch.Tensor],
                        slot_offsets: Sequence[torch.Tensor], gamma: torch.Tensor, beta: torch.Tensor,
                        eps: float, act_mode: str = "dynamic", static_scale: Optional[torch.Tensor] = None,
                        q_out: Optional[torch.Tensor] = None, scale_out: Optional[torch.Tensor] = None,
                        want_pooled: bool = False, want_ln: bool = False):
    """Fused gather -> pool -> concat -> LayerNorm -> int8 (rb_rep_gather_ln_quant_idx).

    Slot values and offsets are all int64 (the reference's collate output) or all
    int32 (half the bytes; ids, offsets and nnz below 2^31).
    Returns (q int8[N, S*512] or None, scale fp32[N] or None, pooled or None, ln or None)."""
    S = len(slot_values)
    dev = require_cuda("rep_gather_ln_quant", table, gamma, beta, *slot_values, *slot_offsets)
    if len(slot_offsets) != S:
        raise ValueError("slot_values and slot_offsets differ in length")
    if table.dim() != 2 or not table.is_contiguous():
        raise ValueError("table must be a contiguous [V, 512] tensor")
    n_items = int(slot_offsets[0].numel()) - 1 if S else 0
    idx_dtype = slot_offsets[0].dtype if S else torch.int64
    if idx_dtype not in (torch.int64, torch.int32):
        raise ValueError("slot values and offsets must be int64 or int32")
    for s in range(S):
        if slot_values[s].dtype != idx_dtype or slot_offsets[s].dtype != idx_dtype:
            raise ValueError("slot values and offsets must all be int64 or all int32")
        if not slot_values[s].is_contiguous() or not slot_offsets[s].is_contiguous():
            raise ValueError("slot values and offsets must be contiguous")
        if slot_offsets[s].numel() - 1 != n_items:
            raise ValueError("every slot needs offsets of length N+1")
    H = S * table.shape[1]
    mode = {"dynamic": L.RB_ACT_DYNAMIC, "static": L.RB_ACT_STATIC, "none": L.RB_ACT_NONE}[act_mode]
    q = scale = None
    if mode != L.RB_ACT_NONE:
        q = torch.empty((n_items, H), dtype=torch.int8, device=dev) if q_out is None else q_out
        if mode == L.RB_ACT_DYNAMIC:
            scale = torch.empty((n_items,), dtype=torch.float32, device=dev) if scale_out is None else scale_out
    pooled = torch.empty((n_items, H), dtype=table.dtype, device=dev) if want_pooled else None
    ln = torch.empty((n_items, H), dtype=table.dtype, device=dev) if (want_ln or mode == L.RB_ACT_NONE) else None
    gamma = _affine_param(gamma)
    beta = _affine_param(beta)
    if static_scale is not None:
        static_scale = static_scale.contiguous()
    with torch.cuda.device(dev):
        L.call("rb_rep_gather_ln_quant_idx", table.data_ptr(), rb_dtype(table), table.shape[0], table.shape[1],
               L.RB_I32 if idx_dtype == torch.int32 else L.RB_I64,
               L.ptr_array([v.data_ptr() for v in slot_values]),
               L.ptr_array([o.data_ptr() for o in slot_offsets]),
               L.i64_array([v.numel() for v in slot_values]), S, n_items,
               gamma.data_ptr(), beta.data_ptr(), rb_dtype(gamma), float(eps), mode,
               _ptr(static_scale), rb_dtype(static_scale) if static_scale is not None else 0,
               _ptr(q), H if q is None else q.stride(0), _ptr(scale), _ptr(pooled), _ptr(ln), _stream(dev))
    return q, scale, pooled, ln


def rep_gather_pool(table: torch.Tensor, slot_values: Sequence[torch.Tensor],
                    slot_offsets: Sequence[torch.Tensor], col_slot: Sequence[int], width_slots: int,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gather + sum-pool of a subset of slots into columns col_slot[j]*512 of [N, width_slots*512]."""
    S = len(slot_values)
    dev = require_cuda("rep_gather_pool", table, *slot_values, *slot_offsets)
    n_items = int(slot_offsets[0].numel()) - 1
    D = table.shape[1]
    if out is None:
        out = torch.empty((n_items, width_slots * D), dtype=table.dtype, device=dev)
    with torch.cuda.device(dev):
        L.call("rb_rep_gather_pool", table.data_ptr(), rb_dtype(table), table.shape[0], D,
               L.ptr_array([v.data_ptr() for v in slot_values]),
               L.ptr_array([o.data_ptr() for o in slot_offsets]),
               L.i64_array([v.numel() for v in slot_values]), L.i32_array(col_slot), S, n_items,
               out.data_ptr(), out.stride(0), _stream(dev))
    return out


def rep_gather_pool_scatter(table: torch.Tensor, slot_values: Sequence[torch.Tensor],
                            slot_offsets: Sequence[torch.Tensor], col_slot: Sequence[int], dest: Sequence[int],
                            dest_begin: Sequence[int], ld: int, item_shift: int = 0) -> None:
    """Gather + sum-pool of a subset of slots, item i written to the rank that owns
    it: dest[d] + (i - dest_begin[d])*ld + col_slot[j]*512 (elements) for
    dest_begin[d] <= i < dest_begin[d+1] (rb_rep_gather_pool_scatter).  ``dest``
    holds raw device addresses, local or mapped from another GPU (ipc_import).
    Items are processed from ``item_shift`` on, wrapping around."""
    S = len(slot_values)
    dev = require_cuda("rep_gather_pool_scatter", table, *slot_values, *slot_offsets)
    n_items = int(slot_offsets[0].numel()) - 1
    if len(dest) + 1 != len(dest_begin):
        raise ValueError("dest_begin needs len(dest) + 1 entries")
    with torch.cuda.device(dev):
        L.call("rb_rep_gather_pool_scatter", table.data_ptr(), rb_dtype(table), table.shape[0], table.shape[1],
               L.ptr_array([v.data_ptr() for v in slot_values]),
               L.ptr_array([o.data_ptr() for o in slot_offsets]),
               L.i64_array([v.numel() for v in slot_values]), L.i32_array(col_slot), S, n_items,
               L.ptr_array(list(dest)), L.i64_array(dest_begin), len(dest), int(ld),
               int(item_shift) if n_items else 0, _stream(dev))


def ipc_export(t: torch.Tensor):
    """(64-byte CUDA IPC handle of the allocation holding t, t's byte offset in it)."""
    require_cuda("ipc_export", t)
    handle = (ctypes.c_char * L.RB_IPC_HANDLE_BYTES)()
    off = ctypes.c_int64(0)
    with torch.cuda.device(t.device):
        L.call("rb_ipc_export", t.data_ptr(), handle, ctypes.byref(off))
    return bytes(handle), int(off.value)


def ipc_import(handle: bytes, offset: int, device: torch.device) -> int:
    """Device address, in this process, of another process's exported buffer."""
    if len(handle) != L.RB_IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle has 64 bytes")
    ptr = ctypes.c_void_p(0)
    buf = (ctypes.c_char * L.RB_IPC_HANDLE_BYTES).from_buffer_copy(handle)
    with torch.cuda.device(device):
        L.call("rb_ipc_import", buf, int(offset), ctypes.byref(ptr))
    return int(ptr.value)


def ipc_close(ptr: int, offset: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        L.call("rb_ipc_close", ptr, int(offset))


def layernorm_quant(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                    act_mode: str = "dynamic", static_scale: Optional[torch.Tensor] = None,
                    want_ln: bool = False):
    """LayerNorm (+ int8 quantisation) of dense rows x[N, S*512] (rb_layernorm_quant)."""
    dev = require_cuda("layernorm_quant", x, gamma, beta)
    if x.dim() != 2 or x.shape[1] % 512 != 0:
        raise ValueError("layernorm_quant expects x as [N, S*512]")
    if x.stride(1) != 1:
        x = x.contiguous()
    n, H = x.shape
    S = H // 512
    mode = {"dynamic": L.RB_ACT_DYNAMIC, "static": L.RB_ACT_STATIC, "none": L.RB_ACT_NONE}[act_mode]
    q = torch.empty((n, H), dtype=torch.int8, device=dev) if mode != L.RB_ACT_NONE else None
    scale = torch.empty((n,), dtype=torch.float32, device=dev) if mode == L.RB_ACT_DYNAMIC else None
    ln = torch.empty((n, H), dtype=x.dtype, device=dev) if (want_ln or mode == L.RB_ACT_NONE) else None
    gamma = _affine_param(gamma)
    beta = _affine_param(beta)
    if static_scale is not None:
        static_scale = static_scale.contiguous()
    with torch.cuda.device(dev):
        L.call("rb_layernorm_quant", x.data_ptr(), rb_dtype(x), n, S, x.stride(0), gamma.data_ptr(),
               beta.data_ptr(), rb_dtype(gamma), float(eps), mode, _ptr(static_scale),
               rb_dtype(static_scale) if static_scale is not None else 0, _ptr(q), H, _ptr(scale), _ptr(ln),
               _stream(dev))
    return q, scale, ln


def layernorm_quant_slots(slot_rows: Sequence[torch.Tensor], gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                          act_mode: str = "dynamic", static_scale: Optional[torch.Tensor] = None,
                          want_ln: bool = False):
    """LayerNorm (+ int8) of rows whose slot s is the [N, 512] view slot_rows[s] (common row stride)."""
    dev = require_cuda("layernorm_quant_slots", gamma, beta, *slot_rows)
    S = len(slot_rows)
    n = slot_rows[0].shape[0]
    ld = slot_rows[0].stride(0)
    for v in slot_rows:
        if tuple(v.shape) != (n, 512) or v.stride() != (ld, 1) or v.dtype != slot_rows[0].dtype:
            raise ValueError("slot rows must be [N, 512] views with one common row stride and dtype")
    H = S * 512
    mode = {"dynamic": L.RB_ACT_DYNAMIC, "static": L.RB_ACT_STATIC, "none": L.RB_ACT_NONE}[act_mode]
    q = torch.empty((n, H), dtype=torch.int8, device=dev) if mode != L.RB_ACT_NONE else None
    scale = torch.empty((n,), dtype=torch.float32, device=dev) if mode == L.RB_ACT_DYNAMIC else None
    ln = torch.empty((n, H), dtype=slot_rows[0].dtype, device=dev) if (want_ln or mode == L.RB_ACT_NONE) else None
    gamma = _affine_param(gamma)
    beta = _affine_param(beta)
    if static_scale is not None:
        static_scale = static_scale.contiguous()
    with torch.cuda.device(dev):
        L.call("rb_layernorm_quant_slots", L.ptr_array([v.data_ptr() for v in slot_rows]), rb_dtype(slot_rows[0]),
               n, S, ld, gamma.data_ptr(), beta.data_ptr(), rb_dtype(gamma), float(eps), mode, _ptr(static_scale),
               rb_dtype(static_scale) if static_scale is not None else 0, _ptr(q), H, _ptr(scale), _ptr(ln),
               _stream(dev))
    return q, scale, ln


# ------------------------------------------------------------- quantisers
def quant_dynamic_per_token_out(x2d: torch.Tensor, xq: torch.Tensor, scale: torch.Tensor):
    dev = require_cuda("dynamic_per_token_quantize_activation", x2d, xq, scale)
    if x2d.dim() != 2 or x2d.stride(1) != 1 or xq.stride(1) != 1:
        raise ValueError("expected 2-D row-major x and xq")
    M, K = x2d.shape
    with torch.cuda.device(dev):
        L.call("rb_quant_dynamic_per_token", x2d.data_ptr(), rb_dtype(x2d), M, K, x2d.stride(0), xq.data_ptr(),
               xq.stride(0), scale.data_ptr(), _stream(dev))
    return xq, scale


def quant_static_out(x: torch.Tensor, scale: torch.Tensor, xq: torch.Tensor) -> torch.Tensor:
    dev = require_cuda("static_quantize_activation", x, scale, xq)
    if not x.is_contiguous() or not xq.is_contiguous():
        raise ValueError("static quantisation expects contiguous tensors")
    with torch.cuda.device(dev):
        L.call("rb_quant_static", x.data_ptr(), rb_dtype(x), x.numel(), scale.data_ptr(), rb_dtype(scale),
               xq.data_ptr(), _stream(dev))
    return xq


def quant_rows_v1(x2d: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda("quantize_rows_int8", x2d)
    M, K = x2d.shape
    q = torch.empty((M, K), dtype=torch.int8, device=dev)
    s = torch.empty((M,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        L.call("rb_quant_rows_v1", x2d.data_ptr(), rb_dtype(x2d), M, K, x2d.stride(0), q.data_ptr(), K,
               s.data_ptr(), _stream(dev))
    return q, s


def quantize_weight_per_channel(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """W[N,K] -> (q int8 [N,K] K-contiguous, scale fp32 [N])."""
    dev = require_cuda("quantize_weight_per_channel", w)
    if w.dim() != 2:
        raise ValueError("expected W as [N, K]")
    if w.stride(1) != 1:
        w = w.contiguous()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=dev)
    s = torch.empty((N,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        L.call("rb_quantize_weight_per_channel", w.data_ptr(), rb_dtype(w), N, K, w.stride(0), q.data_ptr(),
               s.data_ptr(), _stream(dev))
    return q, s


def pack_weight_nk(qweight_t: torch.Tensor) -> torch.Tensor:
    """[K,N] int8 view (any strides) -> [N,K] K-contiguous int8 copy."""
    dev = require_cuda("pack_weight_nk", qweight_t)
    K, N = qweight_t.shape
    dst = torch.empty((N, K), dtype=torch.int8, device=dev)
    with torch.cuda.device(dev):
        L.call("rb_pack_weight_nk", qweight_t.data_ptr(), K, N, qweight_t.stride(0), qweight_t.stride(1),
               dst.data_ptr(), _stream(dev))
    return dst


def as_nk(qweight_t: torch.Tensor) -> torch.Tensor:
    """The K-contiguous [N,K] view of a [K,N] weight, repacking only when needed."""
    K, N = qweight_t.shape
    if qweight_t.stride(0) == 1 and qweight_t.stride(1) >= K and qweight_t.stride(1) % 16 == 0 \
            and qweight_t.data_ptr() % 16 == 0:
        return qweight_t.t()
    return pack_weight_nk(qweight_t)


# ------------------------------------------------------------------- GEMM
_WS_SIZE: Dict[Tuple[int, int, int], int] = {}
_WS: Dict[Tuple[int, int], torch.Tensor] = {}


def _workspace_elems(M: int, N: int, K: int) -> int:
    key = (M, N, K)
    n = _WS_SIZE.get(key)
    if n is None:
        n = _WS_SIZE[key] = int(L.load().rb_w8a8_gemm_workspace_size(M, N, K))
    return n


def _workspace(dev: torch.device, elems: int) -> torch.Tensor:
    """The split-K workspace of the current stream on `dev`, grown on demand.
    One buffer per (device, stream): launches on one stream run in order, so
    consecutive GEMMs on a stream can share it."""
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < elems:
        ws = _WS[key] = torch.empty((elems,), dtype=torch.int32, device=dev)
    return ws


def w8a8_gemm(a: torch.Tensor, b_nk: torch.Tensor, scale_a: Optional[torch.Tensor],
              scale_b: Optional[torch.Tensor], out: torch.Tensor, *, bias: Optional[torch.Tensor] = None,
              sa_per_row: bool = True) -> torch.Tensor:
    """out = ((f32(A @ B^T) * sa) * sb) + bias, or raw int32 when out is int32."""
    dev = require_cuda("w8a8_gemm", a, b_nk, out, scale_a, scale_b, bias)
    if a.dim() != 2 or b_nk.dim() != 2 or a.stride(1) != 1 or b_nk.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("w8a8_gemm expects row-major 2-D operands")
    M, K = a.shape
    N = b_nk.shape[0]
    if b_nk.shape[1] != K:
        raise ValueError(f"shape mismatch: A K={K}, B K={b_nk.shape[1]}")
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out must be [{M}, {N}]")
    raw = out.dtype == torch.int32
    if not raw:
        scale_a = scale_a.contiguous()
        scale_b = scale_b.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    ws_elems = _workspace_elems(M, N, K)
    ws = _workspace(dev, ws_elems) if ws_elems > 0 else None
    with torch.cuda.device(dev):
        L.call("rb_w8a8_gemm_ws", a.data_ptr(), a.stride(0), b_nk.data_ptr(), b_nk.stride(0), M, N, K,
               _ptr(scale_a), rb_dtype(scale_a) if scale_a is not None else 0, 1 if sa_per_row else 0,
               _ptr(scale_b), rb_dtype(scale_b) if scale_b is not None else 0, _ptr(bias),
               rb_dtype(bias) if bias is not None else 0, out.data_ptr(), out.stride(0), rb_dtype(out),
               _ptr(ws), ws_elems, _stream(dev))
    return out


def w8a8_gemm_ln(a: torch.Tensor, b_nk: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                 out: torch.Tensor, ln_gamma: torch.Tensor, ln_beta: torch.Tensor, eps: float, ln_out: torch.Tensor,
                 *, bias: Optional[torch.Tensor] = None, sa_per_row: bool = True):
    """out = ((f32(A @ B^T) * sa) * sb) + bias and ln_out = LayerNorm(out) over its 512
    columns (rb_w8a8_gemm_ln).  Returns (out, ln_out)."""
    dev = require_cuda("w8a8_gemm_ln", a, b_nk, out, ln_out, scale_a, scale_b, bias, ln_gamma, ln_beta)
    if a.dim() != 2 or b_nk.dim() != 2 or a.stride(1) != 1 or b_nk.stride(1) != 1 or out.stride(1) != 1 \
            or ln_out.stride(1) != 1:
        raise ValueError("w8a8_gemm_ln expects row-major 2-D operands")
    M, K = a.shape
    N = b_nk.shape[0]
    if b_nk.shape[1] != K:
        raise ValueError(f"shape mismatch: A K={K}, B K={b_nk.shape[1]}")
    if tuple(out.shape) != (M, N) or tuple(ln_out.shape) != (M, N) or ln_out.dtype != out.dtype:
        raise ValueError(f"out and ln_out must be [{M}, {N}] of one dtype")
    scale_a, scale_b = scale_a.contiguous(), scale_b.contiguous()
    bias = None if bias is None else bias.contiguous()
    ln_gamma, ln_beta = ln_gamma.contiguous(), ln_beta.contiguous()
    with torch.cuda.device(dev):
        L.call("rb_w8a8_gemm_ln", a.data_ptr(), a.stride(0), b_nk.data_ptr(), b_nk.stride(0), M, N, K,
               scale_a.data_ptr(), rb_dtype(scale_a), 1 if sa_per_row else 0, scale_b.data_ptr(), rb_dtype(scale_b),
               _ptr(bias), rb_dtype(bias) if bias is not None else 0, out.data_ptr(), out.stride(0), rb_dtype(out),
               ln_gamma.data_ptr(), ln_beta.data_ptr(), rb_dtype(ln_gamma), float(eps), ln_out.data_ptr(),
               ln_out.stride(0), _stream(dev))
    return out, ln_out


def fp_gemm(a: torch.Tensor, b_nk: torch.Tensor, out: torch.Tensor, *,
            bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = A @ B^T + bias on the tensor cores: A [M, K], B [N, K] both bf16
    (kind::f16) or both fp32 (kind::tf32), fp32 accumulation."""
    dev = require_cuda("fp_gemm", a, b_nk, out, bias)
    if a.dim() != 2 or b_nk.dim() != 2 or a.stride(1) != 1 or b_nk.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("fp_gemm expects row-major 2-D operands")
    if a.dtype != b_nk.dtype or a.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("fp_gemm operands must both be bf16 or both fp32")
    M, K = a.shape
    N = b_nk.shape[0]
    if b_nk.shape[1] != K:
        raise ValueError(f"shape mismatch: A K={K}, B K={b_nk.shape[1]}")
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out must be [{M}, {N}]")
    if bias is not None:
        bias = bias.contiguous()
    with torch.cuda.device(dev):
        L.call("rb_fp_gemm", a.data_ptr(), rb_dtype(a), a.stride(0), b_nk.data_ptr(), b_nk.stride(0), M, N, K,
               _ptr(bias), rb_dtype(bias) if bias is not None else 0, out.data_ptr(), out.stride(0), rb_dtype(out),
               _stream(dev))
    return out


_SMOE_WS: Dict[Tuple[int, int], torch.Tensor] = {}


def smoe_experts(x: torch.Tensor, topk_idx: torch.Tensor, topk_score: torch.Tensor, w1: torch.Tensor,
                 b1: Optional[torch.Tensor], w2: torch.Tensor, b2: Optional[torch.Tensor],
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The SMoE expert layer after the gate (rb_smoe_experts).

    x [T, D] bf16/f16; topk_idx [T, k] int64/int32; topk_score [T, k] in x.dtype;
    w1 [E, F, D], b1 [E, F], w2 [E, D, F], b2 [E, D] in x.dtype.
    Returns out [T, D] = sum over each token's k experts of
    score * (relu(x W1^T + b1) W2^T + b2)."""
    dev = require_cuda("smoe_experts", x, topk_idx, topk_score, w1, b1, w2, b2, out)
    if x.dim() != 2 or topk_idx.dim() != 2 or topk_score.shape != topk_idx.shape:
        raise ValueError("smoe_experts expects x [T, D] and topk_idx/topk_score [T, k]")
    T, D = x.shape
    k = topk_idx.shape[1]
    if topk_idx.shape[0] != T:
        raise ValueError("topk_idx must have one row per token")
    if w1.dim() != 3 or w2.dim() != 3 or w1.shape[2] != D or w2.shape[1] != D or w2.shape[0] != w1.shape[0] \
            or w2.shape[2] != w1.shape[1]:
        raise ValueError("w1 must be [E, F, D] and w2 [E, D, F]")
    E, F = w1.shape[0], w1.shape[1]
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("smoe_experts takes bf16 or f16 activations")
    if topk_idx.dtype not in (torch.int64, torch.int32):
        raise ValueError("topk_idx must be int64 or int32")
    if any(t is not None and t.dtype != x.dtype for t in (topk_score, w1, b1, w2, b2)):
        raise ValueError("scores, weights and biases must share x's dtype")
    if x.stride(1) != 1:
        x = x.contiguous()
    topk_idx, topk_score = topk_idx.contiguous(), topk_score.contiguous()
    w1, w2 = w1.contiguous(), w2.contiguous()
    b1 = None if b1 is None else b1.contiguous()
    b2 = None if b2 is None else b2.contiguous()
    if out is None:
        out = torch.empty((T, D), dtype=x.dtype, device=dev)
    elif tuple(out.shape) != (T, D) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be a row-major [{T}, {D}] {x.dtype} tensor")
    lib = L.load()
    idt = L.RB_I64 if topk_idx.dtype == torch.int64 else L.RB_I32
    need = int(lib.rb_smoe_workspace_size(T, k, E, D, F, rb_dtype(x)))
    if need < 0:
        raise ValueError("rb_smoe_workspace_size rejected the shape")
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _SMOE_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = _SMOE_WS[key] = torch.empty((max(need, 256),), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        L.call("rb_smoe_experts", x.data_ptr(), rb_dtype(x), x.stride(0), T, D, topk_idx.data_ptr(), idt,
               topk_score.data_ptr(), k, E, w1.data_ptr(), _ptr(b1), w2.data_ptr(), _ptr(b2), F, ws.data_ptr(),
               ws.numel(), out.data_ptr(), out.stride(0), _stream(dev))
    return out


def device_error(reset: bool = False) -> int:
    return L.device_error(reset)


def selftest_wait_timeout(budget_ns: int, device=None) -> None:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        L.call("rb_selftest_wait_timeout", int(budget_ns), _stream(dev))
