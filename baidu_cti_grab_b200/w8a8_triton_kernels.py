"""W8A8 int8 Linear on B200 -- same call surface as the reference's
quantization/w8a8_triton_kernels.py, backed by hand-written sm_100a kernels.

Replaced entry points (reference file:line):
  flatten_input                                 :321-323
  quant_backend_name / quant_backend_error      :330-339
  static_quantize_activation[_out]              :375-389  (_static_quant_kernel :23-38)
  dynamic_per_token_quantize_activation[_out]   :392-422  (_dynamic_per_token_quant_kernel :41-64)
  quantize_activation[_out]                     :425-460
  w8a8_scaled_mm[_out]                          :470-564  (_w8a8_scaled_mm[_nomask]_kernel :174-318)
  int8_mm_no_scale[_out]                        :567-640  (_int8_mm_no_scale[_nomask]_kernel :67-171)
  w8a8_linear                                   :643-670

The GEMM is rb_w8a8_gemm (tcgen05 kind::i8, int32 accumulator in TMEM, the
dequant/bias epilogue fused).  It needs the weight K-contiguous: a
``qweight_t`` that is the transposed view of an [N, K] tensor is used as is,
a row-major [K, N] buffer (the quantised checkpoint layout) is repacked once
and cached for as long as that tensor object lives unmodified.
"""

from __future__ import annotations

import torch

from . import _lib, device_ops
from .w8a8_preprocess import QuantizedWeight


def flatten_input(x: torch.Tensor):
    """(x as a contiguous 2-D [rows, K] view, the leading dimensions to restore afterwards)."""
    return x.contiguous().view(-1, x.shape[-1]), x.shape[:-1]


def quant_backend_name() -> str:
    return "cuda_sm100a"


def quant_backend_error():
    return _lib.load_error_message()


def _packed_nk(qweight_t: torch.Tensor) -> torch.Tensor:
    """K-contiguous [N, K] int8 view/copy of qweight_t [K, N]."""
    K, N = qweight_t.shape
    if qweight_t.stride(0) == 1 and qweight_t.stride(1) % 16 == 0 and qweight_t.stride(1) >= K \
            and qweight_t.data_ptr() % 16 == 0:
        return qweight_t.t()
    return device_ops.cached_derived(qweight_t, "packed_nk", device_ops.pack_weight_nk)


def static_quantize_activation_out(x_2d: torch.Tensor, scale: torch.Tensor, xq: torch.Tensor) -> torch.Tensor:
    return device_ops.quant_static_out(x_2d, scale, xq)


def static_quantize_activation(x_2d: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    xq = torch.empty_like(x_2d, dtype=torch.int8)
    return static_quantize_activation_out(x_2d, scale, xq)


def dynamic_per_token_quantize_activation_out(x_2d: torch.Tensor, xq: torch.Tensor, scale: torch.Tensor):
    return device_ops.quant_dynamic_per_token_out(x_2d, xq, scale)


def dynamic_per_token_quantize_activation(x_2d: torch.Tensor):
    M, _ = x_2d.shape
    xq = torch.empty_like(x_2d, dtype=torch.int8)
    scale = torch.empty((M,), device=x_2d.device, dtype=torch.float32)
    return dynamic_per_token_quantize_activation_out(x_2d, xq, scale)


def quantize_activation_out(x_2d: torch.Tensor, xq: torch.Tensor, scale_out: torch.Tensor, *, act_mode: str,
                            static_act_scale: torch.Tensor | None = None):
    assert act_mode in {"static", "dynamic"}
    if act_mode == "static":
        assert static_act_scale is not None
        return static_quantize_activation_out(x_2d, static_act_scale, xq), static_act_scale
    return dynamic_per_token_quantize_activation_out(x_2d, xq, scale_out)


def quantize_activation(x_2d: torch.Tensor, *, act_mode: str, static_act_scale: torch.Tensor | None = None):
    assert act_mode in {"static", "dynamic"}
    if act_mode == "static":
        assert static_act_scale is not None
        return static_quantize_activation(x_2d, static_act_scale), static_act_scale
    return dynamic_per_token_quantize_activation(x_2d)


def w8a8_scaled_mm_out(xq_2d: torch.Tensor, qweight: QuantizedWeight, scale_a: torch.Tensor,
                       out_2d: torch.Tensor, *, bias: torch.Tensor | None = None, static_act: bool) -> torch.Tensor:
    assert xq_2d.ndim == 2
    K = xq_2d.shape[1]
    assert K == qweight.qweight_t.shape[0]
    M = xq_2d.shape[0]
    N = qweight.qweight_t.shape[1]
    assert out_2d.shape == (M, N)
    if xq_2d.stride(1) != 1:
        xq_2d = xq_2d.contiguous()
    return device_ops.w8a8_gemm(xq_2d, _packed_nk(qweight.qweight_t), scale_a, qweight.scale, out_2d,
                                bias=bias, sa_per_row=not static_act)


def w8a8_scaled_mm(xq_2d: torch.Tensor, qweight: QuantizedWeight, scale_a: torch.Tensor, *,
                   bias: torch.Tensor | None = None, out_dtype: torch.dtype, static_act: bool) -> torch.Tensor:
    """int8 A x the quantised weight on the tcgen05 GEMM, with the fp32 scale / bias epilogue fused."""
    assert xq_2d.ndim == 2
    K = xq_2d.shape[1]
    assert K == qweight.qweight_t.shape[0]
    M = xq_2d.shape[0]
    N = qweight.qweight_t.shape[1]
    out_2d = torch.empty((M, N), device=xq_2d.device, dtype=out_dtype)
    return w8a8_scaled_mm_out(xq_2d, qweight, scale_a, out_2d, bias=bias, static_act=static_act)


def int8_mm_no_scale_out(xq_2d: torch.Tensor, qweight: QuantizedWeight, out_2d: torch.Tensor) -> torch.Tensor:
    assert xq_2d.ndim == 2
    K = xq_2d.shape[1]
    assert K == qweight.qweight_t.shape[0]
    M = xq_2d.shape[0]
    N = qweight.qweight_t.shape[1]
    assert out_2d.shape == (M, N)
    if xq_2d.stride(1) != 1:
        xq_2d = xq_2d.contiguous()
    if out_2d.dtype == torch.int32 and out_2d.stride(1) == 1:
        return device_ops.w8a8_gemm(xq_2d, _packed_nk(qweight.qweight_t), None, None, out_2d)
    acc = device_ops.w8a8_gemm(xq_2d, _packed_nk(qweight.qweight_t), None, None,
                               torch.empty((M, N), dtype=torch.int32, device=xq_2d.device))
    out_2d.copy_(acc)
    return out_2d


def int8_mm_no_scale(xq_2d: torch.Tensor, qweight: QuantizedWeight, *, out_dtype: torch.dtype) -> torch.Tensor:
    """Raw int32 accumulators of int8 A x the quantised weight (no scales, no bias)."""
    assert xq_2d.ndim == 2
    K = xq_2d.shape[1]
    assert K == qweight.qweight_t.shape[0]
    M = xq_2d.shape[0]
    N = qweight.qweight_t.shape[1]
    out_2d = torch.empty((M, N), device=xq_2d.device, dtype=out_dtype)
    return int8_mm_no_scale_out(xq_2d, qweight, out_2d)


def w8a8_linear(x: torch.Tensor, qweight: QuantizedWeight, *, bias: torch.Tensor | None = None, act_mode: str,
                static_act_scale: torch.Tensor | None = None) -> torch.Tensor:
    """y = W8A8 Linear(x) for x of shape [..., K]: quantise the activations (static
    per-tensor or dynamic per-token), int8 GEMM, fp32 epilogue, y in x.dtype."""
    assert x.shape[-1] == qweight.qweight_t.shape[0]
    x_2d, original_batch_shape = flatten_input(x)
    xq, scale_a = quantize_activation(x_2d, act_mode=act_mode, static_act_scale=static_act_scale)
    out_2d = w8a8_scaled_mm(xq, qweight, scale_a, bias=bias, out_dtype=x.dtype,
                            static_act=(act_mode == "static"))
    return out_2d.view(*original_batch_shape, qweight.qweight_t.shape[1])
