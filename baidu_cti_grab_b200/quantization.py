"""Dynamic W8A8 Linear (first version of the reference's kernels) on B200 --
same call surface as the reference's kernels/quantization.py.

Replaced entry points (reference file:line):
  quantize_rows_int8_triton            :243-268  (_quantize_rows_int8_kernel :6-35)
  quantize_weight_per_channel_int8     :271-273
  quantize_activation_per_token_int8   :276-278
  w8a8_linear_triton_dynamic_unfused   :281-348  (_w8a8_matmul_kernel :38-105)
  w8a8_linear_triton_dynamic_fused     :351-404  (_w8a8_dynamic_fused_kernel :108-188)
  w8a8_linear_dynamic                  :407-408
  bf16_linear / max_abs_diff / mean_abs_diff  :411-424  (bf16_linear on rb_fp_gemm)

This version rounds with ``trunc(x/scale +- 0.5)`` into [-127, 127] and takes
the weight as W[N, K] (already K-contiguous).  The reference's "fused" kernel
re-quantises each activation tile in registers for every output tile; here
both variants quantise each row once (rb_quant_rows_v1) and run the tcgen05
GEMM -- the arithmetic, and therefore every output bit, is the same.  The
``block_*``/``group_m``/``autotune`` arguments are accepted for call
compatibility; tile shapes are chosen by the kernel.
"""

from __future__ import annotations

import torch

from . import device_ops


def quantize_rows_int8_triton(x):
    if not x.is_cuda:
        raise RuntimeError("quantize_rows_int8_triton expects a CUDA tensor")
    if x.dim() != 2:
        raise ValueError("quantize_rows_int8_triton expects [rows, cols]")
    x = x.contiguous()
    return device_ops.quant_rows_v1(x)


def quantize_weight_per_channel_int8(weight):
    """A Linear weight [N, K] quantised row by row (one scale per output channel)."""
    return quantize_rows_int8_triton(weight)


def quantize_activation_per_token_int8(x):
    """Activations [M, K] quantised row by row (one scale per token)."""
    return quantize_rows_int8_triton(x)


def _check_linear_args(name, x, weight_int8):
    if not x.is_cuda:
        raise RuntimeError(f"{name} expects CUDA tensors")
    if x.dim() != 2 or weight_int8.dim() != 2:
        raise ValueError("expected x [M,K] and weight_int8 [N,K]")
    m, k = x.shape
    n, wk = weight_int8.shape
    if wk != k:
        raise ValueError(f"shape mismatch: x K={k}, weight K={wk}")
    return m, n


def _linear_v1(name, x, weight_int8, weight_scale, bias, out_dtype):
    m, n = _check_linear_args(name, x, weight_int8)
    x = x.contiguous()
    weight_int8 = weight_int8.contiguous()
    weight_scale = weight_scale.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    x_int8, x_scale = device_ops.quant_rows_v1(x)
    out = torch.empty((m, n), device=x.device, dtype=out_dtype)
    return device_ops.w8a8_gemm(x_int8, weight_int8, x_scale, weight_scale, out, bias=bias, sa_per_row=True)


def w8a8_linear_triton_dynamic_unfused(x, weight_int8, weight_scale, bias=None, out_dtype=torch.bfloat16,
                                       block_m=32, block_n=64, block_k=64, group_m=8, autotune=False):
    """x [M, K] (float) -> [M, N] out_dtype: rows quantised once (rb_quant_rows_v1),
    then the tcgen05 int8 GEMM with acc * x_scale[m] * weight_scale[n] + bias[n];
    weight_int8 is [N, K], weight_scale [N] fp32, bias [N] or None."""
    return _linear_v1("w8a8_linear_triton_dynamic_unfused", x, weight_int8, weight_scale, bias, out_dtype)


def w8a8_linear_triton_dynamic_fused(x, weight_int8, weight_scale, bias=None, out_dtype=torch.bfloat16,
                                     block_m=32, block_n=64, block_k=64, group_m=8):
    """The reference's single-kernel variant: same arguments and the same output
    bits as the two-kernel one, which this library runs for both (each row is
    quantised once instead of once per output tile)."""
    return _linear_v1("w8a8_linear_triton_dynamic_fused", x, weight_int8, weight_scale, bias, out_dtype)


def w8a8_linear_dynamic(*args, **kwargs):
    return w8a8_linear_triton_dynamic_fused(*args, **kwargs)


def bf16_linear(x, weight, bias=None):
    """The bf16 Linear the W8A8 path is compared with: x [..., K] and W [N, K] in
    bf16 on the tcgen05 kind::f16 GEMM (fp32 accumulation), output bf16."""
    if not x.is_cuda:
        raise RuntimeError("bf16_linear expects CUDA tensors")
    x2 = x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous()
    w = weight.to(torch.bfloat16).contiguous()
    out = torch.empty((x2.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    device_ops.fp_gemm(x2, w, out, bias=None if bias is None else bias.to(torch.bfloat16))
    return out.view(*x.shape[:-1], w.shape[0])


def max_abs_diff(a, b):
    return (a.float() - b.float()).abs().max().item()


def mean_abs_diff(a, b):
    return (a.float() - b.float()).abs().mean().item()
