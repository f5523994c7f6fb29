"""Unquantised LayerNorm + Linear of the concatenated RepEncoder row -- same call
surface as the reference's kernels/rep_encoder_fusion.py.

  cat_free_layernorm_linear  :115-162  fp32 LayerNorm + Linear that never
                                       concatenates the pooled slots (the
                                       reference's accuracy baseline; torch ops
                                       on the pooled tensors' device).
  layernorm_linear_triton    :169-243  LayerNorm (rb_layernorm_quant without
                                       quantisation: fp32 statistics, output in
                                       x.dtype) followed by the Linear.

The Linear of the unquantised path is a plain library GEMM (cuBLAS through
torch); the quantised path of the RepEncoder is the hand-written tcgen05 GEMM.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import device_ops


def cat_free_layernorm_linear(pooled_embs, layernorm, linear):
    """cat + LayerNorm + Linear without materialising the concatenation (fp32)."""
    if not pooled_embs:
        raise ValueError("pooled_embs must be non-empty")
    rows = pooled_embs[0].shape[0]
    device = pooled_embs[0].device
    total_dim = sum(x.shape[1] for x in pooled_embs)
    acc_dtype = torch.float32
    sum_x = torch.zeros(rows, device=device, dtype=acc_dtype)
    sum_x2 = torch.zeros(rows, device=device, dtype=acc_dtype)
    for x in pooled_embs:
        xf = x.float()
        sum_x += xf.sum(dim=1)
        sum_x2 += (xf * xf).sum(dim=1)
    mean = sum_x / total_dim
    var = torch.clamp(sum_x2 / total_dim - mean * mean, min=0.0)
    rstd = torch.rsqrt(var + layernorm.eps)
    if linear.bias is None:
        out = torch.zeros(rows, linear.out_features, device=device, dtype=acc_dtype)
    else:
        out = linear.bias.float().expand(rows, -1).clone()
    ln_weight = layernorm.weight.float() if layernorm.weight is not None else None
    ln_bias = layernorm.bias.float() if layernorm.bias is not None else None
    linear_weight = linear.weight.float()
    col_start = 0
    for x in pooled_embs:
        col_end = col_start + x.shape[1]
        x_norm = (x.float() - mean[:, None]) * rstd[:, None]
        if ln_weight is not None:
            x_norm = x_norm * ln_weight[col_start:col_end]
        if ln_bias is not None:
            x_norm = x_norm + ln_bias[col_start:col_end]
        out += x_norm @ linear_weight[:, col_start:col_end].t()
        col_start = col_end
    return out.to(dtype=linear.weight.dtype)


def layernorm_linear_triton(x, layernorm, linear, block_m=16, block_n=16, block_k=64, group_m=8):
    """LayerNorm + Linear for a contiguous [M, H] input (H a multiple of 512)."""
    if not x.is_cuda:
        raise RuntimeError("layernorm_linear_triton expects a CUDA tensor")
    if x.dim() != 2:
        raise ValueError("layernorm_linear_triton expects x as [M, H]")
    if layernorm.weight is None or layernorm.bias is None:
        raise ValueError("layernorm_linear_triton requires affine LayerNorm")
    m, h = x.shape
    n, wh = linear.weight.shape
    if wh != h:
        raise ValueError(f"shape mismatch: x H={h}, weight H={wh}")
    if h % 512 != 0:
        raise ValueError("layernorm_linear_triton on B200 needs H to be a multiple of 512")
    x = x.contiguous()
    _, _, ln = device_ops.layernorm_quant(x, layernorm.weight, layernorm.bias, layernorm.eps, act_mode="none")
    bias = None if linear.bias is None else linear.bias.to(x.dtype)
    return F.linear(ln, linear.weight.to(x.dtype), bias)
