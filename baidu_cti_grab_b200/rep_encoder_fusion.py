"""Unquantised LayerNorm + Linear of the concatenated RepEncoder row -- the call
surface of the reference's kernels/rep_encoder_fusion.py, on this package's
sm_100a kernels.

  cat_free_layernorm_linear  :115-162  the accuracy baseline: the 28 pooled
      slot tensors are normalised where they lie (rb_layernorm_quant_slots reads
      each slot through its own row pointer, so the [M, 14336] concatenation of
      the inputs is never built), in fp32 and in the order of ATen's CUDA
      LayerNorm; the Linear is an fp32 matmul (full fp32 products, no tf32), and
      the result is cast to the Linear's dtype.
  layernorm_linear_triton    :169-243  LayerNorm of a contiguous [M, H] row in
      x.dtype (rb_layernorm_quant, statistics in fp32), then the Linear on the
      tensor cores (rb_fp_gemm: bf16 operands through tcgen05 kind::f16, fp32
      operands through kind::tf32 as Triton's tl.dot multiplies them), fp32
      accumulation, + bias in fp32, output in x.dtype.  Tile shapes are the
      kernel's own (128 x 256 output tiles); ``block_*`` / ``group_m`` are
      accepted for call compatibility.

Both need a CUDA device and rows of whole 512-wide slots (the RepEncoder's
layout); there is no CPU path.
"""

from __future__ import annotations

import torch

from . import device_ops


def _affine(layernorm, name):
    if layernorm.weight is None or layernorm.bias is None:
        raise ValueError(f"{name} requires affine LayerNorm")
    return layernorm.weight.detach(), layernorm.bias.detach()


def cat_free_layernorm_linear(pooled_embs, layernorm, linear):
    """LayerNorm(concat(pooled_embs)) -> Linear, in fp32, without building the concatenation.

    pooled_embs: sequence of [M, 512] CUDA tensors (one per slot, any float dtype).
    Returns [M, out_features] in linear.weight.dtype."""
    if len(pooled_embs) == 0:
        raise ValueError("pooled_embs must be non-empty")
    for t in pooled_embs:
        if not t.is_cuda:
            raise RuntimeError("cat_free_layernorm_linear expects CUDA tensors")
        if t.dim() != 2 or t.shape[1] != 512 or t.shape[0] != pooled_embs[0].shape[0]:
            raise ValueError("cat_free_layernorm_linear expects [M, 512] slot tensors with one M")
    gamma, beta = _affine(layernorm, "cat_free_layernorm_linear")
    slots = [t.detach().float().contiguous() for t in pooled_embs]  # fp32, as the reference computes
    _, _, ln = device_ops.layernorm_quant_slots(slots, gamma.float(), beta.float(), layernorm.eps, act_mode="none")
    weight = linear.weight.detach().float()
    if linear.bias is None:
        out = ln @ weight.t()
    else:
        out = torch.addmm(linear.bias.detach().float(), ln, weight.t())
    return out.to(dtype=linear.weight.dtype)


def layernorm_linear_triton(x, layernorm, linear, block_m=16, block_n=16, block_k=64, group_m=8):
    """LayerNorm + Linear of a contiguous [M, H] input (H a multiple of 512), output in x.dtype."""
    if not x.is_cuda:
        raise RuntimeError("layernorm_linear_triton expects a CUDA tensor")
    if x.dim() != 2:
        raise ValueError("layernorm_linear_triton expects x as [M, H]")
    gamma, beta = _affine(layernorm, "layernorm_linear_triton")
    m, h = x.shape
    n, wh = linear.weight.shape
    if wh != h:
        raise ValueError(f"shape mismatch: x H={h}, weight H={wh}")
    if h % 512 != 0:
        raise ValueError("layernorm_linear_triton on B200 needs H to be a multiple of 512")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("layernorm_linear_triton takes bf16 or fp32 rows")
    x = x.contiguous()
    # the normalised row in x.dtype: for bf16 rows this is the reference's
    # x_norm.to(bf16) before its bf16 dot
    _, _, ln = device_ops.layernorm_quant(x, gamma, beta, layernorm.eps, act_mode="none")
    weight = linear.weight.detach().to(x.dtype).contiguous()
    bias = None if linear.bias is None else linear.bias.detach()
    out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    return device_ops.fp_gemm(ln, weight, out, bias=bias)
