"""SMoE layer of the reference's TransformerEncoder (models.py:96-178) on
this package's grouped expert kernels (rb_smoe_experts).

``smoe_forward(moe, x)`` works on the reference's own ``SMoE`` module: its
``gate`` (TopKGate: Linear, softmax, top-k) runs unchanged, the experts run
as one route + two grouped tcgen05 GEMMs + combine, and the load-balancing
loss is the reference's formula on the gate probabilities.  Nothing is read
back to the host (the reference reads ``counts.max()`` to size its padded
expert block, models.py:160).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import device_ops


def _expert_weight(layer: nn.Module, dtype: torch.dtype) -> torch.Tensor:
    """[out, in] weight of an expert Linear in `dtype`: nn.Linear's own weight,
    or for the reference's quantised layer (use_quant) the dequantised
    ``qweight_t.to(dtype) * weight_scale`` that its SMoE stacks
    (models.py:112-115), transposed back to [out, in]."""
    if getattr(layer, "use_quant", False):
        return (layer.qweight_t.to(dtype) * layer.weight_scale).t()
    return layer.weight.to(dtype)


def stacked_expert_params(moe: nn.Module, dtype: torch.dtype):
    """(w1 [E, F, D], b1 [E, F], w2 [E, D, F], b2 [E, D]) of moe.experts in
    `dtype`, cached on the module until a weight changes (same tensors, same
    version counters)."""
    experts = list(moe.experts)
    sig = tuple((id(t), t._version) for ex in experts for lin in (ex.fc1, ex.fc2)
                for t in (getattr(lin, "qweight_t", None) if getattr(lin, "use_quant", False) else lin.weight,
                          lin.bias) if t is not None) + (dtype,)
    cache = getattr(moe, "_b200_stacked", None)
    if cache is not None and cache[0] == sig:
        return cache[1]
    with torch.no_grad():
        w1 = torch.stack([_expert_weight(ex.fc1, dtype) for ex in experts]).contiguous()
        w2 = torch.stack([_expert_weight(ex.fc2, dtype) for ex in experts]).contiguous()
        b1 = None if experts[0].fc1.bias is None else torch.stack([ex.fc1.bias.to(dtype) for ex in experts]).contiguous()
        b2 = None if experts[0].fc2.bias is None else torch.stack([ex.fc2.bias.to(dtype) for ex in experts]).contiguous()
    params = (w1, b1, w2, b2)
    moe._b200_stacked = (sig, params)
    return params


def smoe_forward(moe: nn.Module, x: torch.Tensor):
    """SMoE.forward (models.py:131-178) for x [B, S, D] in bf16/f16 on a CUDA
    device.  Returns (out [B, S, D], moe_loss) like the reference."""
    if not x.is_cuda:
        raise RuntimeError("the b200 SMoE path expects a CUDA tensor")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the b200 SMoE path takes bf16 or f16 activations")
    B, S, D = x.shape
    topk_idx, topk_score, probs = moe.gate(x)
    w1, b1, w2, b2 = stacked_expert_params(moe, x.dtype)
    k = topk_idx.shape[-1]
    out = device_ops.smoe_experts(x.reshape(-1, D), topk_idx.reshape(-1, k), topk_score.reshape(-1, k).to(x.dtype),
                                  w1, b1, w2, b2)
    importance = probs.sum(dim=(0, 1))
    moe_loss = importance.std() / (importance.mean() + 1e-6)
    return out.view(B, S, D), moe_loss
