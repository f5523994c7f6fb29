"""The reference's RepEncoder W8A8 path restated with torch CPU operators.

TEST / BASELINE INFRASTRUCTURE ONLY: used by bench.py's CPU-baseline leg and
its ``--impl reference`` arm to time the reference's algorithm on the host
cores.  It is never imported by the product package.

models.py:24-48 (torch fuse mode): per slot ``values.clamp(0, V-1)`` and
``F.embedding_bag(..., offsets[:-1], mode='sum', padding_idx=0)``, then
``torch.cat`` and ``F.layer_norm`` -- the ATen CPU kernels the reference runs
on CPU.  The W8A8 tail follows quantization/w8a8_triton_kernels.py:56-64
(dynamic per-token quantiser, round half away from zero) and :230-246
(``((acc*sa)*sb)+bias``) with ``torch._int_mm`` as the int8 GEMM.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rep_forward_cpu(table: torch.Tensor, values, offsets, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                    w_nk: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """One RepEncoder W8A8 forward on CPU tensors; returns [N, out] in table dtype."""
    V = table.shape[0]
    pooled = []
    for v, o in zip(values, offsets):
        pooled.append(F.embedding_bag(v.clamp(0, V - 1), table, o[:-1], mode="sum", padding_idx=0))
    x = torch.cat(pooled, dim=1)
    y = F.layer_norm(x, (x.shape[1],), gamma, beta, eps)
    yf = y.float()
    amax = yf.abs().amax(dim=1).clamp(min=1e-8)
    inv = 127.0 / amax
    t = yf * inv[:, None]
    q = (torch.sign(t) * torch.floor(t.abs() + 0.5)).clamp(-128, 127).to(torch.int8)
    acc = torch._int_mm(q, w_nk.t())
    out = (acc.float() * (amax / 127.0)[:, None]) * w_scale[None, :] + bias.float()[None, :]
    return out.to(table.dtype)
