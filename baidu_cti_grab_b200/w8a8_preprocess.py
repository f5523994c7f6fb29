"""Weight preparation for the W8A8 Linear -- the reference's
quantization/w8a8_preprocess.py interface that its GEMM path consumes
(QuantizedWeight, quantize_weight_per_channel, LINEAR_KN_SHAPES).  The
reference's benchmark scaffolding in that file (random artifact files, their
loader, a random-input maker, the calibration-time scale chooser) is not part
of the inference path and is not provided.

``quantize_weight_per_channel`` runs on the GPU (rb_quantize_weight_per_channel)
with the reference's arithmetic (w8a8_preprocess.py:46-57): per output channel
``scale = max(amax, 1e-8) / 127`` and ``q = clamp(round_half_even(W / scale))``.
Its result keeps the reference's layout: ``qweight_t`` is the [K, N] transposed
view of a K-contiguous [N, K] int8 tensor, which the GEMM consumes without a copy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import device_ops

# (K, N): X[M, K] @ W[N, K].T -> Y[M, N]   (w8a8_preprocess.py:12-18)
LINEAR_KN_SHAPES = [
    (512, 1536),
    (512, 512),
    (512, 1024),
    (1024, 512),
    (14336, 512),
]


@dataclass
class QuantizedWeight:
    """An int8 weight as the GEMM reads it.  Field names and shapes are the
    reference's (checkpoints and callers bind to them)."""

    qweight_t: torch.Tensor  # int8 [K, N]: K-contiguous storage is used in place, other layouts are repacked
    scale: torch.Tensor  # per output channel [N], fp32 (or the model dtype after model.to)
    fp_weight: torch.Tensor  # the unquantised [N, K] source weight, for accuracy comparisons

    def to(self, device) -> "QuantizedWeight":
        return QuantizedWeight(
            qweight_t=self.qweight_t.to(device),
            scale=self.scale.to(device),
            fp_weight=self.fp_weight.to(device),
        )


def quantize_weight_per_channel(weight: torch.Tensor) -> QuantizedWeight:
    """Symmetric per-output-channel int8 quantisation of W[N, K] on the GPU."""
    assert weight.ndim == 2
    q_nk, scale = device_ops.quantize_weight_per_channel(weight)
    return QuantizedWeight(qweight_t=q_nk.t(), scale=scale.contiguous(), fp_weight=weight.contiguous())
