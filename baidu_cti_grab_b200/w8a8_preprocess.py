"""Weight preparation for the W8A8 Linear -- same interface as the reference's
quantization/w8a8_preprocess.py (QuantizedWeight, quantize_weight_per_channel,
choose_act_static_scale, artifact helpers, make_input).

``quantize_weight_per_channel`` runs on the GPU (rb_quantize_weight_per_channel)
with the reference's arithmetic (w8a8_preprocess.py:46-57): per output channel
``scale = max(amax, 1e-8) / 127`` and ``q = clamp(round_half_even(W / scale))``.
Its result keeps the reference's layout: ``qweight_t`` is the [K, N] transposed
view of a K-contiguous [N, K] int8 tensor, which the GEMM consumes without a copy.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

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
    # Stored transposed for GEMM: [K, N].
    qweight_t: torch.Tensor
    # Per-output-channel scale: [N].
    scale: torch.Tensor
    # Kept for bf16 reference comparison in benchmarks.
    fp_weight: torch.Tensor

    def to(self, device) -> "QuantizedWeight":
        return QuantizedWeight(
            qweight_t=self.qweight_t.to(device),
            scale=self.scale.to(device),
            fp_weight=self.fp_weight.to(device),
        )


@dataclass
class LinearArtifact:
    K: int
    N: int
    qweight: QuantizedWeight
    static_act_scale: torch.Tensor


def quantize_weight_per_channel(weight: torch.Tensor) -> QuantizedWeight:
    """Symmetric per-output-channel int8 quantisation of W[N, K] on the GPU."""
    assert weight.ndim == 2
    q_nk, scale = device_ops.quantize_weight_per_channel(weight)
    return QuantizedWeight(qweight_t=q_nk.t(), scale=scale.contiguous(), fp_weight=weight.contiguous())


def choose_act_static_scale(calib_x: torch.Tensor) -> torch.Tensor:
    """Calibration-time static per-tensor activation scale (w8a8_preprocess.py:60-63)."""
    scale = calib_x.float().abs().amax().clamp(min=1e-8) / 127.0
    return scale.reshape(1).contiguous()


def artifact_path(artifact_dir: Path, K: int, N: int) -> Path:
    return Path(artifact_dir) / f"linear_K={K}_N={N}.pt"


def prepare_artifacts(artifact_dir: Path, *, dtype: torch.dtype, calib_tokens: int, seed: int,
                      device: str = "cuda") -> None:
    """Random quantised artifacts that mimic a W8A8 checkpoint (w8a8_preprocess.py:70-104)."""
    artifact_dir = Path(artifact_dir)
    artifact_dir.mkdir(parents=True, exist_ok=True)
    generator = torch.Generator(device="cpu").manual_seed(seed)
    for K, N in LINEAR_KN_SHAPES:
        weight = torch.randn((N, K), generator=generator, dtype=dtype) / (K ** 0.5)
        qweight = quantize_weight_per_channel(weight.to(device))
        calib_x = torch.randn((calib_tokens, K), generator=generator, dtype=dtype)
        static_act_scale = choose_act_static_scale(calib_x)
        torch.save(
            {
                "K": K,
                "N": N,
                "qweight_t": qweight.qweight_t.cpu(),
                "weight_scale": qweight.scale.cpu(),
                "fp_weight": qweight.fp_weight.cpu(),
                "static_act_scale": static_act_scale.cpu(),
            },
            artifact_path(artifact_dir, K, N),
        )


def load_artifact(artifact_dir: Path, K: int, N: int, device: str) -> LinearArtifact:
    data = torch.load(artifact_path(artifact_dir, K, N), map_location=device)
    qweight = QuantizedWeight(
        qweight_t=data["qweight_t"].t().contiguous().t(),
        scale=data["weight_scale"].contiguous(),
        fp_weight=data["fp_weight"].contiguous(),
    )
    return LinearArtifact(K=int(data["K"]), N=int(data["N"]), qweight=qweight,
                          static_act_scale=data["static_act_scale"].contiguous())


def make_input(batch_size: int, seq_len, K: int, *, device: str, dtype: torch.dtype) -> torch.Tensor:
    """[B, K] or [B, T, K] random input (w8a8_preprocess.py:123-138)."""
    if seq_len is None:
        return torch.randn((batch_size, K), device=device, dtype=dtype)
    return torch.randn((batch_size, seq_len, K), device=device, dtype=dtype)
