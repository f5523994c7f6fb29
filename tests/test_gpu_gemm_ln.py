"""K2 with the transformer's first LayerNorm fused (rb_w8a8_gemm_ln) on the GPU.

models.py:216-217 begins layer 0 of the encoder with ``residual = x;
x = norm1[0](x)`` on the RepEncoder output.  rb_w8a8_gemm_ln returns both
(below M = 4096 from one kernel with the LayerNorm in the GEMM's epilogue,
from M = 4096 as K2 followed by a LayerNorm(512) pass over its output):
``out`` must equal rb_w8a8_gemm's result and ``ln_out`` ATen's CUDA
LayerNorm(512) of ``out``, bit for bit (and the oracle's restatement of that
LayerNorm, given the GPU's rsqrtf for rstd).
"""

import numpy as np
import pytest

from conftest import gpu_rsqrt

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,static,out_dtype", [(1, False, "bfloat16"), (100, False, "bfloat16"),
                                                (256, True, "bfloat16"), (1000, False, "float32"),
                                                (4099, False, "bfloat16"), (20000, False, "bfloat16"),
                                                (8192, True, "float32")])
def test_gemm_ln_matches_gemm_then_aten_layernorm(cuda_device, M, static, out_dtype):
    import torch
    import torch.nn.functional as F
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops

    dev = cuda_device
    K, N = 28 * 512, 512
    dt = getattr(torch, out_dtype)
    gen = torch.Generator(device=dev).manual_seed(M)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=gen)
    w = torch.randn(N, K, device=dev, generator=gen) / K ** 0.5
    w_nk, w_scale = device_ops.quantize_weight_per_channel(w)
    sa = torch.rand(1 if static else M, device=dev, generator=gen) * 9e-3 + 1e-3
    bias = (0.02 * torch.randn(N, device=dev, generator=gen)).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(N, device=dev, generator=gen)).to(dt)
    beta = (0.05 * torch.randn(N, device=dev, generator=gen)).to(dt)
    out = torch.empty((M, N), dtype=dt, device=dev)
    ln = torch.full((M, N), float("nan"), dtype=dt, device=dev)
    device_ops.w8a8_gemm_ln(a, w_nk, sa, w_scale, out, gamma, beta, 1e-5, ln, bias=bias, sa_per_row=not static)
    ref = device_ops.w8a8_gemm(a, w_nk, sa, w_scale, torch.empty((M, N), dtype=dt, device=dev), bias=bias,
                               sa_per_row=not static)
    assert torch.equal(out, ref)
    assert torch.equal(ln, F.layer_norm(ref, (N,), gamma, beta, 1e-5))
    rows = np.unique(np.linspace(0, M - 1, min(M, 64)).astype(np.int64))
    y, _, _ = O.layernorm_rows(ref[rows].float().cpu().numpy(), gamma.float().cpu().numpy(),
                               beta.float().cpu().numpy(), 1e-5, out_dtype, rsqrt=gpu_rsqrt)
    assert np.array_equal(ln[rows].float().cpu().numpy(), y)


def test_gemm_ln_rejects_other_widths(cuda_device):
    import torch
    from baidu_cti_grab_b200 import device_ops

    dev = cuda_device
    a = torch.zeros((8, 1024), dtype=torch.int8, device=dev)
    b = torch.zeros((256, 1024), dtype=torch.int8, device=dev)
    s = torch.ones(256, device=dev)
    out = torch.empty((8, 256), dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        device_ops.w8a8_gemm_ln(a, b, torch.ones(8, device=dev), s, out, s, s, 1e-5, out.clone())
