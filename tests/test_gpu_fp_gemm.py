"""The unquantised Linear (rb_fp_gemm: tcgen05 kind::f16 / kind::tf32), the
reference's LayerNorm + Linear entry points built on it, and the first-version
dynamic W8A8 entry points, on the GPU.

Floating-point sums: rb_fp_gemm is compared with a float64 matmul of the same
operands.  Tolerances (stated per test): bf16 operands are exact in fp32, so
the only errors are the fp32 accumulation (|err| <= K * 2^-23 * sum|a*b|, far
below a bf16 ulp here) and the final rounding to the output dtype; tf32
rounds each operand to 10 mantissa bits (relative 2^-11 per product).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref64(torch, a, b, bias):
    r = a.double() @ b.double().t()
    return r if bias is None else r + bias.double()


@pytest.mark.parametrize("M,N,K", [(1, 512, 14336), (100, 512, 14336), (300, 48, 592), (1000, 300, 1024),
                                   (4096, 512, 14336), (257, 1030, 520), (128, 256, 64)])
@pytest.mark.parametrize("out_dtype", ["bfloat16", "float32"])
def test_fp_gemm_bf16(cuda_device, M, N, K, out_dtype):
    """bf16 x bf16 -> fp32 accumulators (+ bias): within half a bf16 ulp (+ the
    fp32 accumulation bound) of the float64 product of the same operands."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    gen = torch.Generator(device=cuda_device).manual_seed(M * 31 + N * 7 + K)
    a = (torch.randn(M, K, device=cuda_device, generator=gen) * 0.5).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda_device, generator=gen) / K ** 0.5).to(torch.bfloat16)
    bias = (0.02 * torch.randn(N, device=cuda_device, generator=gen)).to(torch.bfloat16)
    odt = getattr(torch, out_dtype)
    out = device_ops.fp_gemm(a, b, torch.empty((M, N), dtype=odt, device=cuda_device), bias=bias)
    ref = _ref64(torch, a, b, bias)
    accum = K * 2.0 ** -23 * (a.double().abs() @ b.double().abs().t())
    rnd = ref.abs() * (2.0 ** -8 if odt == torch.bfloat16 else 2.0 ** -24)
    assert torch.all((out.double() - ref).abs() <= rnd + accum + 1e-30)


@pytest.mark.parametrize("M,N,K", [(64, 512, 14336), (1000, 300, 1024), (130, 48, 36)])
def test_fp_gemm_tf32(cuda_device, M, N, K):
    """fp32 operands through kind::tf32: rel-L2 <= 2e-3 of the float64 product
    (operands rounded to 10 mantissa bits), and exact on operands that are
    already tf32 values (small integers)."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    gen = torch.Generator(device=cuda_device).manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda_device, generator=gen)
    b = torch.randn(N, K, device=cuda_device, generator=gen) / K ** 0.5
    bias = 0.02 * torch.randn(N, device=cuda_device, generator=gen)
    out = device_ops.fp_gemm(a, b, torch.empty((M, N), dtype=torch.float32, device=cuda_device), bias=bias)
    ref = _ref64(torch, a, b, bias)
    assert float((out.double() - ref).norm() / ref.norm()) <= 2e-3
    ai = torch.randint(-8, 9, (M, K), device=cuda_device, generator=gen).float()
    bi = torch.randint(-8, 9, (N, K), device=cuda_device, generator=gen).float()
    outi = device_ops.fp_gemm(ai, bi, torch.empty((M, N), dtype=torch.float32, device=cuda_device))
    assert torch.equal(outi.double(), ai.double() @ bi.double().t())


def test_fp_gemm_unaligned_takes_cuda_core_path(cuda_device):
    """K not a multiple of 8 (bf16 rows not 16-byte pitched): the CUDA-core kernel, same tolerance."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    M, N, K = 33, 70, 45
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    a = torch.randn(M, K, device=cuda_device, generator=gen).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device, generator=gen).to(torch.bfloat16)
    out = device_ops.fp_gemm(a, b, torch.empty((M, N), dtype=torch.float32, device=cuda_device))
    ref = _ref64(torch, a, b, None)
    assert torch.all((out.double() - ref).abs() <= K * 2.0 ** -23 * (a.double().abs() @ b.double().abs().t()))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_layernorm_linear_triton(cuda_device, dtype):
    """LayerNorm rows bit-exact against ATen's CUDA LayerNorm in x.dtype; the
    Linear within the fp_gemm tolerance of a float64 product of those rows; the
    whole output within rel-L2 1e-2 (bf16) / 2e-3 (fp32) of the fp32 LayerNorm + Linear."""
    import torch
    import torch.nn.functional as F
    from baidu_cti_grab_b200 import device_ops
    from baidu_cti_grab_b200.rep_encoder_fusion import layernorm_linear_triton

    dt = getattr(torch, dtype)
    M, H, N = 777, 28 * 512, 512
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    x = (0.04 * torch.randn(M, H, device=cuda_device, generator=gen)).to(dt)
    ln_mod = torch.nn.LayerNorm(H).to(cuda_device, dt)
    lin = torch.nn.Linear(H, N).to(cuda_device, dt)
    with torch.no_grad():
        ln_mod.weight.copy_(1 + 0.1 * torch.randn(H, device=cuda_device, generator=gen))
        ln_mod.bias.copy_(0.05 * torch.randn(H, device=cuda_device, generator=gen))
    out = layernorm_linear_triton(x, ln_mod, lin)
    assert out.dtype == dt and out.shape == (M, N)
    with torch.no_grad():
        ln = F.layer_norm(x, (H,), ln_mod.weight, ln_mod.bias, ln_mod.eps)
        _, _, ln_k = device_ops.layernorm_quant(x, ln_mod.weight, ln_mod.bias, ln_mod.eps, act_mode="none")
        assert torch.equal(ln, ln_k)
        ref = _ref64(torch, ln, lin.weight, lin.bias)
        if dt == torch.bfloat16:
            accum = H * 2.0 ** -23 * (ln.double().abs() @ lin.weight.double().abs().t())
            assert torch.all((out.double() - ref).abs() <= ref.abs() * 2.0 ** -8 + accum + 1e-30)
        ref32 = F.linear(F.layer_norm(x.float(), (H,), ln_mod.weight.float(), ln_mod.bias.float(), ln_mod.eps),
                         lin.weight.float(), lin.bias.float())
        rel = float((out.float() - ref32).norm() / ref32.norm())
        assert rel <= (1e-2 if dt == torch.bfloat16 else 2e-3)


def test_cat_free_layernorm_linear(cuda_device):
    """Slot tensors normalised in place == ATen's fp32 LayerNorm of their
    concatenation; the fp32 Linear of it within fp32 rounding of torch's."""
    import torch
    import torch.nn.functional as F
    from baidu_cti_grab_b200.rep_encoder_fusion import cat_free_layernorm_linear

    M, S = 300, 28
    gen = torch.Generator(device=cuda_device).manual_seed(12)
    slots = [(0.03 * torch.randn(M, 512, device=cuda_device, generator=gen)).to(torch.bfloat16) for _ in range(S)]
    ln_mod = torch.nn.LayerNorm(S * 512).to(cuda_device)
    lin = torch.nn.Linear(S * 512, 512).to(cuda_device)
    with torch.no_grad():
        ln_mod.weight.copy_(1 + 0.1 * torch.randn(S * 512, device=cuda_device, generator=gen))
        out = cat_free_layernorm_linear(slots, ln_mod, lin)
        x = torch.cat([s.float() for s in slots], dim=1)
        ref = F.linear(F.layer_norm(x, (S * 512,), ln_mod.weight, ln_mod.bias, ln_mod.eps), lin.weight, lin.bias)
    assert out.dtype == torch.float32
    assert float((out - ref).abs().max()) <= 1e-5 * float(ref.abs().max())


@pytest.mark.parametrize("variant", ["w8a8_linear_triton_dynamic_unfused", "w8a8_linear_triton_dynamic_fused",
                                     "w8a8_linear_dynamic"])
@pytest.mark.parametrize("M", [9, 200, 5000])
def test_v1_dynamic_w8a8_linear_matches_oracle(cuda_device, variant, M):
    """kernels/quantization.py's dynamic W8A8 Linear: v1 row quantiser
    (trunc(x/s +- 0.5) in [-127, 127]), int8 GEMM, acc * sa * sw + bias --
    bit-exact against the oracle for every entry point."""
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import quantization as Q

    K, N = 4096, 512
    gen = torch.Generator(device=cuda_device).manual_seed(M)
    x = (0.1 * torch.randn(M, K, device=cuda_device, generator=gen)).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, generator=gen) / K ** 0.5
    w_q, w_s = Q.quantize_weight_per_channel_int8(w)
    bias = (0.02 * torch.randn(N, device=cuda_device, generator=gen)).to(torch.bfloat16)
    out = getattr(Q, variant)(x, w_q, w_s, bias=bias)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    oq, osc = O.quant_rows_v1(x.float().cpu().numpy())
    owq, ows = O.quant_rows_v1(w.cpu().numpy())
    assert np.array_equal(w_q.cpu().numpy(), owq) and np.array_equal(w_s.cpu().numpy(), ows)
    ref = O.scaled_epilogue(O.gemm_i8_i32(oq, owq), osc, ows, bias.float().cpu().numpy(), "bfloat16")
    assert np.array_equal(out.float().cpu().numpy(), ref)


def test_bf16_linear_helper(cuda_device):
    import torch
    from baidu_cti_grab_b200 import quantization as Q

    gen = torch.Generator(device=cuda_device).manual_seed(2)
    x = torch.randn(3, 50, 1024, device=cuda_device, generator=gen)
    w = torch.randn(512, 1024, device=cuda_device, generator=gen) / 32
    out = Q.bf16_linear(x, w)
    assert out.shape == (3, 50, 512) and out.dtype == torch.bfloat16
    ref = x.to(torch.bfloat16).double() @ w.to(torch.bfloat16).double().t()
    assert float((out.double() - ref).abs().max()) <= 2.0 ** -8 * float(ref.abs().max()) + 1e-3
