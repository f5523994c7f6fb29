"""rb_w8a8_gemm_noalloc: the GEMM entry point for callers that cannot allocate
device memory (their memory belongs to another allocator's pool or a
pre-sized arena, or their host forbids cudaMalloc after start-up).

It is called here through the C ABI exactly as such a caller would, with only
its inputs and outputs, and must reproduce the allocating entry point bit for
bit on two calls in a row (the shared scratch array keeps the previous call's
partials, which must not leak into the next result).  This file is collected
last so that a failure here cannot hide another test's result.
"""

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [300, 1000, 2048])
def test_noalloc_gemm_matches_allocating_entry_point(cuda_device, M):
    import torch

    from baidu_cti_grab_b200 import _lib as L
    from baidu_cti_grab_b200 import device_ops

    K, N = 14336, 512
    assert L.load().rb_w8a8_gemm_workspace_size(M, N, K) > 0  # this shape takes the scratch (split-K) path
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        gen = torch.Generator(device=cuda_device).manual_seed(1000 * M + call)
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda_device, generator=gen)
        b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=gen)
        sa = torch.rand(M, device=cuda_device, generator=gen) * 1e-2
        sb = torch.rand(N, device=cuda_device, generator=gen) * 1e-2
        bias = (0.02 * torch.randn(N, device=cuda_device, generator=gen)).to(torch.bfloat16)
        ref = device_ops.w8a8_gemm(a, b, sa, sb, torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device),
                                   bias=bias)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        L.call("rb_w8a8_gemm_noalloc", a.data_ptr(), K, b.data_ptr(), K, M, N, K, sa.data_ptr(), L.RB_F32, 1,
               sb.data_ptr(), L.RB_F32, bias.data_ptr(), L.RB_BF16, out.data_ptr(), N, L.RB_BF16, stream)
        acc = torch.empty((M, N), dtype=torch.int32, device=cuda_device)
        L.call("rb_w8a8_gemm_noalloc", a.data_ptr(), K, b.data_ptr(), K, M, N, K, None, 0, 1, None, 0, None, 0,
               acc.data_ptr(), N, L.RB_I32, stream)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)  # bit-exact: the tolerance of this suite for the GEMM
        assert torch.equal(acc.double(), a.double() @ b.double().t())
