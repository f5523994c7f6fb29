"""K2 (tcgen05 int8 GEMM) and the standalone quantisers on the GPU.

int32 accumulators are bit-exact against the oracle (an exact fp64 matmul)
and the reference's Triton GEMM (golden fixture); the fp32 epilogue
``((acc*sa)*sb)+bias`` is bit-exact against the oracle and the reference; the
bf16 output is bit-exact against the oracle (one RNE of the same fp32 value).
"""

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _bf16_bits(torch, t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_gemm_golden(cuda_device):
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops

    g = load_golden("gemm.npz")
    for tag in ("k14336", "ktail"):
        a = torch.from_numpy(g[f"{tag}_a"]).to(cuda_device)
        b = torch.from_numpy(g[f"{tag}_qweight_nk"]).to(cuda_device)
        M, N = a.shape[0], b.shape[0]
        acc = device_ops.w8a8_gemm(a, b, None, None, torch.empty((M, N), dtype=torch.int32, device=cuda_device))
        assert np.array_equal(acc.cpu().numpy(), g[f"{tag}_acc_ref"])
        sa = torch.from_numpy(g[f"{tag}_sa"]).to(cuda_device)
        sb = torch.from_numpy(g[f"{tag}_wscale"]).to(cuda_device)
        bias = torch.from_numpy(g[f"{tag}_bias"].view(np.int16)).view(torch.bfloat16).to(cuda_device)
        out = device_ops.w8a8_gemm(a, b, sa, sb, torch.empty((M, N), dtype=torch.float32, device=cuda_device),
                                   bias=bias)
        assert np.array_equal(out.cpu().numpy(), g[f"{tag}_out_dyn_ref"])
        st = torch.from_numpy(g[f"{tag}_static_scale"]).to(cuda_device)
        out = device_ops.w8a8_gemm(a, b, st, sb, torch.empty((M, N), dtype=torch.float32, device=cuda_device),
                                   sa_per_row=False)
        assert np.array_equal(out.cpu().numpy(), g[f"{tag}_out_static_ref"])
        # bf16 output: one RNE of the same fp32 value
        outb = device_ops.w8a8_gemm(a, b, sa, sb, torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device),
                                    bias=bias)
        ref = O.f32_to_bf16_bits(g[f"{tag}_out_dyn_ref"])
        assert np.array_equal(_bf16_bits(torch, outb), ref)


@pytest.mark.parametrize("M,K,N", [(1, 14336, 512), (7, 14336, 512), (128, 14336, 512), (129, 4096, 512),
                                   (300, 592, 48), (1000, 14336, 512), (257, 128, 300), (64, 16, 256),
                                   (4096, 14336, 512), (33, 14336, 200), (1024, 14336, 512), (1025, 592, 300),
                                   (3000, 1024, 48), (2048, 14336, 257),
                                   # swapped operands up to M = 256 (the MMA's N side)
                                   (200, 14336, 512), (256, 14336, 520), (250, 592, 300), (160, 4096, 40),
                                   # M <= 16: one 16-byte K chunk, K over one round of
                                   # 128 chunks per CTA, column counts off the 16-column groups
                                   (3, 16, 48), (16, 16400, 40), (9, 2064, 17), (2, 14336, 1),
                                   # CTA-pair path (M >= 4096) with ragged M, N and K blocks; up to
                                   # half the pairs' worth of tiles it splits K (2 or 4 ways here)
                                   (4099, 1040, 300), (6000, 592, 48), (8191, 14336, 512), (4500, 2080, 130)])
def test_gemm_random_shapes(cuda_device, M, K, N):
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops

    rng = np.random.default_rng(M * 7 + K * 3 + N)
    a_np = rng.integers(-128, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    b_np = rng.integers(-128, 128, size=(N, K), dtype=np.int64).astype(np.int8)
    sa_np = rng.uniform(1e-3, 1e-2, size=M).astype(np.float32)
    sb_np = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    bias_np = O.round_to((0.02 * rng.standard_normal(N)).astype(np.float32), "bfloat16")
    a = torch.from_numpy(a_np).to(cuda_device)
    b = torch.from_numpy(b_np).to(cuda_device)
    acc = device_ops.w8a8_gemm(a, b, None, None, torch.empty((M, N), dtype=torch.int32, device=cuda_device))
    oacc = O.gemm_i8_i32(a_np, b_np)
    assert np.array_equal(acc.cpu().numpy(), oacc)
    out = device_ops.w8a8_gemm(a, b, torch.from_numpy(sa_np).to(cuda_device), torch.from_numpy(sb_np).to(cuda_device),
                               torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device),
                               bias=torch.from_numpy(bias_np).to(cuda_device, torch.bfloat16))
    ref = O.scaled_epilogue(oacc, sa_np, sb_np, bias_np, "bfloat16")
    assert np.array_equal(out.float().cpu().numpy(), ref)


def test_gemm_large_m_against_int_mm(cuda_device):
    """Full-size M: int32 accumulators equal torch._int_mm (an independent exact int8 GEMM)."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    M, K, N = 32768, 14336, 512
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda_device, generator=gen)
    b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=gen)
    acc = device_ops.w8a8_gemm(a, b, None, None, torch.empty((M, N), dtype=torch.int32, device=cuda_device))
    ref = torch._int_mm(a, b.t())
    assert torch.equal(acc, ref)


def test_gemm_weight_layouts(cuda_device):
    """qweight_t as a transposed view (no copy) and as a row-major [K,N] buffer (repacked)."""
    import torch
    from baidu_cti_grab_b200 import w8a8_triton_kernels as wk
    from baidu_cti_grab_b200.w8a8_preprocess import QuantizedWeight

    M, K, N = 200, 14336, 512
    gen = torch.Generator(device=cuda_device).manual_seed(9)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda_device, generator=gen)
    w_nk = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=gen)
    scale = torch.rand(N, device=cuda_device) * 1e-2
    q1 = QuantizedWeight(qweight_t=w_nk.t(), scale=scale, fp_weight=torch.empty(0))
    q2 = QuantizedWeight(qweight_t=w_nk.t().contiguous(), scale=scale, fp_weight=torch.empty(0))
    r1 = wk.int8_mm_no_scale(a, q1, out_dtype=torch.int32)
    r2 = wk.int8_mm_no_scale(a, q2, out_dtype=torch.int32)
    assert torch.equal(r1, r2)
    assert torch.equal(r1, torch._int_mm(a, w_nk.t()))


@pytest.mark.parametrize("name", ["bf16", "f32", "f16"])
def test_quantisers_golden(cuda_device, name):
    import torch
    from baidu_cti_grab_b200 import w8a8_triton_kernels as wk, quantization as q1mod

    z = load_golden("quant_edges.npz")
    if name == "bf16":
        x = torch.from_numpy(z["x_bf16"].view(np.int16)).view(torch.bfloat16)
    elif name == "f16":
        x = torch.from_numpy(z["x_f16"].view(np.int16)).view(torch.float16)
    else:
        x = torch.from_numpy(z["x_f32"])
    x = x.to(cuda_device)
    q, s = wk.dynamic_per_token_quantize_activation(x)
    assert np.array_equal(q.cpu().numpy(), z[f"q_dyn_{name}"])
    assert np.array_equal(s.cpu().numpy(), z[f"s_dyn_{name}"])
    q, s = q1mod.quantize_rows_int8_triton(x)
    assert np.array_equal(q.cpu().numpy(), z[f"q_v1_{name}"])
    assert np.array_equal(s.cpu().numpy(), z[f"s_v1_{name}"])
    st = torch.from_numpy(z["static_scale"]).to(cuda_device)
    q = wk.static_quantize_activation(x, st)
    assert np.array_equal(q.cpu().numpy(), z[f"q_static_{name}"])


def test_weight_quant_matches_torch_formula(cuda_device):
    """quantize_weight_per_channel == the reference's torch arithmetic (w8a8_preprocess.py:49-52)."""
    import torch
    from baidu_cti_grab_b200.w8a8_preprocess import quantize_weight_per_channel

    g = load_golden("gemm.npz")
    w = torch.from_numpy(g["ktail_weight_f32"]).to(cuda_device)
    qw = quantize_weight_per_channel(w)
    assert np.array_equal(qw.qweight_t.t().cpu().numpy(), g["ktail_qweight_nk"])
    assert np.array_equal(qw.scale.cpu().numpy(), g["ktail_wscale"])
    w2 = torch.randn(512, 14336, device=cuda_device, dtype=torch.bfloat16)
    qw2 = quantize_weight_per_channel(w2)
    # the reference's formula evaluated by ATen on the CPU, where x / 127.0 is an
    # IEEE division (ATen on CUDA multiplies by a rounded reciprocal instead)
    wc = w2.float().cpu()
    amax = wc.abs().amax(dim=1).clamp(min=1e-8)
    scale = amax / 127.0
    ref = torch.round(wc / scale[:, None]).clamp(-128, 127).to(torch.int8)
    assert torch.equal(qw2.qweight_t.t().cpu(), ref)
    assert torch.equal(qw2.scale.cpu(), scale)
    assert qw2.qweight_t.stride() == (1, 14336)


def test_w8a8_linear_end_to_end(cuda_device):
    """w8a8_linear(act_mode=dynamic|static) on 3-D input == oracle quantiser + GEMM + epilogue."""
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import w8a8_triton_kernels as wk
    from baidu_cti_grab_b200.w8a8_preprocess import quantize_weight_per_channel

    gen = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(3, 50, 14336, device=cuda_device, dtype=torch.bfloat16, generator=gen)
    w = torch.randn(512, 14336, device=cuda_device, generator=gen) / 120.0
    bias = (torch.randn(512, device=cuda_device, generator=gen) * 0.02).to(torch.bfloat16)
    qw = quantize_weight_per_channel(w)
    y = wk.w8a8_linear(x, qw, bias=bias, act_mode="dynamic")
    assert y.shape == (3, 50, 512) and y.dtype == torch.bfloat16
    xf = x.reshape(-1, 14336).float().cpu().numpy()
    q, s = O.quant_dynamic_v2(xf)
    acc = O.gemm_i8_i32(q, qw.qweight_t.t().cpu().numpy())
    ref = O.scaled_epilogue(acc, s, qw.scale.cpu().numpy(), bias.float().cpu().numpy(), "bfloat16")
    assert np.array_equal(y.reshape(-1, 512).float().cpu().numpy(), ref)
    st = torch.tensor([0.03], device=cuda_device)
    y2 = wk.w8a8_linear(x, qw, bias=bias, act_mode="static", static_act_scale=st)
    q2 = O.quant_static_v2(xf, 0.03)
    acc2 = O.gemm_i8_i32(q2, qw.qweight_t.t().cpu().numpy())
    ref2 = O.scaled_epilogue(acc2, np.array([0.03], np.float32), qw.scale.cpu().numpy(),
                             bias.float().cpu().numpy(), "bfloat16", sa_per_row=False)
    assert np.array_equal(y2.reshape(-1, 512).float().cpu().numpy(), ref2)


def test_watchdog_timeout_status(cuda_device):
    """A bounded wait that nothing satisfies returns and reports its code; the context stays usable."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    device_ops.device_error(reset=True)
    device_ops.selftest_wait_timeout(20_000_000)  # 20 ms budget
    torch.cuda.synchronize()
    assert device_ops.device_error(reset=True) == 199
    assert device_ops.device_error() == 0
    x = torch.ones(4, device=cuda_device)
    assert float(x.sum()) == 4.0


@pytest.mark.parametrize("M,N", [(1, 512), (2, 512), (3, 512), (5, 256), (8, 512), (13, 520), (16, 512)])
@pytest.mark.parametrize("out_name", ["bf16", "f32", "i32"])
def test_gemm_small_m_equals_tensor_core_rows(cuda_device, M, N, out_name):
    """M <= 16 runs the dp4a kernel (one launch, no workspace): its rows equal the
    same rows computed by the tensor-core kernel inside a larger M, bit for bit,
    and its int32 accumulators equal an fp64 matmul."""
    import torch
    from baidu_cti_grab_b200 import _lib as L, device_ops

    K = 14336
    assert L.load().rb_w8a8_gemm_workspace_size(M, N, K) == 0
    gen = torch.Generator(device=cuda_device).manual_seed(100 + M)
    a = torch.randint(-128, 128, (40, K), dtype=torch.int8, device=cuda_device, generator=gen)
    b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=gen)
    sa = torch.rand(40, device=cuda_device, generator=gen) * 1e-2
    sb = torch.rand(N, device=cuda_device, generator=gen) * 1e-2
    bias = torch.randn(N, device=cuda_device, generator=gen).to(torch.bfloat16)
    dt = {"bf16": torch.bfloat16, "f32": torch.float32, "i32": torch.int32}[out_name]
    raw = dt == torch.int32
    big = device_ops.w8a8_gemm(a, b, None if raw else sa, None if raw else sb,
                               torch.empty((40, N), dtype=dt, device=cuda_device), bias=None if raw else bias)
    small = device_ops.w8a8_gemm(a[:M], b, None if raw else sa[:M], None if raw else sb,
                                 torch.empty((M, N), dtype=dt, device=cuda_device), bias=None if raw else bias)
    assert torch.equal(small, big[:M])
    acc = device_ops.w8a8_gemm(a[:M], b, None, None, torch.empty((M, N), dtype=torch.int32, device=cuda_device))
    assert torch.equal(acc.double(), a[:M].double() @ b.double().t())


@pytest.mark.parametrize("M", [300, 700, 2048])
def test_gemm_split_k_equals_unsplit(cuda_device, M):
    """The split-K path (workspace given) and the unsplit kernel (rb_w8a8_gemm) agree bit for bit."""
    import torch
    from baidu_cti_grab_b200 import _lib as L, device_ops

    K, N = 14336, 512
    assert L.load().rb_w8a8_gemm_workspace_size(M, N, K) > 0
    gen = torch.Generator(device=cuda_device).manual_seed(M)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=cuda_device, generator=gen)
    b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=cuda_device, generator=gen)
    sa = torch.rand(M, device=cuda_device) * 1e-2
    sb = torch.rand(N, device=cuda_device) * 1e-2
    bias = torch.randn(N, device=cuda_device).to(torch.bfloat16)
    split = device_ops.w8a8_gemm(a, b, sa, sb, torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device),
                                 bias=bias)
    unsplit = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    L.call("rb_w8a8_gemm", a.data_ptr(), K, b.data_ptr(), K, M, N, K, sa.data_ptr(), L.RB_F32, 1, sb.data_ptr(),
           L.RB_F32, bias.data_ptr(), L.RB_BF16, unsplit.data_ptr(), N, L.RB_BF16, stream)
    assert torch.equal(split, unsplit)
    acc = device_ops.w8a8_gemm(a, b, None, None, torch.empty((M, N), dtype=torch.int32, device=cuda_device))
    ref = a.double() @ b.double().t()
    assert torch.equal(acc.double(), ref)
