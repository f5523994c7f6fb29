"""Parity at the benchmark configurations' own sizes (GPU).

* fp32 tables of 100k rows per slot, 64 users, sequence lengths U[1,64],
  ids per item and slot U[1,4] Zipf(1.1): K1 + K2 on the whole batch, bit for
  bit against the oracle and against the reference's path run by ATen.
* bf16 tables of 1M rows per slot (28.7 GB), 1024 users, U[1,200] (~104k
  items), 1+Poisson(1) ids Zipf(1.1) -- the bench's step: the whole batch
  against ATen's EmbeddingBag / cat / LayerNorm on the same GPU and K1's int8
  against the standalone quantiser on ATen's LayerNorm rows; 2048 items
  against the oracle through K2's bf16 output.
* The int8 GEMM sweep's large M (32768, 131072): int32 accumulators against
  torch._int_mm on the full matrix, the bf16 epilogue against the oracle on
  sampled rows.

The oracle gets each sample's table rows gathered into a compact table (ids
renumbered), so it never holds the device table.
"""

import numpy as np
import pytest

from conftest import gpu_rsqrt

pytestmark = pytest.mark.gpu


def _compact_sample(torch, table, batch, i0, i1, slots=28):
    """Items [i0, i1) of `batch` with the table rows their ids touch: returns
    (host table in the oracle's format, batch with renumbered ids)."""
    pieces = []
    sub = {"user_offsets": np.array([0, i1 - i0], dtype=np.int64)}
    for s in range(1, slots + 1):
        vals, offs = batch[s]
        v = vals[offs[i0]:offs[i1]] if i1 < len(offs) - 1 else vals[offs[i0]:]
        o = offs[i0:i1 + 1] - offs[i0]
        pieces.append(v)
        sub[s] = [v, o]
    uniq = np.unique(np.concatenate(pieces + [np.zeros(1, np.int64)]))
    rows = table[torch.from_numpy(uniq).to(table.device)]
    if rows.dtype == torch.bfloat16:
        host = rows.view(torch.int16).cpu().numpy().view(np.uint16)
    else:
        host = rows.cpu().numpy()
    for s in range(1, slots + 1):
        sub[s][0] = np.searchsorted(uniq, sub[s][0]).astype(np.int64)
        sub[s] = tuple(sub[s])
    return host, sub


def _weights(torch, dev, seed, H=28 * 512):
    from baidu_cti_grab_b200.w8a8_preprocess import quantize_weight_per_channel

    gen = torch.Generator(device=dev).manual_seed(seed)
    # nn.Linear's default initialisation of the 14336 -> 512 layer, then the reference's weight prep
    w = ((torch.rand(512, H, device=dev, generator=gen) * 2 - 1) / H ** 0.5)
    bias = ((torch.rand(512, device=dev, generator=gen) * 2 - 1) / H ** 0.5).to(torch.bfloat16)
    qw = quantize_weight_per_channel(w)
    return w, qw, bias


def _ln_params(torch, dev, seed, dtype, H=28 * 512):
    gen = torch.Generator(device=dev).manual_seed(seed)
    g = (1 + 0.1 * torch.randn(H, device=dev, generator=gen)).to(dtype)
    b = (0.05 * torch.randn(H, device=dev, generator=gen)).to(dtype)
    return g, b


def _aten_pooled_slots(torch, table, vals, offs):
    import torch.nn.functional as F

    V = table.shape[0]
    for v, o in zip(vals, offs):
        yield F.embedding_bag(v.clamp(0, V - 1), table, o[:-1], mode="sum", padding_idx=0)


def test_cpu_fp32_config_whole_batch(cuda_device):
    """fp32 tables, 100k rows per slot, 64 users: every output bit against the
    oracle and against ATen; the bf16 output also within rel-L2 3e-2 of the fp32
    unquantised LayerNorm + Linear."""
    import torch
    import torch.nn.functional as F
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops, synth

    dev = cuda_device
    cfg = synth.CPU_FP32_SMALL
    batch = synth.make_batch(cfg, seed=0)
    table = synth.make_table_torch(cfg.num_rows, seed=0, dtype=torch.float32, device=dev)
    g, b = _ln_params(torch, dev, 1, torch.float32)
    w, qw, bias = _weights(torch, dev, 2)
    vals = [torch.from_numpy(batch[s][0]).to(dev) for s in range(1, 29)]
    offs = [torch.from_numpy(batch[s][1]).to(dev) for s in range(1, 29)]
    n = len(batch[1][1]) - 1
    q, scale, pooled, ln = device_ops.rep_gather_ln_quant(table, vals, offs, g, b, 1e-5, want_pooled=True,
                                                          want_ln=True)
    w_nk = qw.qweight_t.t()
    out = device_ops.w8a8_gemm(q, w_nk, scale, qw.scale, torch.empty((n, 512), dtype=torch.bfloat16, device=dev),
                               bias=bias)
    torch.cuda.synchronize()
    # the oracle on the whole batch
    host, sub = _compact_sample(torch, table, batch, 0, n)
    oq, osc, opooled, oln = O.rep_forward(host, "float32", sub, g.cpu().numpy(), b.cpu().numpy(), 1e-5,
                                          intermediates=True, rsqrt=gpu_rsqrt)
    assert np.array_equal(pooled.cpu().numpy(), opooled)
    assert np.array_equal(ln.cpu().numpy(), oln)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(scale.cpu().numpy(), osc)
    ref = O.scaled_epilogue(O.gemm_i8_i32(oq, w_nk.cpu().numpy()), osc, qw.scale.cpu().numpy(),
                            bias.float().cpu().numpy(), "bfloat16")
    assert np.array_equal(out.float().cpu().numpy(), ref)
    # the reference's path with ATen's CUDA kernels
    x = torch.cat(list(_aten_pooled_slots(torch, table, vals, offs)), dim=1)
    assert torch.equal(x, pooled)
    assert torch.equal(F.layer_norm(x, (x.shape[1],), g, b, 1e-5), ln)
    # the fp32 unquantised LayerNorm + Linear
    ref32 = F.linear(ln, w, bias.float())
    rel = float((out.float() - ref32).norm() / ref32.norm())
    assert rel <= 3e-2


def test_prod_bf16_config_full_batch(cuda_device):
    """The bench's step (bf16, 1M rows per slot, 1024 users): the whole batch
    against ATen, 2048 items through K2 against the oracle."""
    import torch
    import torch.nn.functional as F
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops, synth

    dev = cuda_device
    cfg = synth.PROD_BF16_1M
    batch = synth.make_batch(cfg, seed=0)
    table = synth.make_table_torch(cfg.num_rows, seed=0, device=dev)
    g, b = _ln_params(torch, dev, 3, torch.bfloat16)
    _, qw, bias = _weights(torch, dev, 4)
    vals = [torch.from_numpy(batch[s][0]).to(dev) for s in range(1, 29)]
    offs = [torch.from_numpy(batch[s][1]).to(dev) for s in range(1, 29)]
    n = len(batch[1][1]) - 1
    assert n > 100_000
    q, scale, pooled, ln = device_ops.rep_gather_ln_quant(table, vals, offs, g, b, 1e-5, want_pooled=True,
                                                          want_ln=True)
    w_nk = qw.qweight_t.t()
    out = device_ops.w8a8_gemm(q, w_nk, scale, qw.scale, torch.empty((n, 512), dtype=torch.bfloat16, device=dev),
                               bias=bias)
    # whole batch: pooled slots == ATen EmbeddingBag, LayerNorm rows == ATen LayerNorm
    for s, eb in enumerate(_aten_pooled_slots(torch, table, vals, offs)):
        assert torch.equal(eb, pooled[:, s * 512:(s + 1) * 512]), f"slot {s + 1}"
    ln_ref = F.layer_norm(pooled, (pooled.shape[1],), g, b, 1e-5)
    assert torch.equal(ln_ref, ln)
    del ln_ref
    # whole batch: the fused quantiser == the standalone one (pinned to the
    # reference's Triton quantiser) on the LayerNorm rows
    q2 = torch.empty_like(q)
    s2 = torch.empty_like(scale)
    device_ops.quant_dynamic_per_token_out(ln, q2, s2)
    assert torch.equal(q, q2) and torch.equal(scale, s2)
    # 2048 items spread over the batch against the oracle, through K2
    rng = np.random.default_rng(5)
    starts = np.sort(rng.choice(n - 256, size=8, replace=False))
    for i0 in starts:
        i1 = int(i0) + 256
        host, sub = _compact_sample(torch, table, batch, int(i0), i1)
        oq, osc = O.rep_forward(host, "bfloat16", sub, g.float().cpu().numpy(), b.float().cpu().numpy(), 1e-5,
                                rsqrt=gpu_rsqrt)
        assert np.array_equal(q[i0:i1].cpu().numpy(), oq)
        assert np.array_equal(scale[i0:i1].cpu().numpy(), osc)
        ref = O.scaled_epilogue(O.gemm_i8_i32(oq, w_nk.cpu().numpy()), osc, qw.scale.cpu().numpy(),
                                bias.float().cpu().numpy(), "bfloat16")
        assert np.array_equal(out[i0:i1].float().cpu().numpy(), ref)


@pytest.mark.parametrize("M", [32768, 131072])
def test_gemm_sweep_large_m(cuda_device, M):
    """A int8 U[-127,127], per-channel scales U[1e-3,1e-2], per-token scales,
    bias N(0, 0.02): int32 accumulators == torch._int_mm on the whole matrix;
    the bf16 output == the oracle's epilogue on 512 sampled rows."""
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops

    dev = cuda_device
    K, N = 28 * 512, 512
    gen = torch.Generator(device=dev).manual_seed(M)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=gen)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=gen)
    sa = torch.rand(M, device=dev, generator=gen) * 9e-3 + 1e-3
    sb = torch.rand(N, device=dev, generator=gen) * 9e-3 + 1e-3
    bias = (0.02 * torch.randn(N, device=dev, generator=gen)).to(torch.bfloat16)
    acc = device_ops.w8a8_gemm(a, b, None, None, torch.empty((M, N), dtype=torch.int32, device=dev))
    assert torch.equal(acc, torch._int_mm(a, b.t()))
    out = device_ops.w8a8_gemm(a, b, sa, sb, torch.empty((M, N), dtype=torch.bfloat16, device=dev), bias=bias)
    rows = torch.from_numpy(np.sort(np.random.default_rng(M).choice(M, 512, replace=False))).to(dev)
    oacc = O.gemm_i8_i32(a[rows].cpu().numpy(), b.cpu().numpy())
    assert np.array_equal(oacc, acc[rows].cpu().numpy())
    ref = O.scaled_epilogue(oacc, sa[rows].cpu().numpy(), sb.cpu().numpy(), bias.float().cpu().numpy(), "bfloat16")
    assert np.array_equal(out[rows].float().cpu().numpy(), ref)
