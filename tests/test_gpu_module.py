"""The drop-in RepEncoder (fuse_mode "b200") end to end on the GPU.

* bit-exact against the oracle (K1 + K2 restated on the CPU);
* against the reference's algorithm run by ATen on the same GPU
  (nn.EmbeddingBag + cat + nn.LayerNorm in bf16, then the W8A8 quantiser and
  GEMM): pooled rows, LayerNorm rows, int8 rows, scales and the bf16 output
  bit-exact (the tolerance max-abs <= 2e-2, rel-L2 <= 1e-3 is also asserted);
* against the fp32 unquantised LayerNorm + Linear (cat_free_layernorm_linear):
  rel-L2 <= 3e-2.
"""

import numpy as np
import pytest

from conftest import gpu_rsqrt

pytestmark = pytest.mark.gpu

MAX_ABS_W8A8 = 2e-2
REL_L2_W8A8 = 1e-3
REL_L2_FP32 = 3e-2


def _setup(torch, dev, users=96, rows=2000, seed=21):
    from baidu_cti_grab_b200 import synth
    from baidu_cti_grab_b200.rep_encoder import RepEncoder

    cfg = synth.WorkloadConfig("module-test", rows, "bfloat16", users, 1, 120, "1+poisson1", 1.1)
    batch_np = synth.make_batch(cfg, seed=seed)
    table = synth.make_table_torch(cfg.num_rows, seed=seed, device=dev)
    gen = torch.Generator(device=dev).manual_seed(seed)
    H = 28 * 512
    gamma = (1 + 0.1 * torch.randn(H, device=dev, generator=gen)).to(torch.bfloat16)
    beta = (0.05 * torch.randn(H, device=dev, generator=gen)).to(torch.bfloat16)
    # nn.Linear's default initialisation, U(-1/sqrt(H), 1/sqrt(H)) (random-init model weights)
    w = ((torch.rand(512, H, device=dev, generator=gen) * 2 - 1) / H ** 0.5).to(torch.bfloat16)
    bias = (0.02 * torch.randn(512, device=dev, generator=gen)).to(torch.bfloat16)
    rep = RepEncoder.from_parts(table, gamma, beta, w, bias)
    batch = {"user_offsets": torch.from_numpy(batch_np["user_offsets"]).to(dev)}
    for s in range(1, 29):
        batch[s] = [torch.from_numpy(batch_np[s][0]).to(dev), torch.from_numpy(batch_np[s][1])]  # offsets on CPU
    return rep, batch, batch_np


def _rel_l2(a, b):
    a = a.float()
    b = b.float()
    return float((a - b).norm() / b.norm())


def test_module_matches_oracle(cuda_device):
    import torch
    from oracle import oracle as O

    rep, batch, batch_np = _setup(torch, cuda_device)
    out, inter = __import__("baidu_cti_grab_b200.rep_encoder", fromlist=["x"]).rep_encoder_forward(
        rep, batch, return_intermediates=True)
    torch.cuda.synchronize()
    table = rep.emb.weight.view(torch.int16).cpu().numpy().view(np.uint16)
    g = rep.input_norm.weight.float().cpu().numpy()
    b = rep.input_norm.bias.float().cpu().numpy()
    oq, oscale = O.rep_forward(table, "bfloat16", batch_np, g, b, 1e-5, rsqrt=gpu_rsqrt)
    assert np.array_equal(inter["q"].cpu().numpy(), oq)
    assert np.array_equal(inter["scale"].cpu().numpy(), oscale)
    w_nk, w_scale = rep._b200_wcache[1].cpu().numpy(), rep._b200_wcache[2].cpu().numpy()
    ref = O.scaled_epilogue(O.gemm_i8_i32(oq, w_nk), oscale, w_scale, rep.linear.bias.float().cpu().numpy(),
                            "bfloat16")
    assert np.array_equal(out.float().cpu().numpy(), ref)
    assert out.dtype == torch.bfloat16 and out.shape == (oq.shape[0], 512)


def test_module_against_aten_reference_on_gpu(cuda_device):
    import torch
    import torch.nn.functional as F
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward
    from oracle import oracle as O

    rep, batch, _ = _setup(torch, cuda_device, seed=22)
    out, inter = rep_encoder_forward(rep, batch, return_intermediates=True)
    # the reference's torch path (models.py:27-47) with ATen's CUDA kernels
    V = rep.emb.weight.shape[0]
    pooled = []
    for s in range(1, 29):
        v, o = batch[s]
        o = o.to(v.device)
        pooled.append(F.embedding_bag(v.clamp(0, V - 1), rep.emb.weight, o[:-1], mode="sum", padding_idx=0))
    x = torch.cat(pooled, dim=1)
    assert torch.equal(x, inter["pooled"])
    ln = F.layer_norm(x, (x.shape[1],), rep.input_norm.weight, rep.input_norm.bias, 1e-5)
    # LayerNorm rows: bit-exact against ATen's CUDA LayerNorm
    assert torch.equal(ln, inter["ln"])
    # int8 rows and scales: the reference's dynamic quantiser (oracle restatement,
    # pinned to the reference's Triton kernel) on ATen's LayerNorm output
    q_ref, sa_ref = O.quant_dynamic_v2(ln.float().cpu().numpy())
    assert np.array_equal(inter["q"].cpu().numpy(), q_ref)
    assert np.array_equal(inter["scale"].cpu().numpy(), sa_ref)
    # bf16 output: the int8 GEMM + the reference's epilogue order with ATen ops
    w_nk, w_scale = rep._b200_wcache[1], rep._b200_wcache[2]
    acc = torch._int_mm(torch.from_numpy(q_ref).to(cuda_device), w_nk.t())
    sa = torch.from_numpy(sa_ref).to(cuda_device)
    ref = ((acc.float() * sa[:, None]) * w_scale[None, :] + rep.linear.bias.float()).to(torch.bfloat16)
    assert torch.equal(out, ref)
    assert (out.float() - ref.float()).abs().max().item() <= MAX_ABS_W8A8
    assert _rel_l2(out, ref) <= REL_L2_W8A8


def test_module_against_fp32_unquantised(cuda_device):
    import torch
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward
    from baidu_cti_grab_b200.rep_encoder_fusion import cat_free_layernorm_linear

    rep, batch, _ = _setup(torch, cuda_device, seed=23)
    out, inter = rep_encoder_forward(rep, batch, return_intermediates=True)
    pooled = [p.float() for p in inter["pooled"].split(512, dim=1)]
    ln32 = torch.nn.LayerNorm(28 * 512).to(cuda_device)
    with torch.no_grad():
        ln32.weight.copy_(rep.input_norm.weight.float())
        ln32.bias.copy_(rep.input_norm.bias.float())
    lin32 = torch.nn.Linear(28 * 512, 512).to(cuda_device)
    with torch.no_grad():
        lin32.weight.copy_(rep.linear.weight.float())
        lin32.bias.copy_(rep.linear.bias.float())
    with torch.no_grad():
        ref = cat_free_layernorm_linear(pooled, ln32, lin32)
    assert _rel_l2(out, ref) <= REL_L2_FP32


def test_install_into_reference_shaped_module(cuda_device):
    """install() adds fuse_mode 'b200' to a RepEncoder class with the reference's layout."""
    import types

    import torch
    import torch.nn as nn
    from baidu_cti_grab_b200.rep_encoder import install, rep_encoder_forward

    class RefLike(nn.Module):  # the reference's attribute layout (models.py:14-22)
        def __init__(self, rep):
            super().__init__()
            self.emb, self.input_norm, self.linear = rep.emb, rep.input_norm, rep.linear
            self.slot_num, self.fuse_mode = 28, "b200"

        def forward(self, batch):
            raise AssertionError("reference path must not run for fuse_mode b200")

    rep, batch, _ = _setup(torch, cuda_device, users=8, seed=24)
    mod = types.SimpleNamespace(RepEncoder=RefLike)
    install(mod)
    m = RefLike(rep)
    out = m(batch)
    assert torch.equal(out, rep_encoder_forward(rep, batch))


def test_static_quantised_checkpoint_layer(cuda_device):
    """A StaticQuantizedLinear-shaped layer (row-major qweight_t [K,N] buffer, static scale)."""
    import torch
    import torch.nn as nn
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward
    from baidu_cti_grab_b200.w8a8_preprocess import quantize_weight_per_channel

    rep, batch, _ = _setup(torch, cuda_device, users=16, seed=25)
    qw = quantize_weight_per_channel(rep.linear.weight.float())
    lin = nn.Module()
    lin.use_quant = True
    lin.qweight_t = qw.qweight_t.contiguous()  # row-major [K, N] as in the quantised checkpoint
    lin.weight_scale = qw.scale.to(torch.bfloat16)  # model.to(bf16) casts the buffers
    lin.static_act_scale = torch.tensor([0.05], device=cuda_device).to(torch.bfloat16)
    lin.bias = rep.linear.bias
    rep.linear = lin
    out, inter = rep_encoder_forward(rep, batch, return_intermediates=True)
    assert inter["scale"] is None
    s = lin.static_act_scale.float()
    t = (inter["ln"].float() * (1.0 / s)).double()  # fp32 product, rounded half away in float64
    q_ref = (torch.sign(t) * torch.floor(t.abs() + 0.5)).clamp(-128, 127).to(torch.int8)
    assert torch.equal(q_ref, inter["q"])
    acc = torch._int_mm(inter["q"], qw.qweight_t)
    ref = ((acc.float() * s) * lin.weight_scale.float()[None, :] + lin.bias.float()).to(torch.bfloat16)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("index_dtype", ["auto", "int64"])
@pytest.mark.parametrize("chunk_items", [None, 700, 97])
def test_host_pipeline_matches_direct_forward(cuda_device, chunk_items, index_dtype):
    """HostPipeline (overlapped H2D / forward / D2H), with whole batches and
    with batches cut into item chunks, packed as int32 (auto) or int64, returns
    exactly the direct forward's output on the reference's int64 batch."""
    import torch
    from baidu_cti_grab_b200 import synth
    from baidu_cti_grab_b200.pipeline import HostPipeline, pack_batch
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward

    rep, _, _ = _setup(torch, cuda_device, users=4, seed=26)
    cfg = synth.WorkloadConfig("pipe", 2000, "bfloat16", 40, 1, 90, "1+poisson1", 1.1)
    host = [synth.make_batch(cfg, seed=100 + i) for i in range(5)]
    packed = [pack_batch(b, chunk_items=chunk_items, index_dtype=index_dtype) for b in host]
    want = torch.int32 if index_dtype == "auto" else torch.int64
    assert all(pb.host.dtype == want for pb in packed)
    if chunk_items == 97:
        assert all(len(pb.chunks) > 10 for pb in packed)
    outs = [torch.empty((pb.num_items, 512), dtype=torch.bfloat16).pin_memory() for pb in packed]
    pipe = HostPipeline(rep, max_ids=max(pb.num_ids for pb in packed),
                        max_items=max(pb.num_items for pb in packed), max_chunks=64)
    pipe.run(packed, outs)
    pipe.synchronize()
    for b, o in zip(host, outs):
        dev_b = {s: (torch.from_numpy(b[s][0]).to(cuda_device), torch.from_numpy(b[s][1]).to(cuda_device))
                 for s in range(1, 29)}
        ref = rep_encoder_forward(rep, dev_b)
        assert torch.equal(o, ref.cpu())


@pytest.mark.parametrize("world", [2, 4, 8])
def test_slot_sharded_path_emulated_on_one_gpu(cuda_device, world):
    """The slot-sharded path (pool own slots -> exchange -> per-slot LayerNorm/int8 -> GEMM)
    with `world` ranks emulated in one process: the exchange is a copy between the
    emulated ranks' buffers.  Every rank's rows equal the single-GPU fused forward."""
    import torch
    from baidu_cti_grab_b200 import sharding, device_ops, synth
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward

    R = 300
    cfg = synth.WorkloadConfig("sharded", R, "bfloat16", 24, 1, 60, "1+poisson1", 1.2)
    b = synth.make_batch(cfg, seed=31)
    table = synth.make_table_torch(cfg.num_rows, seed=31, device=cuda_device)
    rep, _, _ = _setup(torch, cuda_device, users=2, seed=31)
    rep.emb.weight = torch.nn.Parameter(table, requires_grad=False)
    values = [torch.from_numpy(b[s][0]).to(cuda_device) for s in range(1, 29)]
    offsets = [torch.from_numpy(b[s][1]).to(cuda_device) for s in range(1, 29)]
    full = rep_encoder_forward(rep, {s: (values[s - 1], offsets[s - 1]) for s in range(1, 29)})
    w_nk, w_scale = rep._b200_wcache[1], rep._b200_wcache[2]
    plans = [sharding.make_slot_plan(r, world, b["user_offsets"]) for r in range(world)]
    encs = [sharding.SlotShardedRepEncoder(p, sharding.build_local_table(table, p, R), R, rep.input_norm.weight,
                                           rep.input_norm.bias, 1e-5, w_nk, w_scale, rep.linear.bias,
                                           all_to_all=lambda *a: None) for p in plans]
    pooled = [e.pool_local(values, offsets) for e in encs]
    for r, e in enumerate(encs):
        def fake_a2a(out, inp, out_splits, in_splits, r=r):
            i0, i1 = plans[r].my_items
            mine = i1 - i0
            for j in range(world):
                out[j * mine:(j + 1) * mine].copy_(pooled[j][i0:i1])
        e.all_to_all = fake_a2a
        got = e.finish(pooled[r])
        i0, i1 = plans[r].my_items
        assert torch.equal(got, full[i0:i1])


@pytest.mark.parametrize("world", [2, 3, 8])
def test_pool_scatter_exchange_emulated_on_one_gpu(cuda_device, world):
    """The slot-sharded path with the exchange done by the pooling kernel
    (rb_rep_gather_pool_scatter), `world` ranks emulated in one process whose
    "peer" buffers are ordinary local tensors: each rank's receive buffer equals
    the rows the all-to-all path delivers, and its output equals the single-GPU
    fused forward, bit for bit, over two steps (both receive buffers)."""
    import torch
    from baidu_cti_grab_b200 import sharding, synth
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward

    R = 300
    cfg = synth.WorkloadConfig("scatter", R, "bfloat16", 20, 1, 60, "1+poisson1", 1.2)
    b = synth.make_batch(cfg, seed=41)
    table = synth.make_table_torch(cfg.num_rows, seed=41, device=cuda_device)
    rep, _, _ = _setup(torch, cuda_device, users=2, seed=41)
    rep.emb.weight = torch.nn.Parameter(table, requires_grad=False)
    values = [torch.from_numpy(b[s][0]).to(cuda_device) for s in range(1, 29)]
    offsets = [torch.from_numpy(b[s][1]).to(cuda_device) for s in range(1, 29)]
    full = rep_encoder_forward(rep, {s: (values[s - 1], offsets[s - 1]) for s in range(1, 29)})
    w_nk, w_scale = rep._b200_wcache[1], rep._b200_wcache[2]
    plans = [sharding.make_slot_plan(r, world, b["user_offsets"]) for r in range(world)]
    encs = [sharding.SlotShardedRepEncoder(p, sharding.build_local_table(table, p, R), R, rep.input_norm.weight,
                                           rep.input_norm.bias, 1e-5, w_nk, w_scale, rep.linear.bias,
                                           all_to_all=lambda *a: None) for p in plans]
    exs = [sharding.PeerExchange(p, torch.bfloat16, cuda_device, peer_ptrs=[[0] * world] * 2) for p in plans]
    for ex in exs:
        ex.ptrs = [[exs[d].bufs[k].data_ptr() for d in range(world)] for k in range(2)]
    pooled = [e.pool_local(values, offsets) for e in encs]
    for step in range(2):
        ks = [ex.next_buffer() for ex in exs]
        assert len(set(ks)) == 1 and ks[0] == step
        for ex in exs:
            ex.bufs[ks[0]].fill_(float("nan"))  # a stale row would show up
        for r, e in enumerate(encs):
            e.pool_scatter(values, offsets, exs[r], ks[r])
        for r, e in enumerate(encs):
            i0, i1 = plans[r].my_items
            recv = exs[r].received(ks[r])
            for j in range(world):
                nloc = len(plans[j].slots)
                assert torch.equal(recv[j, :, : nloc * 512], pooled[j][i0:i1, : nloc * 512])
            got = e.finish_received(recv)
            assert torch.equal(got, full[i0:i1])


def test_pool_scatter_fp32_table_matches_pool(cuda_device):
    """rb_rep_gather_pool_scatter with an fp32 table (rows stored slot by slot,
    not through the shared-memory row copy) and items taken from a shifted
    start: every destination row equals rb_rep_gather_pool's, bit for bit."""
    import torch
    from baidu_cti_grab_b200 import device_ops, synth

    cfg = synth.WorkloadConfig("scatter32", 200, "float32", 12, 1, 30, "uniform1-4", 1.1)
    b = synth.make_batch(cfg, seed=7)
    table = torch.from_numpy(synth.make_table_numpy(cfg.num_rows, seed=7, dtype="float32")).to(cuda_device)
    slots = [3, 11, 20]
    vals = [torch.from_numpy(b[s][0]).to(cuda_device) for s in slots]
    offs = [torch.from_numpy(b[s][1]).to(cuda_device) for s in slots]
    n = len(b[1][1]) - 1
    width = 4 * 512
    ref = device_ops.rep_gather_pool(table, vals, offs, [0, 1, 2], 4)
    cut = [0, n // 3, (2 * n) // 3, n]
    bufs = [torch.full((max(1, cut[d + 1] - cut[d]), width), float("nan"), device=cuda_device) for d in range(3)]
    device_ops.rep_gather_pool_scatter(table, vals, offs, [0, 1, 2], [t.data_ptr() for t in bufs], cut, width,
                                       item_shift=cut[2])
    for d in range(3):
        rows = cut[d + 1] - cut[d]
        assert torch.equal(bufs[d][:rows, : 3 * 512], ref[cut[d]:cut[d + 1], : 3 * 512])
