"""K1 (fused gather -> pool -> LayerNorm -> int8) on the GPU against the oracle.

Bit-exact: pooled rows, LayerNorm rows, int8 activations and per-token scales
(the oracle restates the reference's arithmetic, its LayerNorm in the order of
ATen's CUDA kernel, with rstd from the GPU's rsqrtf).  Against the golden
fixtures recorded from the reference's RepEncoder on ATen CPU + its Triton
quantiser: pooled rows bit-exact; ATen's CPU LayerNorm reduces in yet another
order than its CUDA kernel, so the int8 rows may differ there by one step on a
few elements.
"""

import numpy as np
import pytest

from conftest import golden_rep, gpu_rsqrt

pytestmark = pytest.mark.gpu


def _to_dev_batch(torch, batch, dev, slots=28):
    vals = [torch.from_numpy(np.ascontiguousarray(batch[s][0])).to(dev) for s in range(1, slots + 1)]
    offs = [torch.from_numpy(np.ascontiguousarray(batch[s][1])).to(dev) for s in range(1, slots + 1)]
    return vals, offs


def _table_tensor(torch, table_np, dt, dev):
    if dt == "bfloat16":
        return torch.from_numpy(table_np.view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(table_np).to(dev)


def _row_f32(torch, t):
    return t.float().cpu().numpy()


def _run_k1(torch, table, vals, offs, gamma, beta, eps, act_mode="dynamic", static_scale=None):
    from baidu_cti_grab_b200 import device_ops

    return device_ops.rep_gather_ln_quant(table, vals, offs, gamma, beta, eps, act_mode=act_mode,
                                          static_scale=static_scale, want_pooled=True, want_ln=True)


@pytest.mark.parametrize("fixture", ["rep_bf16.npz", "rep_f32.npz"])
def test_k1_golden_bit_exact(cuda_device, fixture):
    import torch
    from oracle import oracle as O

    dt, table_np, batch, gamma, beta, eps, z = golden_rep(fixture)
    tdt = torch.bfloat16 if dt == "bfloat16" else torch.float32
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    g = torch.from_numpy(gamma).to(cuda_device, tdt)
    b = torch.from_numpy(beta).to(cuda_device, tdt)
    q, scale, pooled, ln = _run_k1(torch, table, vals, offs, g, b, eps)
    torch.cuda.synchronize()
    oq, oscale, opooled, oln = O.rep_forward(table_np, dt, batch, gamma, beta, eps, intermediates=True,
                                             rsqrt=gpu_rsqrt)
    assert np.array_equal(_row_f32(torch, pooled), opooled)
    assert np.array_equal(_row_f32(torch, ln), oln)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(scale.cpu().numpy(), oscale)
    # the CPU-recorded fixtures: pooled rows exact; ATen's CPU LayerNorm order may move an int8 by one step
    tof = O.bf16_bits_to_f32 if dt == "bfloat16" else (lambda a: a.astype(np.float32))
    assert np.array_equal(_row_f32(torch, pooled), tof(z["pooled_ref"]))
    dq = np.abs(q.cpu().numpy().astype(np.int32) - z["q_dyn_ref"].astype(np.int32))
    assert dq.max() <= 1
    assert (dq != 0).mean() <= 1e-3


def test_k1_static_mode(cuda_device):
    import torch
    from oracle import oracle as O

    dt, table_np, batch, gamma, beta, eps, z = golden_rep("rep_bf16.npz")
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    g = torch.from_numpy(gamma).to(cuda_device, torch.bfloat16)
    b = torch.from_numpy(beta).to(cuda_device, torch.bfloat16)
    for sdt in (torch.float32, torch.bfloat16):
        s = torch.from_numpy(z["static_scale"]).to(cuda_device, sdt)
        q, scale, _, _ = _run_k1(torch, table, vals, offs, g, b, eps, act_mode="static", static_scale=s)
        assert scale is None
        oq, _ = O.rep_forward(table_np, dt, batch, gamma, beta, eps, act_mode="static",
                              static_scale=float(s.float().item()), rsqrt=gpu_rsqrt)
        assert np.array_equal(q.cpu().numpy(), oq)


@pytest.mark.parametrize("dt,seed,users", [("bfloat16", 11, 48), ("float32", 12, 16)])
def test_k1_synthetic_bit_exact(cuda_device, dt, seed, users):
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import synth

    cfg = synth.WorkloadConfig("test", 500, dt, users, 1, 60, "1+poisson1", 1.1)
    batch = synth.make_batch(cfg, seed=seed)
    table_np = synth.make_table_numpy(cfg.num_rows, seed=seed, dtype=dt)
    rng = np.random.default_rng(seed)
    gamma = (1.0 + 0.2 * rng.standard_normal(28 * 512)).astype(np.float32)
    beta = (0.05 * rng.standard_normal(28 * 512)).astype(np.float32)
    tdt = torch.bfloat16 if dt == "bfloat16" else torch.float32
    gamma = O.round_to(gamma, dt)
    beta = O.round_to(beta, dt)
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    q, scale, pooled, ln = _run_k1(torch, table, vals, offs, torch.from_numpy(gamma).to(cuda_device, tdt),
                                   torch.from_numpy(beta).to(cuda_device, tdt), 1e-5)
    oq, oscale, opooled, oln = O.rep_forward(table_np, dt, batch, gamma, beta, 1e-5, intermediates=True,
                                             rsqrt=gpu_rsqrt)
    assert np.array_equal(_row_f32(torch, pooled), opooled)
    assert np.array_equal(_row_f32(torch, ln), oln)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(scale.cpu().numpy(), oscale)


@pytest.mark.parametrize("param_dtype,offset", [("float32", 0), ("float32", 4), ("float16", 0), ("bfloat16", 8)])
def test_k1_affine_param_dtypes_on_bf16_rows(cuda_device, param_dtype, offset):
    """LayerNorm gamma/beta in fp32 (32-byte aligned, and only 16-byte aligned:
    a view 4 floats into a buffer), fp16 or bf16 while the table is bf16."""
    import torch
    from oracle import oracle as O

    dt, table_np, batch, gamma, beta, eps, _ = golden_rep("rep_bf16.npz")
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    rng = np.random.default_rng(5)
    g32 = (1.0 + 0.3 * rng.standard_normal(28 * 512)).astype(np.float32)
    b32 = (0.1 * rng.standard_normal(28 * 512)).astype(np.float32)
    tdt = getattr(torch, param_dtype)

    def put(a):
        buf = torch.zeros(a.size + offset, dtype=tdt, device=cuda_device)
        view = buf[offset:]
        view.copy_(torch.from_numpy(a))
        return view

    g, b = put(g32), put(b32)
    assert g.data_ptr() % 16 == 0
    g32, b32 = g.float().cpu().numpy(), b.float().cpu().numpy()  # the values the kernel sees
    q, scale, _, ln = _run_k1(torch, table, vals, offs, g, b, eps)
    oq, oscale, _, oln = O.rep_forward(table_np, dt, batch, g32, b32, eps, intermediates=True,
                                       rsqrt=gpu_rsqrt)
    assert np.array_equal(_row_f32(torch, ln), oln)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(scale.cpu().numpy(), oscale)


@pytest.mark.parametrize("dt,S", [("float32", 28), ("bfloat16", 28), ("bfloat16", 5), ("bfloat16", 32),
                                  ("float32", 7)])
def test_k1_edge_cases(cuda_device, dt, S):
    """Zero items, one item, every bag empty, ids out of range / negative / padding,
    bags longer than the 32-id window, odd bag lengths; bf16 and fp32 tables, the
    28-slot kernel and the generic slot count (5, 7 and the maximum 32)."""
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops

    dev = cuda_device
    V = 40
    H = S * 512
    t32 = (np.random.default_rng(0).standard_normal((V, 512)) * 0.02).astype(np.float32)
    table_np = O.f32_to_bf16_bits(t32) if dt == "bfloat16" else t32
    table = _table_tensor(torch, table_np, dt, dev)
    tdt = torch.bfloat16 if dt == "bfloat16" else torch.float32
    g = torch.ones(H, device=dev, dtype=tdt)
    b = torch.zeros(H, device=dev, dtype=tdt)
    # zero items
    vals = [torch.zeros(0, dtype=torch.int64, device=dev) for _ in range(S)]
    offs = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(S)]
    q, s, _, _ = device_ops.rep_gather_ln_quant(table, vals, offs, g, b, 1e-5)
    assert q.shape == (0, H)
    # four items: all bags empty for item 0, item 1 has odd ids (padding, negative,
    # past the vocabulary), item 2 a 40-id bag, item 3 a 3-id bag (odd length)
    batch = {"user_offsets": np.array([0, 4])}
    rng = np.random.default_rng(1)
    for sl in range(1, S + 1):
        ids = np.concatenate([np.array([0, -7, V + 5, 3], dtype=np.int64), rng.integers(0, V, 43)])
        batch[sl] = (ids, np.array([0, 0, 4, 44, 47], dtype=np.int64))
    vals, offs = _to_dev_batch(torch, batch, dev, slots=S)
    q, s, pooled, ln = device_ops.rep_gather_ln_quant(table, vals, offs, g, b, 1e-5, want_pooled=True,
                                                      want_ln=True)
    oq, os_, opooled, oln = O.rep_forward(table_np, dt, batch, np.ones(H, np.float32), np.zeros(H, np.float32),
                                          1e-5, num_slots=S, intermediates=True, rsqrt=gpu_rsqrt)
    assert np.array_equal(_row_f32(torch, pooled), opooled)
    assert np.all(_row_f32(torch, pooled)[0] == 0)
    assert np.array_equal(_row_f32(torch, ln), oln)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy(), os_)


@pytest.mark.parametrize("dt,S", [("bfloat16", 28), ("float32", 28), ("bfloat16", 5)])
def test_k1_int32_indices_equal_int64(cuda_device, dt, S):
    """Ids and offsets given as int32 (the packed ingestion format) give the same
    bits as int64 in every output: pooled rows, LayerNorm rows, int8 and scales,
    on a synthetic batch and on padding / negative / out-of-range ids, an empty
    bag, a 40-id bag and an odd-length bag.  Mixed widths are refused."""
    import torch
    from oracle import oracle as O
    from baidu_cti_grab_b200 import device_ops, synth

    dev = cuda_device
    V = 300
    H = S * 512
    t32 = (np.random.default_rng(5).standard_normal((V, 512)) * 0.02).astype(np.float32)
    table_np = O.f32_to_bf16_bits(t32) if dt == "bfloat16" else t32
    table = _table_tensor(torch, table_np, dt, dev)
    tdt = torch.bfloat16 if dt == "bfloat16" else torch.float32
    gen = torch.Generator(device="cpu").manual_seed(9)
    g = (1 + 0.1 * torch.randn(H, generator=gen)).to(tdt).to(dev)
    b = (0.1 * torch.randn(H, generator=gen)).to(tdt).to(dev)
    cfg = synth.WorkloadConfig("idx", (V - 1) // S, dt, 24, 1, 30, "1+poisson1", 1.1, num_slots=S)
    batches = [synth.make_batch(cfg, seed=77)]
    edge = {"user_offsets": np.array([0, 4])}
    rng = np.random.default_rng(2)
    for sl in range(1, S + 1):
        ids = np.concatenate([np.array([0, -7, V + 5, 3], dtype=np.int64), rng.integers(0, V, 43)])
        edge[sl] = (ids, np.array([0, 0, 4, 44, 47], dtype=np.int64))
    batches.append(edge)
    for batch in batches:
        v64, o64 = _to_dev_batch(torch, batch, dev, slots=S)
        v32, o32 = [v.to(torch.int32) for v in v64], [o.to(torch.int32) for o in o64]
        r64 = _run_k1(torch, table, v64, o64, g, b, 1e-5)
        r32 = _run_k1(torch, table, v32, o32, g, b, 1e-5)
        for x, y in zip(r64, r32):
            assert torch.equal(x, y)
    with pytest.raises(ValueError):
        device_ops.rep_gather_ln_quant(table, v32[:-1] + v64[-1:], o32, g, b, 1e-5)


def test_dense_layernorm_quant_matches_fused(cuda_device):
    """rb_layernorm_quant on pooled rows == the fused kernel's LayerNorm/int8 stage."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    dt, table_np, batch, gamma, beta, eps, _ = golden_rep("rep_bf16.npz")
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    g = torch.from_numpy(gamma).to(cuda_device, torch.bfloat16)
    b = torch.from_numpy(beta).to(cuda_device, torch.bfloat16)
    q, s, pooled, ln = _run_k1(torch, table, vals, offs, g, b, eps)
    q2, s2, ln2 = device_ops.layernorm_quant(pooled, g, b, eps, want_ln=True)
    assert torch.equal(q, q2) and torch.equal(s, s2) and torch.equal(ln, ln2)
    _, _, ln3 = device_ops.layernorm_quant(pooled, g, b, eps, act_mode="none")
    assert torch.equal(ln, ln3)


def test_gather_pool_column_placement(cuda_device):
    """rb_rep_gather_pool writes each slot's pooled row at its requested column block."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    dt, table_np, batch, gamma, beta, eps, _ = golden_rep("rep_bf16.npz")
    table = _table_tensor(torch, table_np, dt, cuda_device)
    vals, offs = _to_dev_batch(torch, batch, cuda_device)
    _, _, pooled, _ = _run_k1(torch, table, vals, offs, torch.from_numpy(gamma).to(cuda_device, torch.bfloat16),
                              torch.from_numpy(beta).to(cuda_device, torch.bfloat16), eps)
    sel = [3, 7, 11, 27, 0]
    out = device_ops.rep_gather_pool(table, [vals[s] for s in sel], [offs[s] for s in sel],
                                     col_slot=list(range(len(sel)))[::-1], width_slots=len(sel))
    for j, s in enumerate(sel):
        c = len(sel) - 1 - j
        assert torch.equal(out[:, c * 512:(c + 1) * 512], pooled[:, s * 512:(s + 1) * 512])
