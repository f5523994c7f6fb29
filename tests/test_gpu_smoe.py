"""The SMoE expert layer (rb_smoe_experts, smoe.smoe_forward) on the GPU.

Two references, both on the same inputs:

* a float64 emulation of the reference's bf16/fp16 op sequence
  (models.py:131-178): every dot product exact, then each torch op's rounding
  to the model dtype -- bmm, + bias, relu, bmm, + bias, * score, index_add_ of
  the k rows into zeros;
* the reference's own torch formulation restated here (stable argsort, padded
  [E, max_count, D] block, torch.bmm on cuBLAS, index_add_).

Tolerance (floating point; the kernel accumulates each dot product in fp32,
the float64 emulation exactly): every element is within 2^-5 * mag + 2^-14
of the emulation, mag being the sum over the token's k rows of |second bmm|
+ |bias| (each of the three roundings after the bmm can flip by one unit in
the last place, at most 2^-7 of those values, and flipped hidden values add
a little more), the output's relative L2 error is at most 4e-3, and at least
98 % of the elements are identical for bf16, 95 % for fp16 (three more
mantissa bits, so a fixed fp32 accumulation difference flips more
roundings); a wrong rounding step would break most of them.  Against the cuBLAS formulation the
same bounds, with at least 99 % identical: both accumulate in fp32 on the
tensor cores, and at the bench's token count they agree bit for bit.
"""

import pytest

pytestmark = pytest.mark.gpu


def _round(torch, v, dtype):
    return v.to(dtype).double()


def _emulate(torch, x, idx, score, w1, b1, w2, b2):
    """float64 dot products, rounded to x.dtype where the reference rounds.
    Returns (out, mag): mag sums, over each token's k rows, |second bmm| +
    |bias| -- the size of the values whose rounding can flip before the score
    scales them down."""
    dt = x.dtype
    T, D = x.shape
    k = idx.shape[1]
    E = w1.shape[0]
    out = torch.zeros((T, D), dtype=torch.float64, device=x.device)
    mag = torch.zeros_like(out)
    for s in range(k):
        y = torch.zeros((T, D), dtype=torch.float64, device=x.device)
        for e in range(E):
            rows = torch.nonzero(idx[:, s] == e).flatten()
            if rows.numel() == 0:
                continue
            h = _round(torch, x[rows].double() @ w1[e].double().t(), dt)
            if b1 is not None:
                h = _round(torch, h + b1[e].double(), dt)
            h = h.clamp_min(0)
            acc = _round(torch, h @ w2[e].double().t(), dt)
            ye = acc if b2 is None else _round(torch, acc + b2[e].double(), dt)
            y[rows] = _round(torch, ye * score[rows, s].double()[:, None], dt)
            mag[rows] += acc.abs() + (0 if b2 is None else b2[e].double().abs())
        out = _round(torch, out + y, dt)
    return out, mag


def _reference_torch(torch, x, idx, score, w1, b1, w2, b2):
    """The reference's formulation (models.py:137-172) in torch on the GPU."""
    T, D = x.shape
    k = idx.shape[1]
    E = w1.shape[0]
    route_expert = idx.reshape(-1)
    route_weight = score.reshape(-1)
    route_token = torch.arange(T, device=x.device).repeat_interleave(k)
    order = torch.argsort(route_expert, stable=True)
    se, sw, st = route_expert[order], route_weight[order], route_token[order]
    counts = torch.bincount(se, minlength=E)
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.arange(se.numel(), device=x.device) - torch.repeat_interleave(starts, counts)
    packed = x.new_zeros((E, int(counts.max()), D))
    packed[se, pos] = x[st]
    hidden = torch.bmm(packed, w1.transpose(1, 2)) + (b1.unsqueeze(1) if b1 is not None else 0)
    hidden = torch.relu(hidden)
    pout = torch.bmm(hidden, w2.transpose(1, 2)) + (b2.unsqueeze(1) if b2 is not None else 0)
    routed = pout[se, pos] * sw.unsqueeze(-1)
    out = torch.zeros_like(x)
    out.index_add_(0, st, routed)
    return out


def _inputs(torch, dev, T, D, F, E, k, dtype, seed, skew=None):
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randn(T, D, device=dev, generator=gen)).to(dtype)
    logits = torch.randn(T, E, device=dev, generator=gen)
    if skew is not None:
        logits = logits + skew.to(dev)
    probs = torch.softmax(logits.to(dtype), dim=-1)
    score, idx = torch.topk(probs, k, dim=-1)
    w1 = (torch.randn(E, F, D, device=dev, generator=gen) / D ** 0.5).to(dtype)
    b1 = (0.1 * torch.randn(E, F, device=dev, generator=gen)).to(dtype)
    w2 = (torch.randn(E, D, F, device=dev, generator=gen) / F ** 0.5).to(dtype)
    b2 = (0.1 * torch.randn(E, D, device=dev, generator=gen)).to(dtype)
    return x, idx, score, w1, b1, w2, b2


def _check(torch, out, ref, mag, exact_min):
    d = (out.double() - ref).abs()
    excess = d - (2.0 ** -5 * mag + 2.0 ** -14)
    i = int(torch.argmax(excess))
    r, c = divmod(i, out.shape[1])
    assert float(excess.max()) <= 0, (f"row {r} col {c}: out {float(out[r, c])} ref {float(ref[r, c])} "
                                      f"mag {float(mag[r, c])}")
    rel = float((out.double() - ref).norm() / ref.norm().clamp_min(1e-30))
    assert rel <= 4e-3, rel
    exact = float((out.double() == ref).double().mean())
    assert exact >= exact_min, exact


@pytest.mark.parametrize("T,D,F,E,k,dtype", [
    (1, 512, 1024, 8, 2, "bfloat16"),
    (1000, 512, 1024, 8, 2, "bfloat16"),
    (4099, 512, 1024, 8, 2, "float16"),
    (777, 256, 512, 4, 1, "bfloat16"),
    (300, 128, 192, 3, 3, "bfloat16"),
])
def test_smoe_experts_against_float64_emulation(cuda_device, T, D, F, E, k, dtype):
    import torch
    from baidu_cti_grab_b200 import device_ops

    dt = getattr(torch, dtype)
    x, idx, score, w1, b1, w2, b2 = _inputs(torch, cuda_device, T, D, F, E, k, dt, seed=T + E)
    out = device_ops.smoe_experts(x, idx, score, w1, b1, w2, b2)
    assert out.dtype == dt and out.shape == (T, D)
    ref, mag = _emulate(torch, x, idx, score, w1, b1, w2, b2)
    _check(torch, out, ref, mag, 0.98 if dt == torch.bfloat16 else 0.95)
    # the same result with int32 expert ids, and run twice (deterministic)
    out32 = device_ops.smoe_experts(x, idx.to(torch.int32), score, w1, b1, w2, b2)
    assert torch.equal(out, out32)


def test_smoe_experts_against_reference_formulation_cublas(cuda_device):
    import torch
    from baidu_cti_grab_b200 import device_ops

    T, D, F, E, k = 5000, 512, 1024, 8, 2
    x, idx, score, w1, b1, w2, b2 = _inputs(torch, cuda_device, T, D, F, E, k, torch.bfloat16, seed=3)
    out = device_ops.smoe_experts(x, idx, score, w1, b1, w2, b2)
    ref = _reference_torch(torch, x, idx, score, w1, b1, w2, b2)
    _, mag = _emulate(torch, x, idx, score, w1, b1, w2, b2)
    _check(torch, out, ref.double(), mag, 0.99)


def test_smoe_experts_unbalanced_and_empty_experts(cuda_device):
    """Most tokens on one expert, some experts with no rows, segments that end
    inside a 128-row block: every token's rows still land where they belong."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    T, D, F, E, k = 3001, 512, 1024, 8, 2
    skew = torch.tensor([6.0, 0.0, -30.0, 3.0, -30.0, 0.0, -30.0, 0.0])
    x, idx, score, w1, b1, w2, b2 = _inputs(torch, cuda_device, T, D, F, E, k, torch.bfloat16, seed=4, skew=skew)
    counts = torch.bincount(idx.reshape(-1), minlength=E)
    assert int((counts == 0).sum()) >= 2 and int(counts.max()) > T // 2
    out = device_ops.smoe_experts(x, idx, score, w1, b1, w2, b2)
    ref, mag = _emulate(torch, x, idx, score, w1, b1, w2, b2)
    _check(torch, out, ref, mag, 0.98)


def test_smoe_experts_without_bias(cuda_device):
    import torch
    from baidu_cti_grab_b200 import device_ops

    x, idx, score, w1, _, w2, _ = _inputs(torch, cuda_device, 640, 512, 1024, 8, 2, torch.bfloat16, seed=5)
    out = device_ops.smoe_experts(x, idx, score, w1, None, w2, None)
    ref, mag = _emulate(torch, x, idx, score, w1, None, w2, None)
    _check(torch, out, ref, mag, 0.98)


def test_smoe_experts_large_token_count(cuda_device):
    """The token count of a 1024-user batch (~103k items, 206k routed rows):
    relative L2 and sampled element bounds against the float64 emulation."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    T, D, F, E, k = 103725, 512, 1024, 8, 2
    x, idx, score, w1, b1, w2, b2 = _inputs(torch, cuda_device, T, D, F, E, k, torch.bfloat16, seed=6)
    out = device_ops.smoe_experts(x, idx, score, w1, b1, w2, b2)
    rows = torch.unique(torch.linspace(0, T - 1, 4096, device=cuda_device).long())
    ref, mag = _emulate(torch, x[rows], idx[rows], score[rows], w1, b1, w2, b2)
    _check(torch, out[rows], ref, mag, 0.98)


def test_smoe_experts_invalid_expert_adds_nothing(cuda_device):
    """An expert id outside [0, E) is skipped (its row adds nothing) and the
    device error word records it; the other rows are unaffected."""
    import torch
    from baidu_cti_grab_b200 import device_ops

    x, idx, score, w1, b1, w2, b2 = _inputs(torch, cuda_device, 257, 512, 1024, 8, 2, torch.bfloat16, seed=7)
    device_ops.device_error(reset=True)
    bad = idx.clone()
    bad[10, 1] = 8
    bad[200, 0] = -1
    out = device_ops.smoe_experts(x, bad, score, w1, b1, w2, b2)
    torch.cuda.synchronize()
    assert device_ops.device_error(reset=True) == 301
    keep = torch.ones_like(score)
    keep[10, 1] = 0
    keep[200, 0] = 0
    # the emulation with the bad entries' scores zeroed: their rows are exactly +0
    ref, mag = _emulate(torch, x, idx, score * keep, w1, b1, w2, b2)
    _check(torch, out, ref, mag, 0.98)


def test_smoe_forward_on_reference_layout(cuda_device):
    """smoe_forward on a module with the reference's SMoE attributes (experts
    of fc1/fc2 Linears, gate.w_g, k) equals the expert kernel on the gate's
    routing, and its loss is the reference's importance formula."""
    import torch
    import torch.nn as nn
    from baidu_cti_grab_b200 import device_ops
    from baidu_cti_grab_b200.smoe import smoe_forward, stacked_expert_params

    D, F, E = 512, 1024, 8

    class Expert(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1, self.fc2 = nn.Linear(D, F), nn.Linear(F, D)

    class Gate(nn.Module):
        def __init__(self):
            super().__init__()
            self.w_g = nn.Linear(D, E)
            self.k = 2

        def forward(self, x):
            probs = torch.softmax(self.w_g(x), dim=-1)
            score, idx = torch.topk(probs, self.k, dim=-1)
            return idx, score, probs

    class Moe(nn.Module):
        def __init__(self):
            super().__init__()
            self.experts = nn.ModuleList([Expert() for _ in range(E)])
            self.gate = Gate()
            self.k = 2

    torch.manual_seed(8)
    moe = Moe().to(cuda_device, torch.bfloat16)
    x = torch.randn(1, 900, D, device=cuda_device).to(torch.bfloat16)
    with torch.no_grad():
        out, loss = smoe_forward(moe, x)
        idx, score, probs = moe.gate(x)
        w1, b1, w2, b2 = stacked_expert_params(moe, torch.bfloat16)
        direct = device_ops.smoe_experts(x[0], idx[0], score[0], w1, b1, w2, b2)
        assert torch.equal(out[0], direct)
        imp = probs.sum(dim=(0, 1))
        assert torch.equal(loss, imp.std() / (imp.mean() + 1e-6))
        ref, mag = _emulate(torch, x[0], idx[0], score[0], w1, b1, w2, b2)
        _check(torch, out[0], ref, mag, 0.98)
        # the stacked weights are cached until a weight changes
        assert stacked_expert_params(moe, torch.bfloat16)[0] is w1
        moe.experts[3].fc1.weight.mul_(2)
        assert stacked_expert_params(moe, torch.bfloat16)[0] is not w1
