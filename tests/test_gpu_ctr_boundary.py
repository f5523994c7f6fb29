"""The RepEncoder -> Transformer boundary in b200 mode (ctr_boundary) on the GPU.

A CTRModel-shaped model is built here with the reference's attribute layout
(CTRModel: rep_encoder / seq_encoder / linear, models.py:251-257; the encoder
begins each layer with ``residual = x; x = norm1[i](x)`` on ``x.unsqueeze(0)``
and calls ``moe[i](x)`` after norm2, models.py:208-249; SMoE: experts of
fc1/fc2, gate, k, models.py:96-107).  The b200 forward must equal, bit for
bit, the same model run step by step with this package's unfused calls:
K1 + K2, then ATen's LayerNorm, then the b200 SMoE -- so the fused norm1,
the hooks and the extension plumbing change nothing but the launches.
"""

import types

import pytest

from test_gpu_module import _setup

pytestmark = pytest.mark.gpu


def _model(torch, nn, F, rep, attn_mode, seed=0):
    D, FF, E = 512, 1024, 8
    seen = {}

    class Expert(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1, self.fc2 = nn.Linear(D, FF), nn.Linear(FF, D)

    class Gate(nn.Module):
        def __init__(self):
            super().__init__()
            self.w_g, self.k = nn.Linear(D, E), 2

        def forward(self, x):
            probs = torch.softmax(self.w_g(x), dim=-1)
            score, idx = torch.topk(probs, self.k, dim=-1)
            return idx, score, probs

    class Moe(nn.Module):
        def __init__(self):
            super().__init__()
            self.experts = nn.ModuleList([Expert() for _ in range(E)])
            self.gate, self.k, self.num_experts = Gate(), 2, E

        def forward(self, x):
            raise AssertionError("the torch SMoE must not run in b200 mode")

    class Encoder(nn.Module):
        def __init__(self):
            super().__init__()
            self.attn_mode, self.num_layers = attn_mode, 2
            self.norm1 = nn.ModuleList([nn.LayerNorm(D) for _ in range(2)])
            self.norm2 = nn.ModuleList([nn.LayerNorm(D) for _ in range(2)])
            self.proj = nn.ModuleList([nn.Linear(D, D) for _ in range(2)])
            self.moe = nn.ModuleList([Moe() for _ in range(2)])

        def forward(self, x, extension):
            seen["extension"] = extension
            x = x.unsqueeze(0)
            loss = 0.0
            for i in range(self.num_layers):
                residual = x
                x = self.norm1[i](x)
                if "mask" in extension:
                    a = F.scaled_dot_product_attention(x[:, None], x[:, None], x[:, None],
                                                       attn_mask=extension["mask"])[:, 0]
                else:
                    a = x
                x = residual + self.proj[i](a)
                residual = x
                x = self.norm2[i](x)
                m, l = self.moe[i](x)
                x = residual + m
                loss = loss + l
            return x, loss

    class Ctr(nn.Module):
        def __init__(self):
            super().__init__()
            self.rep_encoder, self.seq_encoder, self.linear = rep, Encoder(), nn.Linear(D, 1)

        def forward(self, batch):
            raise AssertionError("the reference CTRModel body must not run in b200 mode")

    torch.manual_seed(seed)
    model = Ctr()
    model.seq_encoder.to(rep.emb.weight.device, torch.bfloat16)
    model.linear.to(rep.emb.weight.device, torch.bfloat16)
    with torch.no_grad():
        for n in list(model.seq_encoder.norm1) + list(model.seq_encoder.norm2):
            n.weight.add_(0.1 * torch.randn_like(n.weight))
            n.bias.add_(0.05 * torch.randn_like(n.bias))
    return model.eval(), Moe, Ctr, seen


@pytest.mark.parametrize("attn_mode", ["sdpa", "flash_varlen"])
def test_ctr_forward_b200_equals_unfused_steps(cuda_device, attn_mode):
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from baidu_cti_grab_b200 import ctr_boundary
    from baidu_cti_grab_b200.rep_encoder import rep_encoder_forward

    rep, batch, batch_np = _setup(torch, cuda_device, users=24, seed=41)
    rep.fuse_mode = "b200"
    model, Moe, Ctr, seen = _model(torch, nn, F, rep, attn_mode)
    ctr_boundary.install_ctr(types.SimpleNamespace(CTRModel=Ctr, SMoE=Moe))
    enc = model.seq_encoder
    norm0 = enc.norm1[0]
    calls = []
    hook = norm0.register_forward_hook(lambda *a: calls.append(1))
    with torch.no_grad():
        logits, loss = model(batch)
    hook.remove()
    assert not calls  # layer 0's norm1 came from the GEMM epilogue
    assert enc.norm1[0] is norm0 and not ctr_boundary.b200_encoder_active()
    n_items = int(batch_np["user_offsets"][-1])
    lengths = batch_np["user_offsets"][1:] - batch_np["user_offsets"][:-1]
    ext = seen["extension"]
    if attn_mode == "flash_varlen":
        assert ext["max_seqlen"] == int(lengths.max())
        assert ext["cu_seqlens"].dtype == torch.int32 and ext["cu_seqlens"].is_cuda
    else:
        assert ext["mask"].shape == (1, 1, n_items, n_items)

    with torch.no_grad():
        x = rep_encoder_forward(rep, batch)  # unfused K2
        uo = batch["user_offsets"]
        if attn_mode == "flash_varlen":
            extension = {"cu_seqlens": uo.to(torch.int32), "max_seqlen": int(lengths.max())}
        else:
            extension = {"mask": ctr_boundary.causal_user_mask(uo, n_items)[None, None]}
        with ctr_boundary._encoder_b200():
            encoded, want_loss = enc(x=x, extension=extension)
        want = torch.clamp(model.linear(encoded.reshape(-1, 512)), min=-15.0, max=15.0)
    assert logits.shape == (n_items, 1)
    assert torch.equal(logits, want) and torch.equal(loss, want_loss)


def test_ctr_forward_b200_with_host_user_offsets(cuda_device):
    """user_offsets left on the host (the collate's output before
    move_batch_to_device): same result, no device read for max_seqlen."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from baidu_cti_grab_b200 import ctr_boundary

    rep, batch, batch_np = _setup(torch, cuda_device, users=12, seed=42)
    rep.fuse_mode = "b200"
    model, Moe, Ctr, seen = _model(torch, nn, F, rep, "flash_varlen", seed=1)
    ctr_boundary.install_ctr(types.SimpleNamespace(CTRModel=Ctr, SMoE=Moe))
    with torch.no_grad():
        on_dev = model(batch)
        host = dict(batch)
        host["user_offsets"] = batch["user_offsets"].cpu()
        on_host = model(host)
    assert torch.equal(on_dev[0], on_host[0]) and torch.equal(on_dev[1], on_host[1])
    assert seen["extension"]["cu_seqlens"].is_cuda
