"""install() on the reference's own ``models`` module: the real RepEncoder,
TransformerEncoder, SMoE and CTRModel classes (models.py:14-297).

Runs where the reference checkout can be imported: set RB_REFERENCE_DIR to
it (the directory holding models.py); skipped otherwise.  There is no GPU
here, so these tests check on the CPU what does not need one:

* after install(), the reference's own fuse modes give bit-identical outputs;
* fuse mode "b200" on CPU tensors raises (no silent fallback);
* the b200 CTRModel forward, with the two device calls replaced by stand-ins
  that compute the reference's own math (the torch RepEncoder + LayerNorm,
  the torch SMoE), reproduces the reference's CTRModel output bit for bit:
  layer 0's norm1 is taken from the stand-in (the encoder never calls it),
  the sdpa mask is built without a host read, every SMoE layer goes through
  the b200 hook, and the modules are left as they were.

load_model() builds the full 5M-row table (10 GB in fp32); these tests build
the same classes with a 2000-row table instead.
"""

import os
import sys

import numpy as np
import pytest

REF = os.environ.get("RB_REFERENCE_DIR")
pytestmark = pytest.mark.skipif(not REF or not os.path.exists(os.path.join(REF or "", "models.py")),
                                reason="set RB_REFERENCE_DIR to a reference checkout to run")


@pytest.fixture(scope="module")
def models():
    pytest.importorskip("torch")
    sys.path.insert(0, REF)
    try:
        import models as m
    finally:
        sys.path.remove(REF)
    return m


def _batch(torch, users=7, seed=3):
    from baidu_cti_grab_b200 import synth

    cfg = synth.WorkloadConfig("dropin", 70, "float32", users, 1, 6, "uniform1-4", 1.1)
    b = synth.make_batch(cfg, seed=seed)
    out = {"user_offsets": torch.from_numpy(np.asarray(b["user_offsets"], dtype=np.int64))}
    for s in range(1, 29):
        v, o = b[s]
        out[s] = [torch.from_numpy(np.asarray(v, dtype=np.int64)), torch.from_numpy(np.asarray(o, dtype=np.int64))]
    return out


def _model(torch, models, seed=0):
    torch.manual_seed(seed)
    rep = models.RepEncoder(vocab_size=28 * 70 + 1, emb_dim=512, padding_idx=0, slot_num=28, d_model=512,
                            fuse_mode="torch")
    enc = models.TransformerEncoder(d_model=512, n_heads=8, num_layers=2, dim_ff=256, act="relu", attn_mode="sdpa")
    model = models.CTRModel(rep, enc, d_model=512)
    with torch.no_grad():  # non-trivial LayerNorm affine parameters
        for norm in list(enc.norm1) + [rep.input_norm]:
            norm.weight.add_(0.1 * torch.randn_like(norm.weight))
            norm.bias.add_(0.05 * torch.randn_like(norm.bias))
    return model.eval()


def test_install_keeps_reference_modes(models):
    import torch
    from baidu_cti_grab_b200.rep_encoder import install

    model = _model(torch, models)
    batch = _batch(torch)
    with torch.no_grad():
        before = {m: None for m in ("torch", "cat_free_ref")}
        for mode in before:
            model.rep_encoder.fuse_mode = mode
            before[mode] = model(batch)
        install(models)
        install(models)  # idempotent
        assert models.RepEncoder._b200_installed and models.CTRModel._b200_installed
        assert models.SMoE._b200_installed
        for mode, (logits, loss) in before.items():
            model.rep_encoder.fuse_mode = mode
            got_logits, got_loss = model(batch)
            assert torch.equal(got_logits, logits) and torch.equal(got_loss, loss)


def test_b200_mode_on_cpu_raises(models):
    import torch
    from baidu_cti_grab_b200.rep_encoder import install

    install(models)
    model = _model(torch, models)
    model.rep_encoder.fuse_mode = "b200"
    with torch.no_grad(), pytest.raises(RuntimeError):
        model(_batch(torch))
    with torch.no_grad(), pytest.raises(RuntimeError):
        model.rep_encoder(_batch(torch))


def test_b200_ctr_forward_wiring_reproduces_reference(models, monkeypatch):
    import torch
    import torch.nn.functional as F
    from baidu_cti_grab_b200 import ctr_boundary, smoe
    from baidu_cti_grab_b200.rep_encoder import install

    install(models)
    model = _model(torch, models, seed=1)
    batch = _batch(torch, users=9, seed=5)
    rep, enc = model.rep_encoder, model.seq_encoder
    with torch.no_grad():
        rep.fuse_mode = "torch"
        want_logits, want_loss = model(batch)

    # the reference's own RepEncoder (torch mode) and SMoE, standing in for the kernels
    ref_rep_forward = models.RepEncoder.forward
    ref_moe_forward = models.SMoE.forward
    calls = {"rep": [], "moe": 0}

    def rep_standin(module, b, norm=None):
        saved, module.fuse_mode = module.fuse_mode, "torch"
        try:
            out = ref_rep_forward(module, b)
        finally:
            module.fuse_mode = saved
        calls["rep"].append(norm)
        if norm is None:
            return out
        return out, F.layer_norm(out, norm.normalized_shape, norm.weight, norm.bias, norm.eps)

    def moe_standin(module, x):
        calls["moe"] += 1
        assert ctr_boundary.b200_encoder_active()
        ctr_boundary._ACTIVE.on = False  # the reference's SMoE may not re-enter the hook
        try:
            return ref_moe_forward(module, x)
        finally:
            ctr_boundary._ACTIVE.on = True

    monkeypatch.setattr(ctr_boundary, "rep_encoder_forward", rep_standin)
    monkeypatch.setattr(smoe, "smoe_forward", moe_standin)
    norm0 = enc.norm1[0]
    norm0_calls = []
    hook = norm0.register_forward_hook(lambda *a: norm0_calls.append(1))
    try:
        with torch.no_grad():
            rep.fuse_mode = "b200"
            logits, loss = model(batch)
            rep.fuse_mode = "torch"
            again_logits, _ = model(batch)
    finally:
        hook.remove()
    assert torch.equal(logits, want_logits) and torch.equal(loss, want_loss)
    assert torch.equal(again_logits, want_logits)
    assert calls["rep"] == [norm0]                  # one RepEncoder call, layer 0's norm1 fused into it
    assert calls["moe"] == enc.num_layers           # every SMoE layer through the b200 hook
    assert len(norm0_calls) == 1                    # the torch-mode rerun only: b200 never called norm1[0]
    assert enc.norm1[0] is norm0 and not ctr_boundary.b200_encoder_active()
    assert "forward" not in vars(rep)


def test_causal_user_mask_matches_reference(models):
    import torch
    from baidu_cti_grab_b200.ctr_boundary import causal_user_mask

    model = _model(torch, models)
    uo = torch.tensor([0, 3, 3, 4, 9, 12])
    assert torch.equal(causal_user_mask(uo, 12), model.get_sequence_causal_mask(uo))
