"""RepEncoder on B200: the reference's models.RepEncoder (models.py:14-48) with
the forward pass replaced by two sm_100a kernels.

    K1  rb_rep_gather_ln_quant   28-slot embedding-bag gather + fp32 sum-pool +
                                 concat + LayerNorm + int8 quantisation; the
                                 [N, 14336] row never reaches HBM
    K2  rb_w8a8_gemm             tcgen05 int8 GEMM [N,14336] x [14336,512] with
                                 the dequant / bias epilogue fused

``rep_encoder_forward(rep, batch)`` works on any module with the reference's
attribute layout -- ``emb`` (nn.EmbeddingBag, mode='sum', padding_idx=0),
``input_norm`` (nn.LayerNorm), ``linear`` (nn.Linear, or the reference's
quantised ``StaticQuantizedLinear`` with ``qweight_t``/``weight_scale``/
``static_act_scale``/``bias`` buffers) and ``slot_num`` -- so it serves the
reference's own module instances unchanged.  ``install(models)`` adds the
``fuse_mode == "b200"`` branch to the reference's RepEncoder.forward.

Activation quantisation: with an fp ``nn.Linear`` the weight is quantised per
output channel once (cached until the weight changes) and activations are
quantised per token (dynamic, the default).  With the quantised checkpoint
layer (``use_quant``) the stored static per-tensor scale is used, as the
reference's StaticQuantizedLinear does.
"""

from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch
import torch.nn as nn

from . import device_ops

FUSE_MODE = "b200"


# pinned staging buffer per (device, index dtype) for host-resident slot arrays,
# with the event of the last copy out of it
_STAGING: Dict[tuple, tuple] = {}


def _stage_to_device(host: Sequence[torch.Tensor], dtype: torch.dtype, device: torch.device):
    """Copy host tensors to `device` as one contiguous transfer through a reused
    pinned buffer: one H2D copy instead of one synchronous pageable copy per
    array.  Returns the device views, in order."""
    sizes = [t.numel() for t in host]
    total = sum(sizes)
    key = (device.index, dtype)
    buf, done = _STAGING.get(key, (None, None))
    if done is not None:
        done.synchronize()  # the previous copy out of the buffer has finished
    if buf is None or buf.numel() < total:
        buf = torch.empty((max(total, 1),), dtype=dtype, pin_memory=True)
    pos = 0
    for t, n in zip(host, sizes):
        buf[pos:pos + n].copy_(t.reshape(-1))
        pos += n
    flat = torch.empty((total,), dtype=dtype, device=device)
    flat.copy_(buf[:total], non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(device))
    _STAGING[key] = (buf, done)
    return list(torch.split(flat, sizes))


def _slot_tensors(batch, slot_num: int, device: torch.device):
    """Device values/offsets of every slot: int32 when the batch holds only int32
    arrays (the packed ingestion format, half the bytes), else int64 as in the
    reference's collate.  Arrays still on the host (the reference moves a CPU
    offsets tensor to the values' device, models.py:31) travel in one staged copy."""
    arrays = []
    for i in range(slot_num):
        v, o = batch[i + 1]
        arrays.append(v if torch.is_tensor(v) else torch.as_tensor(v))
        arrays.append(o if torch.is_tensor(o) else torch.as_tensor(o))
    idx = torch.int32 if all(t.dtype == torch.int32 for t in arrays) else torch.int64
    on_host = [k for k, t in enumerate(arrays) if t.device != device]
    if on_host:
        for k, t in zip(on_host, _stage_to_device([arrays[k] for k in on_host], idx, device)):
            arrays[k] = t
    arrays = [t if t.dtype == idx and t.is_contiguous() else t.to(idx).contiguous() for t in arrays]
    return arrays[0::2], arrays[1::2]


def _quantized_weight(rep: nn.Module):
    """(w_nk int8 [N,K], w_scale [N], bias, static_scale or None) for rep.linear."""
    lin = rep.linear
    if getattr(lin, "use_quant", False):
        from .w8a8_triton_kernels import _packed_nk
        return _packed_nk(lin.qweight_t), lin.weight_scale, lin.bias, lin.static_act_scale
    w = lin.weight
    q_nk, w_scale = device_ops.cached_derived(w, "w8a8_per_channel",
                                              lambda x: device_ops.quantize_weight_per_channel(x.detach()))
    rep._b200_wcache = (None, q_nk, w_scale)
    return q_nk, w_scale, lin.bias, None


def _fusable_norm(norm, d_model: int, dtype: torch.dtype) -> bool:
    return (norm is not None and d_model == 512 and dtype in (torch.bfloat16, torch.float16, torch.float32)
            and getattr(norm, "weight", None) is not None and getattr(norm, "bias", None) is not None
            and tuple(getattr(norm, "normalized_shape", ())) == (512,))


def rep_encoder_forward(rep: nn.Module, batch, act_mode: Optional[str] = None,
                        return_intermediates: bool = False, out: Optional[torch.Tensor] = None,
                        norm: Optional[nn.Module] = None):
    """Fused B200 forward of a RepEncoder-shaped module on a reference batch dict.

    Returns rep_emb [N, d_model] in the table dtype (written into ``out`` when
    given), and with return_intermediates a dict with q, scale, pooled and ln.
    With ``norm`` (the transformer's first nn.LayerNorm(512), models.py:216-217)
    the GEMM also applies it in its epilogue (rb_w8a8_gemm_ln) and the call
    returns (rep_emb, norm(rep_emb)) -- bit-identical to running the module on
    rep_emb."""
    table = rep.emb.weight
    device = table.device
    if device.type != "cuda":
        raise RuntimeError("RepEncoder fuse_mode 'b200' expects the module on a CUDA device")
    if rep.emb.mode != "sum" or rep.emb.padding_idx not in (0, None):
        raise ValueError("fuse_mode 'b200' implements EmbeddingBag(mode='sum', padding_idx=0)")
    values, offsets = _slot_tensors(batch, rep.slot_num, device)
    w_nk, w_scale, bias, static_scale = _quantized_weight(rep)
    if act_mode is None:
        act_mode = "static" if static_scale is not None else "dynamic"
    if act_mode == "static" and static_scale is None:
        raise ValueError("act_mode 'static' needs a quantised linear with static_act_scale")
    ln = rep.input_norm
    if ln.weight is None or ln.bias is None:
        raise ValueError("fuse_mode 'b200' needs an affine LayerNorm")
    q, scale, pooled, ln_out = device_ops.rep_gather_ln_quant(
        table.detach(), values, offsets, ln.weight.detach(), ln.bias.detach(), ln.eps, act_mode=act_mode,
        static_scale=static_scale, want_pooled=return_intermediates, want_ln=return_intermediates)
    n = q.shape[0]
    if out is None:
        out = torch.empty((n, w_nk.shape[0]), dtype=table.dtype, device=device)
    elif tuple(out.shape) != (n, w_nk.shape[0]) or out.dtype != table.dtype:
        raise ValueError(f"out must be [{n}, {w_nk.shape[0]}] {table.dtype}")
    sa = scale if act_mode == "dynamic" else static_scale
    bias_d = None if bias is None else bias.detach()
    if norm is not None and _fusable_norm(norm, w_nk.shape[0], out.dtype):
        normed = torch.empty_like(out)
        device_ops.w8a8_gemm_ln(q, w_nk, sa, w_scale, out, norm.weight.detach(), norm.bias.detach(), norm.eps,
                                normed, bias=bias_d, sa_per_row=(act_mode == "dynamic"))
    else:
        device_ops.w8a8_gemm(q, w_nk, sa, w_scale, out, bias=bias_d, sa_per_row=(act_mode == "dynamic"))
        normed = None if norm is None else norm(out)
    res = out if norm is None else (out, normed)
    if return_intermediates:
        return res, {"q": q, "scale": scale, "pooled": pooled, "ln": ln_out}
    return res


class RepEncoder(nn.Module):
    """Drop-in for models.RepEncoder whose forward runs the B200 kernels.

    Constructor arguments and parameter names match the reference
    (models.py:14-22), so its state dicts load unchanged."""

    def __init__(self, vocab_size, emb_dim, padding_idx=0, slot_num=0, d_model=0, fuse_mode=FUSE_MODE,
                 act_mode: Optional[str] = None):
        super().__init__()
        self.emb = nn.EmbeddingBag(num_embeddings=vocab_size, embedding_dim=emb_dim, padding_idx=padding_idx,
                                   mode="sum")
        self.emb_dim = emb_dim
        self.slot_num = slot_num
        self.fuse_mode = fuse_mode
        self.act_mode = act_mode
        self.input_norm = nn.LayerNorm(slot_num * emb_dim)
        self.linear = nn.Linear(in_features=slot_num * emb_dim, out_features=d_model)

    def forward(self, batch):
        return rep_encoder_forward(self, batch, act_mode=self.act_mode)

    @classmethod
    def from_parts(cls, table: torch.Tensor, ln_weight: torch.Tensor, ln_bias: torch.Tensor,
                   linear_weight: torch.Tensor, linear_bias: Optional[torch.Tensor], eps: float = 1e-5,
                   act_mode: Optional[str] = None) -> "RepEncoder":
        """Wrap existing device tensors (no copy): table [V, D], LayerNorm affine
        [S*D], Linear weight [d_model, S*D] and bias [d_model]."""
        V, D = table.shape
        with torch.device("meta"):
            m = cls(V, D, 0, ln_weight.numel() // D, linear_weight.shape[0], act_mode=act_mode)
        m.emb.weight = nn.Parameter(table, requires_grad=False)
        m.input_norm.weight = nn.Parameter(ln_weight, requires_grad=False)
        m.input_norm.bias = nn.Parameter(ln_bias, requires_grad=False)
        m.input_norm.eps = eps
        m.linear.weight = nn.Parameter(linear_weight, requires_grad=False)
        m.linear.bias = None if linear_bias is None else nn.Parameter(linear_bias, requires_grad=False)
        return m


def install(models_module) -> None:
    """Add fuse_mode "b200" to a reference ``models`` module.

    After ``install(models)``, ``models.load_model(..., rep_fuse_mode="b200")``
    and ``infer.py --rep-fuse-mode b200`` run this package's kernels:
    RepEncoder.forward runs K1 + K2; CTRModel.forward, when its RepEncoder is
    in b200 mode, takes the encoder's first LayerNorm (norm1[0],
    models.py:216-217) from K2's fused epilogue, builds the attention
    extension without a mid-forward host sync and runs every SMoE layer
    through the grouped expert kernels (ctr_boundary.install_ctr).  Every
    other fuse mode keeps the reference's own code path."""
    cls = models_module.RepEncoder
    if not getattr(cls, "_b200_installed", False):
        original = cls.forward

        def forward(self, batch):
            if getattr(self, "fuse_mode", None) == FUSE_MODE:
                return rep_encoder_forward(self, batch)
            return original(self, batch)

        cls.forward = forward
        cls._b200_installed = True
    from .ctr_boundary import install_ctr

    install_ctr(models_module)
