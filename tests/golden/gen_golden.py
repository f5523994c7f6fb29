"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference is checked out (read-only), naming its directory:

    TRITON_INTERPRET=1 python tests/golden/gen_golden.py REFERENCE_DIR
    (or set RB_REFERENCE_DIR instead of passing the argument)

It imports the reference's own modules (models.RepEncoder, the W8A8 Triton
kernels, the v1 quantisation kernels) and runs them on CPU:

* RepEncoder.forward in fp32 and bf16 (ATen CPU EmbeddingBag / cat /
  LayerNorm); the pooled slot outputs and the LayerNorm output are captured
  with forward hooks on ``rep.emb`` and ``rep.input_norm``.
* The Triton kernels run under the Triton interpreter (TRITON_INTERPRET=1).
  The interpreter cannot evaluate ``tl.extra.cuda.libdevice.round``; it is
  given C ``roundf`` semantics (round half away from zero, evaluated in
  float64 where x + 0.5 is exact for every fp32 x) -- the meaning of the
  ``__nv_roundf`` symbol that the reference binds.
* The interpreter's fp32 -> bf16 cast truncates, unlike the GPU's RNE, so the
  scaled GEMM is asked for fp32 output; the fixtures hold fp32.

Nothing here is needed at test time: the tests read only the .npz files.
"""

from __future__ import annotations

import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RB_REFERENCE_DIR", "")
if not REF or not os.path.isdir(REF):
    sys.exit("usage: gen_golden.py REFERENCE_DIR (or RB_REFERENCE_DIR): the reference checkout to import")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REF)
sys.path.insert(0, os.path.join(REF, "quantization"))
sys.path.insert(0, REPO)

import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402


def _patch_roundf():
    lib = tl.extra.cuda.libdevice

    def round_half_away(x, _semantic=None):
        data = x.handle.data
        wide = data.astype(np.float64)
        r = (np.sign(wide) * np.floor(np.abs(wide) + 0.5)).astype(data.dtype)
        return tl.core.tensor(_interp.TensorHandle(r, x.handle.dtype.scalar), x.type)

    lib.round = round_half_away


_patch_roundf()

import models  # noqa: E402
from kernels import quantization as ref_v1  # noqa: E402
import w8a8_preprocess as ref_prep  # noqa: E402
import w8a8_triton_kernels as ref_v2  # noqa: E402

from baidu_cti_grab_b200 import synth  # noqa: E402

S, D = 28, 512


def _edge_batch(rng, n_items, rows_per_slot):
    """Batch with empty bags, padding ids (0), negative ids and ids past the vocab."""
    V = S * rows_per_slot + 1
    batch = {"user_offsets": np.array([0, n_items // 2, n_items], dtype=np.int64)}
    for s in range(1, S + 1):
        k = rng.integers(0, 6, size=n_items)
        k[0] = 0  # first item: empty bag in every slot
        if s % 3 == 0:
            k[n_items - 1] = 0  # last item empty in some slots
        offsets = np.zeros(n_items + 1, dtype=np.int64)
        np.cumsum(k, out=offsets[1:])
        vals = synth.slot_ids(rng, s, rows_per_slot, 1.1, int(offsets[-1]))
        if len(vals) >= 4:
            vals[1] = 0  # padding id
            vals[2] = -5  # clamps to 0 -> padding
            vals[3] = V + 1000  # clamps to V-1
        batch[s] = (vals, offsets)
    return batch


def _run_reference_rep(table_f32: np.ndarray, batch, gamma, beta, dtype):
    """models.RepEncoder.forward on CPU, capturing pooled slots and LN output."""
    V = table_f32.shape[0]
    rep = models.RepEncoder(vocab_size=V, emb_dim=D, padding_idx=0, slot_num=S, d_model=512,
                            fuse_mode="torch")
    with torch.no_grad():
        rep.emb.weight.copy_(torch.from_numpy(table_f32))
        rep.input_norm.weight.copy_(torch.from_numpy(gamma))
        rep.input_norm.bias.copy_(torch.from_numpy(beta))
    rep = rep.to(dtype)
    pooled, ln = [], []
    rep.emb.register_forward_hook(lambda m, i, o: pooled.append(o.detach().clone()))
    rep.input_norm.register_forward_hook(lambda m, i, o: ln.append(o.detach().clone()))
    tb = {"user_offsets": torch.from_numpy(batch["user_offsets"])}
    for s in range(1, S + 1):
        tb[s] = (torch.from_numpy(batch[s][0]), torch.from_numpy(batch[s][1]))
    with torch.no_grad():
        out = rep(tb)
    return torch.cat(pooled, dim=1), ln[0], out, rep


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def gen_rep(path, dtype, n_items, rows_per_slot, seed):
    rng = np.random.default_rng(seed)
    batch = _edge_batch(rng, n_items, rows_per_slot)
    V = S * rows_per_slot + 1
    table = synth.make_table_numpy(V, D, seed=seed, std=0.02, dtype="float32")
    # a few heavy rows so that some items saturate the int8 range unevenly
    table[5] *= 40.0
    gamma = (1.0 + 0.1 * rng.standard_normal(S * D)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(S * D)).astype(np.float32)
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float32
    pooled, ln, _, rep = _run_reference_rep(table, batch, gamma, beta, tdt)
    # the reference's own dynamic per-token quantiser (Triton, interpreted)
    q2, s2 = ref_v2.dynamic_per_token_quantize_activation(ln)
    q1, s1 = _v1_quant(ln)
    static_scale = torch.tensor([float(ln.float().abs().max()) / 127.0], dtype=torch.float32)
    qs = ref_v2.static_quantize_activation(ln, static_scale)
    arrays = {
        "table": _bits(rep.emb.weight.detach()),
        "gamma": _bits(rep.input_norm.weight.detach()),
        "beta": _bits(rep.input_norm.bias.detach()),
        "user_offsets": batch["user_offsets"],
        "pooled_ref": _bits(pooled),
        "ln_ref": _bits(ln),
        "q_dyn_ref": q2.numpy(),
        "scale_dyn_ref": s2.numpy(),
        "q_v1_ref": q1.numpy(),
        "scale_v1_ref": s1.numpy(),
        "static_scale": static_scale.numpy(),
        "q_static_ref": qs.numpy(),
        "eps": np.array([rep.input_norm.eps], dtype=np.float64),
    }
    for s in range(1, S + 1):
        arrays[f"values_{s}"] = batch[s][0]
        arrays[f"offsets_{s}"] = batch[s][1]
    np.savez_compressed(path, dtype=np.array(dtype), **arrays)
    print("wrote", path, {k: v.shape for k, v in arrays.items() if hasattr(v, "shape") and v.size > 64})


def _v1_quant(x: torch.Tensor):
    """kernels/quantization.py:243-268 without the is_cuda guard (interpreter on CPU)."""
    x = x.contiguous()
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=torch.int8)
    scale = torch.empty((rows,), dtype=torch.float32)
    block_k = ref_v1._next_power_of_2(cols)
    ref_v1._quantize_rows_int8_kernel[(rows,)](x, q, scale, rows, cols, x.stride(0), x.stride(1),
                                                q.stride(0), q.stride(1), BLOCK_K=block_k, num_warps=8)
    return q, scale


def gen_quant_edges(path, seed):
    """Quantiser edge rows: zeros, exact .5 ties, one dominant value, tiny values."""
    rng = np.random.default_rng(seed)
    K = 1000  # not a power of two: exercises the kernels' masking
    x = (0.05 * rng.standard_normal((8, K))).astype(np.float32)
    x[0] = 0.0  # amax clamp (1e-8 / 1e-8*127 paths)
    # row 1: values that land exactly on k + 0.5 after scaling by 127/amax with amax = 127
    x[1] = (np.arange(K) % 255 - 127).astype(np.float32) + 0.5
    x[1, 0] = 127.0
    x[1] = np.clip(x[1], -127.0, 127.0)
    x[2, 17] = 30.0  # one dominant value
    x[3] = (1e-10 * rng.standard_normal(K)).astype(np.float32)  # amax below 1e-8
    x[4] = -np.abs(x[4])  # all negative
    x[5] = np.abs(x[5])
    x[6, :] = x[6, :] * 1e4
    xb = torch.from_numpy(x).to(torch.bfloat16)
    x16 = torch.from_numpy(x).to(torch.float16)
    arrays = {"x_bf16": _bits(xb), "x_f32": x, "x_f16": x16.numpy().view(np.uint16)}
    for name, t in (("bf16", xb), ("f32", torch.from_numpy(x)), ("f16", x16)):
        q2, s2 = ref_v2.dynamic_per_token_quantize_activation(t)
        q1, s1 = _v1_quant(t)
        st = torch.tensor([0.0123], dtype=torch.float32)
        qs = ref_v2.static_quantize_activation(t, st)
        arrays[f"q_dyn_{name}"] = q2.numpy()
        arrays[f"s_dyn_{name}"] = s2.numpy()
        arrays[f"q_v1_{name}"] = q1.numpy()
        arrays[f"s_v1_{name}"] = s1.numpy()
        arrays[f"q_static_{name}"] = qs.numpy()
    arrays["static_scale"] = np.array([0.0123], dtype=np.float32)
    np.savez_compressed(path, **arrays)
    print("wrote", path)


def gen_gemm(path, seed):
    """int8 GEMM + scaled epilogue through the reference Triton kernels (interpreted)."""
    rng = np.random.default_rng(seed)
    cases = {}
    for tag, (M, K, N) in {"k14336": (6, 14336, 32), "ktail": (5, 592, 48)}.items():
        W = torch.from_numpy((rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32))
        qw = ref_prep.quantize_weight_per_channel(W)  # qweight_t = [K,N] view of [N,K] storage
        a = torch.from_numpy(rng.integers(-128, 128, size=(M, K), dtype=np.int64).astype(np.int8))
        a[0, :] = 127
        a[1, :] = -128
        sa = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=M).astype(np.float32))
        bias = torch.from_numpy((0.02 * rng.standard_normal(N)).astype(np.float32)).to(torch.bfloat16)
        acc = ref_v2.int8_mm_no_scale(a, qw, out_dtype=torch.int32)
        out_dyn = ref_v2.w8a8_scaled_mm(a, qw, sa, bias=bias, out_dtype=torch.float32, static_act=False)
        sst = torch.tensor([0.004], dtype=torch.float32)
        out_st = ref_v2.w8a8_scaled_mm(a, qw, sst, bias=None, out_dtype=torch.float32, static_act=True)
        if K * N <= 1 << 16:  # the fp32 weight is stored only for the small case
            cases[f"{tag}_weight_f32"] = W.numpy()
        cases[f"{tag}_qweight_nk"] = qw.qweight_t.t().contiguous().numpy()
        cases[f"{tag}_wscale"] = qw.scale.numpy()
        cases[f"{tag}_a"] = a.numpy()
        cases[f"{tag}_sa"] = sa.numpy()
        cases[f"{tag}_bias"] = _bits(bias)
        cases[f"{tag}_acc_ref"] = acc.numpy()
        cases[f"{tag}_out_dyn_ref"] = out_dyn.numpy()
        cases[f"{tag}_static_scale"] = sst.numpy()
        cases[f"{tag}_out_static_ref"] = out_st.numpy()
    np.savez_compressed(path, **cases)
    print("wrote", path)


if __name__ == "__main__":
    torch.manual_seed(0)
    gen_rep(os.path.join(HERE, "rep_bf16.npz"), "bfloat16", n_items=10, rows_per_slot=8, seed=1)
    gen_rep(os.path.join(HERE, "rep_f32.npz"), "float32", n_items=4, rows_per_slot=4, seed=2)
    gen_quant_edges(os.path.join(HERE, "quant_edges.npz"), seed=3)
    gen_gemm(os.path.join(HERE, "gemm.npz"), seed=4)
