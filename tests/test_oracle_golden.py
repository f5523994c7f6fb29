"""The CPU oracle against the golden vectors produced by the reference itself.

tests/golden/gen_golden.py ran the reference's RepEncoder (ATen CPU) and its
Triton kernels (interpreter) on these inputs.  The oracle must reproduce:
pooled rows, every quantiser and the int8 GEMM + scaled epilogue bit for bit.

The oracle's LayerNorm follows ATen's CUDA kernel, the one the reference runs
on the GPU; tests/golden/gen_golden_aten_cuda.py recorded that kernel on a
B200 (ln_aten_cuda.npz) and the oracle must reproduce its mean, rstd and
output rows bit for bit.  ATen's CPU LayerNorm reduces in another order, so
against the CPU-recorded RepEncoder fixtures the LayerNorm rows may differ by
one bf16 ulp on a few elements and the end-to-end int8 by one step there.
"""

import numpy as np
import pytest

from conftest import golden_rep, load_golden
from oracle import oracle as O


@pytest.mark.parametrize("name", ["rep_bf16.npz", "rep_f32.npz"])
def test_rep_pooled_and_quantisers(name):
    dt, table, batch, gamma, beta, eps, z = golden_rep(name)
    q, sc, pooled, ln = O.rep_forward(table, dt, batch, gamma, beta, eps, intermediates=True)
    tof = O.bf16_bits_to_f32 if dt == "bfloat16" else (lambda a: a.astype(np.float32))
    pref, lref = tof(z["pooled_ref"]), tof(z["ln_ref"])
    assert np.array_equal(pooled.view(np.uint32), pref.view(np.uint32))
    # quantisers given the reference's own LayerNorm output: bit-exact
    q2, s2 = O.quant_dynamic_v2(lref)
    assert np.array_equal(q2, z["q_dyn_ref"]) and np.array_equal(s2, z["scale_dyn_ref"])
    q1, s1 = O.quant_rows_v1(lref)
    assert np.array_equal(q1, z["q_v1_ref"]) and np.array_equal(s1, z["scale_v1_ref"])
    assert np.array_equal(O.quant_static_v2(lref, z["static_scale"][0]), z["q_static_ref"])
    # LayerNorm: ATen CUDA's order vs ATen CPU's -- bf16 rows agree except for rare 1-ulp ties
    if dt == "bfloat16":
        diff = ln != lref
        assert diff.mean() < 1e-3
        ulp = np.abs(ln.view(np.int32) - lref.view(np.int32)) >> 16
        assert ulp.max() <= 1
    else:
        assert np.abs(ln - lref).max() < 1e-5
    dq = np.abs(q.astype(np.int32) - z["q_dyn_ref"].astype(np.int32))
    assert dq.max() <= 1 and (dq != 0).mean() < 1e-3


@pytest.mark.parametrize("name", ["bf16", "f32", "f16"])
def test_quant_edges(name):
    z = load_golden("quant_edges.npz")
    if name == "bf16":
        x = O.bf16_bits_to_f32(z["x_bf16"])
    elif name == "f16":
        x = z["x_f16"].view(np.float16).astype(np.float32)
    else:
        x = z["x_f32"]
    q, s = O.quant_dynamic_v2(x)
    assert np.array_equal(q, z[f"q_dyn_{name}"]) and np.array_equal(s, z[f"s_dyn_{name}"])
    q, s = O.quant_rows_v1(x)
    assert np.array_equal(q, z[f"q_v1_{name}"]) and np.array_equal(s, z[f"s_v1_{name}"])
    assert np.array_equal(O.quant_static_v2(x, z["static_scale"][0]), z[f"q_static_{name}"])


@pytest.mark.parametrize("tag", ["k14336", "ktail"])
def test_gemm_and_epilogue(tag):
    g = load_golden("gemm.npz")
    a, b = g[f"{tag}_a"], g[f"{tag}_qweight_nk"]
    acc = O.gemm_i8_i32(a, b)
    assert np.array_equal(acc, g[f"{tag}_acc_ref"])
    assert np.array_equal(O.gemm_i8_i32_loops(a, b), acc)
    bias = O.bf16_bits_to_f32(g[f"{tag}_bias"])
    out = O.scaled_epilogue(acc, g[f"{tag}_sa"], g[f"{tag}_wscale"], bias, "float32")
    assert np.array_equal(out, g[f"{tag}_out_dyn_ref"])
    out = O.scaled_epilogue(acc, g[f"{tag}_static_scale"], g[f"{tag}_wscale"], None, "float32", sa_per_row=False)
    assert np.array_equal(out, g[f"{tag}_out_static_ref"])


def test_weight_quant_restatement():
    """quantize_weight_per_channel arithmetic (w8a8_preprocess.py:49-52) in numpy == the fixture."""
    g = load_golden("gemm.npz")
    w = g["ktail_weight_f32"]
    amax = np.maximum(np.abs(w).max(axis=1), np.float32(1e-8)).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -128, 127).astype(np.int8)
    assert np.array_equal(q, g["ktail_qweight_nk"])
    assert np.array_equal(scale, g["ktail_wscale"])


def test_oracle_planted_error_is_caught():
    """A one-ulp change in a table row must change the oracle's pooled output (the check has teeth)."""
    dt, table, batch, gamma, beta, eps, z = golden_rep("rep_bf16.npz")
    bad = table.copy()
    ids = batch[1][0]
    row = int([i for i in ids if 0 < i < table.shape[0]][0])
    bad[row, 3] ^= 1
    _, _, pooled, _ = O.rep_forward(bad, dt, batch, gamma, beta, eps, intermediates=True)
    assert not np.array_equal(pooled, O.bf16_bits_to_f32(z["pooled_ref"]))


def _aten_cuda_cases():
    z = load_golden("ln_aten_cuda.npz")
    return z, [str(c) for c in z["cases"]]


@pytest.mark.parametrize("case", _aten_cuda_cases()[1])
def test_layernorm_matches_aten_cuda(case):
    """Mean, rstd and every LayerNorm output element equal ATen's CUDA kernel.
    rstd = rsqrtf(var + eps) is the GPU's approximation: the fixture carries its
    values on a window of fp32 arguments, in which the oracle's own
    fl(var + eps) must be found and must give ATen's rstd."""
    z, _ = _aten_cuda_cases()
    bf = str(z[f"{case}_dtype"]) == "bf16"
    tof = O.bf16_bits_to_f32 if bf else (lambda a: a.astype(np.float32))
    x, g, b = tof(z[f"{case}_x"]), tof(z[f"{case}_gamma"]), tof(z[f"{case}_beta"])
    eps = float(z["eps"][0])
    args, vals = z[f"{case}_rsqrt_arg"], z[f"{case}_rsqrt_val"]

    def rsqrt(v):
        out = np.empty_like(v)
        for r in range(len(v)):
            hit = np.nonzero(args[r] == v[r])[0]
            assert hit.size == 1, f"row {r}: fl(var + eps) = {v[r]!r} outside the recorded window"
            out[r] = vals[r, hit[0]]
        return out

    y, mean, rstd = O.layernorm_rows(x, g, b, eps, "bfloat16" if bf else "float32", rsqrt=rsqrt)
    assert np.array_equal(mean, z[f"{case}_mean"])
    assert np.array_equal(rstd, z[f"{case}_rstd"])
    assert np.array_equal(y.view(np.uint32), tof(z[f"{case}_y"]).view(np.uint32))
    # the CPU-only default (correctly rounded 1/sqrt) is within 2 ulp of rsqrtf
    _, _, r_cpu = O.layernorm_rows(x, g, b, eps, "float32")
    assert np.abs(r_cpu.view(np.int32).astype(np.int64) - rstd.view(np.int32)).max() <= 2


def test_layernorm_fixture_is_order_sensitive():
    """The recorded means are not order-free: the correctly rounded mean (a
    float64 sum) differs from ATen's on some rows, so reproducing the fixture
    needs ATen's exact reduction order, not just an accurate one."""
    z, cases = _aten_cuda_cases()
    moved = 0
    for case in cases:
        bf = str(z[f"{case}_dtype"]) == "bf16"
        x = (O.bf16_bits_to_f32 if bf else (lambda a: a.astype(np.float32)))(z[f"{case}_x"])
        h = x.shape[1]
        mean_other = (x.astype(np.float64).sum(axis=1) / h).astype(np.float32)
        moved += int(np.sum(mean_other != z[f"{case}_mean"]))
    assert moved > 0
