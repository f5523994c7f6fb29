"""Record ATen's CUDA LayerNorm on seeded rows: tests/golden/ln_aten_cuda.npz.

Run on a machine with a B200 (the fixture pins the oracle's LayerNorm to the
GPU kernel that the reference's nn.LayerNorm runs there, models.py:21,45):

    python tests/golden/gen_golden_aten_cuda.py [out.npz]

For every case it stores the rows x, gamma, beta and what
``torch.native_layer_norm`` returns on the GPU: y, mean and rstd.  rstd comes
from CUDA's rsqrtf, a hardware approximation that the CPU cannot evaluate, so
the fixture also carries torch.rsqrt (the same rsqrtf) on a window of +-64
fp32 neighbours of each row's fp64 var + eps; the CPU test looks the oracle's
own fl(var + eps) up in that window.  The rows imitate the RepEncoder's
pooled rows (sums of 1-4 table rows ~N(0, 0.02), rounded to the row dtype)
plus rows with a large common offset, widely varying magnitudes, mostly zero
and all-zero rows, and row widths of 1, 6, 28 and 32 slots of 512.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (tag, row dtype, slots, kind, rows)
CASES = [
    ("bf16_s28_pooled", "bf16", 28, "pooled", 6),
    ("bf16_s28_offset", "bf16", 28, "offset", 2),
    ("bf16_s28_wide", "bf16", 28, "wide", 2),
    ("bf16_s28_sparse", "bf16", 28, "sparse", 2),
    ("bf16_s28_const", "bf16", 28, "const", 1),
    ("bf16_s6_pooled", "bf16", 6, "pooled", 4),
    ("bf16_s1_pooled", "bf16", 1, "pooled", 4),
    ("bf16_s32_pooled", "bf16", 32, "pooled", 2),
    ("f32_s28_pooled", "f32", 28, "pooled", 3),
    ("f32_s28_offset", "f32", 28, "offset", 1),
]
WINDOW = 64


def make_rows(rng, rows, slots, kind, torch_dtype):
    h = slots * 512
    if kind == "pooled":
        k = rng.integers(1, 5, size=(rows, slots, 1))
        acc = np.zeros((rows, slots, 512), np.float32)
        for j in range(4):
            v = torch.from_numpy((0.02 * rng.standard_normal((rows, slots, 512))).astype(np.float32))
            acc += np.where(j < k, v.to(torch_dtype).float().numpy(), 0).astype(np.float32)
        x = acc.reshape(rows, h)
    elif kind == "offset":
        x = (1.0 + 0.01 * rng.standard_normal((rows, h))).astype(np.float32)
    elif kind == "wide":
        x = (rng.standard_normal((rows, h)) * np.exp(rng.uniform(-6, 6, size=(rows, 1)))).astype(np.float32)
    elif kind == "sparse":
        x = (0.02 * rng.standard_normal((rows, h))).astype(np.float32)
        x[:, rng.random(h) < 0.7] = 0.0
        x[: max(1, rows // 2)] = 0.0  # all-zero rows: var = 0
    elif kind == "const":
        x = np.full((rows, h), 0.3, np.float32)
    else:
        raise ValueError(kind)
    return x


def main(out_path: str) -> None:
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(20260)
    res = {"cases": np.array([c[0] for c in CASES]), "eps": np.array([1e-5], np.float32)}
    for tag, dt, slots, kind, rows in CASES:
        h = slots * 512
        tdt = torch.bfloat16 if dt == "bf16" else torch.float32
        x = torch.from_numpy(make_rows(rng, rows, slots, kind, tdt)).to(dev).to(tdt)
        g = torch.from_numpy((1 + 0.1 * rng.standard_normal(h)).astype(np.float32)).to(dev).to(tdt)
        b = torch.from_numpy((0.05 * rng.standard_normal(h)).astype(np.float32)).to(dev).to(tdt)
        y, mean, rstd = torch.native_layer_norm(x, [h], g, b, 1e-5)
        s64 = x.double().var(dim=1, unbiased=False) + 1e-5
        k = torch.arange(-WINDOW, WINDOW + 1, device=dev, dtype=torch.int32)
        cand = (s64.float().view(torch.int32)[:, None] + k[None, :]).view(torch.float32)
        rsq = torch.rsqrt(cand)
        torch.cuda.synchronize()

        def host(t):
            return t.view(torch.int16).cpu().numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.cpu().numpy()

        res[f"{tag}_slots"] = np.array([slots])
        res[f"{tag}_dtype"] = np.array(dt)
        res[f"{tag}_x"] = host(x)
        res[f"{tag}_gamma"] = host(g)
        res[f"{tag}_beta"] = host(b)
        res[f"{tag}_y"] = host(y)
        res[f"{tag}_mean"] = mean.float().cpu().numpy().reshape(-1)
        res[f"{tag}_rstd"] = rstd.float().cpu().numpy().reshape(-1)
        res[f"{tag}_rsqrt_arg"] = cand.cpu().numpy()
        res[f"{tag}_rsqrt_val"] = rsq.cpu().numpy()
    res["torch_version"] = np.array(torch.__version__)
    res["device"] = np.array(torch.cuda.get_device_name(dev))
    np.savez_compressed(out_path, **res)
    print(f"wrote {out_path} ({os.path.getsize(out_path)} bytes) with torch {torch.__version__}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ln_aten_cuda.npz"))
