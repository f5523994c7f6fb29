"""Shared test setup: the `gpu` marker, repo on sys.path, golden fixture loaders."""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name))


def golden_rep(name):
    """(dtype, table, batch, gamma f32, beta f32, eps, npz) from a rep_*.npz fixture."""
    from oracle import oracle as O

    z = load_golden(name)
    dt = str(z["dtype"])
    batch = {"user_offsets": z["user_offsets"]}
    for s in range(1, 29):
        batch[s] = (z[f"values_{s}"], z[f"offsets_{s}"])
    if dt == "bfloat16":
        gamma = O.bf16_bits_to_f32(z["gamma"])
        beta = O.bf16_bits_to_f32(z["beta"])
    else:
        gamma = z["gamma"].astype(np.float32)
        beta = z["beta"].astype(np.float32)
    return dt, z["table"], batch, gamma, beta, float(z["eps"][0]), z


def gpu_rsqrt(v):
    """CUDA's rsqrtf of fp32 values, evaluated on the GPU (torch.rsqrt): the
    function that gives rstd in ATen's CUDA LayerNorm and in K1.  GPU tests hand
    it to the oracle, which cannot evaluate the hardware approximation itself."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to("cuda")
    return torch.rsqrt(t).cpu().numpy()


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs an sm_100 device")
    from baidu_cti_grab_b200 import build

    build.build()
    return torch.device("cuda", 0)
