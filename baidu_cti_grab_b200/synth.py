"""Seeded synthetic RepEncoder batches in the reference's batch-dict layout.

The reference's data pipeline (Utils/data_utils.py:172-211, ``make_collate_fn``)
produces, per batch::

    batch["user_offsets"]  int64 [U+1]      item ranges of each user
    batch[s] = (values, offsets)            s = 1..28
        values   int64 [nnz_s]              feature-sign ids of slot s, item-major
        offsets  int64 [N+1]                offsets[i]..offsets[i+1] = item i's bag

The organisers' dataset is not available, so workloads are generated here from
a seed with the shapes and distributions of the benchmark configurations:

* One shared table ``[S*R + 1, 512]`` (the reference uses one shared
  ``nn.EmbeddingBag``, models.py:17).  Slot ``s`` owns rows ``1+(s-1)R .. sR``;
  row 0 is the padding row.
* Ids within a slot: ``z ~ Zipf(a)``, ``r = (z-1) mod R``, then scattered with a
  per-slot affine bijection ``r -> (r*m_s + c_s) mod R`` (m_s ~ R*frac,
  coprime with R) so that hot ids land on unrelated rows, plus the slot base.
* Bag sizes per item and slot follow the configuration's distribution.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, Tuple

import numpy as np

NUM_SLOTS = 28
EMB_DIM = 512

@dataclasses.dataclass(frozen=True)
class WorkloadConfig:
    """One synthetic workload (sizes and distributions)."""

    name: str
    rows_per_slot: int
    table_dtype: str  # "float32" | "bfloat16"
    num_users: int
    seq_lo: int
    seq_hi: int
    bag: str  # "uniform1-4" | "1+poisson1" | "heavy64"
    zipf_a: float
    num_slots: int = NUM_SLOTS
    emb_dim: int = EMB_DIM

    @property
    def num_rows(self) -> int:
        return self.num_slots * self.rows_per_slot + 1


# Benchmark configurations (names state what they are).
CPU_FP32_SMALL = WorkloadConfig("cpu-fp32-100k-rows-64-users", 100_000, "float32", 64, 1, 64,
                                "uniform1-4", 1.1)
PROD_BF16_1M = WorkloadConfig("bf16-1M-rows-1024-users", 1_000_000, "bfloat16", 1024, 1, 200,
                              "1+poisson1", 1.1)
LARGE_VOCAB_10M = WorkloadConfig("bf16-10M-rows-4096-users", 10_000_000, "bfloat16", 4096, 1, 256,
                                 "heavy64", 1.2)

CONFIGS = {c.name: c for c in (CPU_FP32_SMALL, PROD_BF16_1M, LARGE_VOCAB_10M)}


def _bag_sizes(rng: np.random.Generator, kind: str, n: int) -> np.ndarray:
    if kind == "uniform1-4":
        return rng.integers(1, 5, size=n, dtype=np.int64)
    if kind == "1+poisson1":
        return 1 + rng.poisson(1.0, size=n).astype(np.int64)
    if kind == "heavy64":
        # heavy tail on 1..64: min(64, Zipf(1.5))
        return np.minimum(64, rng.zipf(1.5, size=n)).astype(np.int64)
    raise ValueError(f"unknown bag distribution {kind!r}")


def _affine(slot: int, rows: int) -> Tuple[int, int]:
    """Per-slot bijection r -> (r*mult + add) mod rows with mult ~ rows * frac,
    frac in [0.25, 0.75) from the golden-ratio sequence, coprime with rows."""
    frac = 0.25 + 0.5 * ((0.6180339887498949 * slot) % 1.0)
    mult = max(1, int(rows * frac)) | 1
    while np.gcd(mult, rows) != 1:
        mult += 2
    add = (slot * 7919) % rows
    return mult % rows if rows > 1 else 0, add


def slot_ids(rng: np.random.Generator, slot: int, rows_per_slot: int, zipf_a: float,
             count: int) -> np.ndarray:
    """Zipf ids of one slot (1-based slot index), scattered and offset into the shared table.
    zipf_a <= 0 draws the rows uniformly instead (no hot rows: the control case)."""
    if zipf_a <= 0:
        return 1 + (slot - 1) * rows_per_slot + rng.integers(0, rows_per_slot, size=count, dtype=np.int64)
    z = rng.zipf(zipf_a, size=count).astype(np.int64)
    r = (z - 1) % rows_per_slot
    mult, add = _affine(slot, rows_per_slot)
    r = (r * mult + add) % rows_per_slot
    return 1 + (slot - 1) * rows_per_slot + r


def make_batch(cfg: WorkloadConfig, seed: int = 0, num_users: int | None = None
               ) -> Dict[object, object]:
    """Build one batch dict (numpy arrays) for ``cfg``.

    Returns ``{"user_offsets": int64[U+1], s: (values int64[nnz_s], offsets int64[N+1])}``
    for s = 1..num_slots.
    """
    rng = np.random.default_rng(seed)
    users = cfg.num_users if num_users is None else num_users
    seq = rng.integers(cfg.seq_lo, cfg.seq_hi + 1, size=users, dtype=np.int64)
    user_offsets = np.zeros(users + 1, dtype=np.int64)
    np.cumsum(seq, out=user_offsets[1:])
    n_items = int(user_offsets[-1])
    batch: Dict[object, object] = {"user_offsets": user_offsets}
    for s in range(1, cfg.num_slots + 1):
        k = _bag_sizes(rng, cfg.bag, n_items)
        offsets = np.zeros(n_items + 1, dtype=np.int64)
        np.cumsum(k, out=offsets[1:])
        values = slot_ids(rng, s, cfg.rows_per_slot, cfg.zipf_a, int(offsets[-1]))
        batch[s] = (values, offsets)
    return batch


def batch_stats(batch: Dict[object, object], num_slots: int = NUM_SLOTS) -> Tuple[int, int]:
    """(items, total ids over all slots)."""
    n = int(batch["user_offsets"][-1])
    nnz = sum(int(len(batch[s][0])) for s in range(1, num_slots + 1))
    return n, nnz


def make_table_numpy(num_rows: int, emb_dim: int = EMB_DIM, seed: int = 0, std: float = 0.02,
                     dtype: str = "float32") -> np.ndarray:
    """Host table ~N(0, std) with a zero padding row.  bfloat16 is returned as uint16 bits."""
    rng = np.random.default_rng(seed + 12345)
    t = (rng.standard_normal((num_rows, emb_dim), dtype=np.float32) * np.float32(std))
    t[0] = 0.0
    if dtype == "float32":
        return t
    if dtype == "bfloat16":
        u = t.view(np.uint32).astype(np.uint64)
        u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
        return u.astype(np.uint16)
    raise ValueError(dtype)


def make_table_torch(num_rows: int, emb_dim: int = EMB_DIM, seed: int = 0, std: float = 0.02,
                     dtype=None, device="cuda", chunk_rows: int = 1 << 20):
    """Device table ~N(0, std) generated in chunks on ``device`` (row 0 = padding, zeros)."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 12345)
    t = torch.empty((num_rows, emb_dim), dtype=dtype, device=device)
    for r0 in range(0, num_rows, chunk_rows):
        r1 = min(num_rows, r0 + chunk_rows)
        t[r0:r1].normal_(0.0, std, generator=gen)
    t[0].zero_()
    return t
