"""Synthetic workload generator: batch-dict layout and distributions."""

import numpy as np

from baidu_cti_grab_b200 import synth


def test_batch_layout_matches_reference_collate():
    cfg = synth.WorkloadConfig("t", 1000, "bfloat16", 20, 1, 30, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=3)
    uo = b["user_offsets"]
    assert uo.dtype == np.int64 and uo[0] == 0 and np.all(np.diff(uo) >= 1)
    n = int(uo[-1])
    for s in range(1, 29):
        v, o = b[s]
        assert v.dtype == np.int64 and o.dtype == np.int64
        assert len(o) == n + 1 and o[0] == 0 and o[-1] == len(v)
        assert np.all(np.diff(o) >= 1)  # 1 + Poisson(1) >= 1 id per bag
        lo, hi = 1 + (s - 1) * cfg.rows_per_slot, s * cfg.rows_per_slot
        assert v.min() >= lo and v.max() <= hi


def test_zipf_hot_rows_are_scattered():
    rows = 100_000
    rng = np.random.default_rng(0)
    ids = synth.slot_ids(rng, 5, rows, 1.1, 200_000)
    vals, counts = np.unique(ids, return_counts=True)
    hot = vals[np.argsort(-counts)[:10]]
    # the hottest rows are not consecutive row numbers
    assert np.ptp(hot) > 1000
    assert counts.max() > 100 * np.median(counts)


def test_prod_config_sizes():
    cfg = synth.PROD_BF16_1M
    assert cfg.num_rows == 28 * 1_000_000 + 1
    b = synth.make_batch(cfg, seed=1000, num_users=64)
    n, nnz = synth.batch_stats(b)
    assert 64 <= n <= 64 * 200
    assert 1.7 * 28 * n < nnz < 2.3 * 28 * n  # mean bag size 2


def test_uniform_ids_control_stay_in_their_slot():
    cfg = synth.WorkloadConfig("uniform", 1000, "bfloat16", 16, 1, 20, "1+poisson1", 0.0)
    b = synth.make_batch(cfg, seed=9)
    for s in range(1, 29):
        v = b[s][0]
        assert v.min() >= 1 + (s - 1) * 1000 and v.max() <= s * 1000
    # no hot rows: the most frequent row of a slot is rare
    v = b[1][0]
    assert np.bincount(v - 1).max() <= max(8, len(v) // 50)
