"""Multi-rank logic on CPU: user partitioning and the slot-sharded pooled-row
exchange, run as world-size-2 gloo process groups with the oracle standing in
for the GPU kernels; plus failure detection on the host (a rank that dies
before a collective makes the others fail fast instead of hanging)."""

import os
import socket
import time

import numpy as np
import pytest

from baidu_cti_grab_b200 import sharding, synth
from oracle import oracle as O

S = 28
D = 512


def _batch(seed=5, users=12, rows=60):
    cfg = synth.WorkloadConfig("gloo", rows, "float32", users, 1, 9, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=seed)
    table = synth.make_table_numpy(cfg.num_rows, seed=seed, dtype="float32")
    rng = np.random.default_rng(seed)
    gamma = (1 + 0.1 * rng.standard_normal(S * D)).astype(np.float32)
    beta = (0.05 * rng.standard_normal(S * D)).astype(np.float32)
    return cfg, b, table, gamma, beta


def test_partition_users_is_balanced_and_contiguous():
    rng = np.random.default_rng(0)
    seq = rng.integers(1, 200, size=1024)
    uo = np.concatenate([[0], np.cumsum(seq)])
    for world in (1, 2, 3, 8):
        parts = sharding.partition_users(uo, world)
        assert parts[0][0] == 0 and parts[-1][1] == uo[-1]
        for (a, b), (c, d) in zip(parts, parts[1:]):
            assert b == c
        sizes = [b - a for a, b in parts]
        assert max(sizes) - min(sizes) <= 2 * 200
        assert all(a in uo and b in uo for a, b in parts)


def test_slice_items_matches_full_oracle():
    cfg, b, table, gamma, beta = _batch()
    q, s = O.rep_forward(table, "float32", b, gamma, beta)
    uo = b["user_offsets"]
    for i0, i1 in sharding.partition_users(uo, 3, sharding.item_weights_by_ids(b)):
        sub = sharding.slice_items(b, i0, i1)
        qs, ss = O.rep_forward(table, "float32", sub, gamma, beta)
        assert np.array_equal(qs, q[i0:i1]) and np.array_equal(ss, s[i0:i1])


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _run(fn, world, port, *args, deadline_s=90):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + deadline_s
    for _ in procs:
        r, payload = q.get(timeout=max(1, deadline - time.time()))
        res[r] = payload
    for p in procs:
        p.join(timeout=30)
    return res


def _init(rank, world, port, timeout_s=60):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _user_partition_rank(rank, world, port, q):
    try:
        import torch

        dist = _init(rank, world, port)
        cfg, b, table, gamma, beta = _batch()
        i0, i1 = sharding.partition_users(b["user_offsets"], world, sharding.item_weights_by_ids(b))[rank]
        qs, _ = O.rep_forward(table, "float32", sharding.slice_items(b, i0, i1), gamma, beta)
        # gather every rank's rows for the check (verification only; no collective on the data path)
        sizes = [None] * world
        dist.all_gather_object(sizes, (i0, i1, qs.tobytes()))
        dist.destroy_process_group()
        q.put((rank, sizes))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, repr(exc)))


def test_user_partitioned_gloo_world2():
    res = _run(_user_partition_rank, 2, _free_port())
    cfg, b, table, gamma, beta = _batch()
    qf, _ = O.rep_forward(table, "float32", b, gamma, beta)
    got = res[0]
    assert not isinstance(got, str), got
    rows = [np.frombuffer(buf, dtype=np.int8).reshape(i1 - i0, S * D) for i0, i1, buf in got]
    assert np.array_equal(np.concatenate(rows), qf)


def _slot_shard_rank(rank, world, port, q):
    try:
        import torch

        dist = _init(rank, world, port)
        cfg, b, table, gamma, beta = _batch(seed=7)
        plan = sharding.make_slot_plan(rank, world, b["user_offsets"])
        n = len(b[1][1]) - 1
        # this rank pools its slots for every item (the GPU kernel's job; the oracle stands in)
        pooled = torch.zeros((n, plan.s_max * D), dtype=torch.float32)
        for k, s in enumerate(plan.slots):
            v, o = b[s]
            pooled[:, k * D:(k + 1) * D] = torch.from_numpy(
                O.embedding_bag_sum(table, "float32", v, o))

        def a2a(out, inp, out_splits, in_splits):
            dist.all_to_all_single(out, inp, out_splits, in_splits)

        views = sharding.slot_sharded_rows(plan, pooled, a2a, lambda shape: torch.empty(shape))
        row = torch.cat([v for v in views], dim=1).numpy()
        qs, ss = O.quant_dynamic_v2(O.layernorm_rows(row, gamma, beta, 1e-5, "float32")[0])
        i0, i1 = plan.my_items
        dist.destroy_process_group()
        q.put((rank, (i0, i1, qs.tobytes(), ss.tobytes())))
    except Exception as exc:
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("world", [2, 3])
def test_slot_sharded_exchange_gloo(world):
    res = _run(_slot_shard_rank, world, _free_port())
    cfg, b, table, gamma, beta = _batch(seed=7)
    qf, sf = O.rep_forward(table, "float32", b, gamma, beta)
    for r in range(world):
        got = res[r]
        assert not isinstance(got, str), got
        i0, i1, qb, sb = got
        assert np.array_equal(np.frombuffer(qb, dtype=np.int8).reshape(i1 - i0, S * D), qf[i0:i1])
        assert np.array_equal(np.frombuffer(sb, dtype=np.float32), sf[i0:i1])


def _dying_rank(rank, world, port, q):
    try:
        import torch

        dist = _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "exited"))
            q.close()
            q.join_thread()  # make sure the message leaves before the hard exit
            os._exit(0)  # leaves between steps, before the collective
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
            q.put((rank, "collective returned"))
        except Exception as exc:
            q.put((rank, ("failed", time.time() - t0, type(exc).__name__)))
    except Exception as exc:
        q.put((rank, ("init failed", repr(exc))))


def test_dead_rank_is_detected_not_hung():
    res = _run(_dying_rank, 2, _free_port())
    assert res[1] == "exited"
    status = res[0]
    assert isinstance(status, tuple) and status[0] == "failed", status
    assert status[1] < 60


def test_peer_exchange_destinations():
    """PeerExchange.dest_args: rank r's rows for rank d start at block r of d's
    receive buffer; item boundaries are the plan's item ranges (CPU only, no IPC)."""
    import torch
    from baidu_cti_grab_b200 import sharding

    uo = np.array([0, 5, 9, 20, 26, 40], dtype=np.int64)
    world = 3
    plans = [sharding.make_slot_plan(r, world, uo) for r in range(world)]
    exs = [sharding.PeerExchange(p, torch.bfloat16, torch.device("cpu"), peer_ptrs=[[0] * world] * 2) for p in plans]
    bases = [[1 << 40 | (d << 32) | (k << 28) for d in range(world)] for k in range(2)]
    for ex in exs:
        ex.ptrs = bases
    width = plans[0].s_max * 512
    assert exs[0].width == width
    for r, ex in enumerate(exs):
        assert ex.bufs[0].shape == (world, max(1, plans[r].my_items[1] - plans[r].my_items[0]), width)
        for k in range(2):
            dest, begin, ld = ex.dest_args(k)
            assert ld == width
            assert begin == [a for a, _ in plans[r].item_ranges] + [40]
            for d in range(world):
                n_d = plans[d].my_items[1] - plans[d].my_items[0]
                assert dest[d] == bases[k][d] + r * max(1, n_d) * width * 2
        assert [ex.next_buffer() for _ in range(3)] == [0, 1, 0]
