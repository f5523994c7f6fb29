"""pack_batch cuts a batch into item chunks without changing any item's bag (CPU only)."""

import numpy as np
import pytest
import torch

from baidu_cti_grab_b200 import synth
from baidu_cti_grab_b200.pipeline import pack_batch


def _bags(values, offsets):
    """Reference bag semantics: bag i = values[off[i]:off[i+1]], the last bag runs to the end."""
    n = len(offsets) - 1
    return [values[offsets[i]:(offsets[i + 1] if i + 1 < n else len(values))] for i in range(n)]


def _chunk_bags(pb):
    """Per slot, the bags of every item as the packed chunks describe them."""
    flat = pb.host.numpy()
    S = pb.num_slots
    out = {s: [] for s in range(1, S + 1)}
    for ch in pb.chunks:
        parts = np.split(flat[ch.start: ch.start + ch.size], np.cumsum(ch.lengths)[:-1])
        for s in range(1, S + 1):
            bags = _bags(parts[s - 1], parts[S + s - 1])
            assert len(bags) == ch.num_items
            out[s].extend(bags)
    return out


@pytest.mark.parametrize("chunk_items", [None, 1, 7, 64, 10_000])
def test_chunks_keep_every_bag(chunk_items):
    cfg = synth.WorkloadConfig("pack", 500, "bfloat16", 12, 1, 40, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=4)
    # trailing ids after the last offset belong to the last bag (offsets[:-1] semantics)
    v, o = b[3]
    b[3] = (np.concatenate([v, np.array([5, 6, 7], dtype=v.dtype)]), o)
    pb = pack_batch(b, pin=False, chunk_items=chunk_items)
    n = len(b[1][1]) - 1
    assert pb.num_items == n
    assert sum(c.num_items for c in pb.chunks) == n
    if chunk_items:
        assert all(c.num_items <= chunk_items for c in pb.chunks)
    got = _chunk_bags(pb)
    for s in range(1, 29):
        want = _bags(np.asarray(b[s][0], dtype=np.int64), np.asarray(b[s][1], dtype=np.int64))
        assert len(got[s]) == n
        for g, w in zip(got[s], want):
            assert np.array_equal(g, w)


def test_chunking_rejects_decreasing_offsets():
    cfg = synth.WorkloadConfig("pack", 500, "bfloat16", 8, 1, 40, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=5)
    v, o = b[2]
    o = o.copy()
    o[3], o[4] = o[4] + 1, o[3]
    b[2] = (v, o)
    with pytest.raises(ValueError):
        pack_batch(b, pin=False, chunk_items=4)
    pb = pack_batch(b, pin=False, chunk_items=None)  # whole batch: passed through as given
    assert len(pb.chunks) == 1


def test_empty_batch_packs_as_one_empty_chunk():
    b = {"user_offsets": np.zeros(1, dtype=np.int64)}
    for s in range(1, 29):
        b[s] = (np.zeros(0, dtype=np.int64), np.zeros(1, dtype=np.int64))
    pb = pack_batch(b, pin=False, chunk_items=4)
    assert pb.num_items == 0 and pb.num_ids == 0 and len(pb.chunks) == 1
    assert pb.chunks[0].num_items == 0 and pb.host.numel() == 28  # 28 one-entry offset arrays


def test_index_dtype_auto_int32_and_int64_fallback():
    cfg = synth.WorkloadConfig("pack", 500, "bfloat16", 6, 1, 20, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=8)
    p32 = pack_batch(b, pin=False, chunk_items=5)
    p64 = pack_batch(b, pin=False, chunk_items=5, index_dtype="int64")
    assert p32.host.dtype == torch.int32 and p64.host.dtype == torch.int64
    assert p32.nbytes * 2 == p64.nbytes
    assert np.array_equal(p32.host.numpy().astype(np.int64), p64.host.numpy())
    assert [c.lengths for c in p32.chunks] == [c.lengths for c in p64.chunks]
    # an id beyond int32: auto keeps int64, an explicit int32 request is refused
    v, o = b[7]
    b[7] = (np.concatenate([v[:-1], np.array([1 << 33], dtype=np.int64)]), o)
    assert pack_batch(b, pin=False, chunk_items=5).host.dtype == torch.int64
    with pytest.raises(ValueError):
        pack_batch(b, pin=False, index_dtype="int32")


@pytest.mark.parametrize("chunk_items,parts", [(None, 4), (37, 4), (37, 3), (5, 8)])
def test_tail_ranges_keep_every_bag(chunk_items, parts):
    """The last chunk of a pipeline run is computed in item ranges: offsets
    o[a:b+1] (absolute within the chunk) over values cut at o[b] give every
    item the bag it has in the whole chunk."""
    from baidu_cti_grab_b200.pipeline import HostPipeline

    cfg = synth.WorkloadConfig("pack", 500, "bfloat16", 9, 1, 30, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=12)
    pb = pack_batch(b, pin=False, chunk_items=chunk_items)
    ch = pb.chunks[-1]
    tail = HostPipeline._tail_bounds(pb, ch, parts)
    assert tail is not None
    bounds, offs = tail
    assert bounds[0] == 0 and bounds[-1] == ch.num_items and len(bounds) == min(parts, ch.num_items) + 1
    flat = pb.host.numpy()[ch.start: ch.start + ch.size]
    S = pb.num_slots
    vals = np.split(flat, np.cumsum(ch.lengths)[:-1])[:S]
    for s in range(S):
        whole = _bags(vals[s], offs[s])
        got = []
        for a, bb in zip(bounds[:-1], bounds[1:]):
            v = vals[s] if bb == ch.num_items else vals[s][: int(offs[s][bb])]
            o = offs[s][a: bb + 1]
            got.extend(v[int(o[i]): (int(o[i + 1]) if i + 1 < len(o) - 1 else len(v))] for i in range(len(o) - 1))
        assert len(got) == len(whole)
        for g, w in zip(got, whole):
            assert np.array_equal(g, w)


def test_tail_ranges_refuse_unsplittable_chunks():
    from baidu_cti_grab_b200.pipeline import HostPipeline

    cfg = synth.WorkloadConfig("pack", 500, "bfloat16", 3, 1, 3, "1+poisson1", 1.1)
    b = synth.make_batch(cfg, seed=13)
    pb = pack_batch(b, pin=False, chunk_items=None)
    assert HostPipeline._tail_bounds(pb, pb.chunks[0], 1) is None  # one range: nothing to split
    v, o = b[4]
    o = o.copy()
    if len(o) > 2:
        o[1], o[2] = o[2] + 1, o[1]
        b[4] = (v, o)
        pb = pack_batch(b, pin=False, chunk_items=None)  # passed through as given
        assert HostPipeline._tail_bounds(pb, pb.chunks[0], 2) is None
