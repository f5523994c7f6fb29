"""Host-resident batches through the RepEncoder with copies overlapped.

A serving loop hands the model one batch dict after another from host
memory.  ``pack_batch`` packs a batch's 28 (values, offsets) pairs into one
pinned buffer, cut into item chunks: each chunk holds its own items' values
and offsets (rebased to the chunk), so one contiguous copy brings a chunk to
the device.  The buffer is int32 when every id and offset fits (half the bytes
of the reference's int64 collate output; the kernel widens them, so results
are identical), else int64.  ``HostPipeline`` then runs, on three CUDA streams,

    copy-in (H2D of chunk c+1) | compute (K1 + K2 of chunk c) | copy-out (D2H of chunk c-1)

so that PCIe traffic in both directions hides behind the kernels and only the
first chunk's copy-in and the last chunk's copy-out are exposed.  Each batch
has its own device input and output buffer (double buffered), guarded by CUDA
events; results land in caller-visible pinned host tensors.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .rep_encoder import rep_encoder_forward

# items per chunk: a 104k-item batch goes in two chunks.  Each chunk's GEMM
# still fills the GPU with 256-row tiles, and only half a batch's copy-in and
# copy-out is exposed at the ends of a run (measured on one B200 over 10
# batches: 38.6M items/s unchunked, 40.8M in two chunks, 40.6M in four, 34.7M
# in eight, where the small GEMMs lose more than the copies gain).
DEFAULT_CHUNK_ITEMS = 65536


@dataclass
class PackedChunk:
    """Items [item_begin, item_begin + num_items) of a packed batch."""

    start: int          # first element of the chunk in the packed buffer
    lengths: List[int]  # values of slots 1..S, then offsets of slots 1..S (rebased to the chunk)
    item_begin: int
    num_items: int

    @property
    def size(self) -> int:
        return sum(self.lengths)


@dataclass
class PackedBatch:
    """One batch in a single pinned int32/int64 buffer, chunk after chunk; a chunk
    holds the values of slots 1..S, then their offsets rebased to the chunk."""

    host: torch.Tensor  # pinned int32 or int64
    chunks: List[PackedChunk]
    num_slots: int
    num_items: int

    @property
    def nbytes(self) -> int:
        return self.host.numel() * self.host.element_size()

    @property
    def num_ids(self) -> int:
        return sum(sum(c.lengths[: self.num_slots]) for c in self.chunks)


def _as_np(a) -> np.ndarray:
    return (a.numpy() if torch.is_tensor(a) else np.asarray(a)).astype(np.int64, copy=False)


def pack_batch(batch: Dict[object, object], num_slots: int = 28, pin: bool = True,
               chunk_items: Optional[int] = DEFAULT_CHUNK_ITEMS, index_dtype: str = "auto") -> PackedBatch:
    """Pack a reference batch dict (numpy arrays or CPU tensors) into one pinned buffer.

    ``index_dtype``: "int64", "int32" (ValueError if an id or offset does not
    fit) or "auto" (int32 when everything fits, else int64).

    With ``chunk_items`` (None: one chunk) the items are cut into about equal
    chunks of at most that many.  Every chunk computes exactly what the whole
    batch would: item i's bag is values[offsets[i]:offsets[i+1]] and the last
    item's bag runs to the end of ``values``, as in the reference.  Cutting
    needs offsets that never decrease and stay within ``values``; other
    batches must be packed as one chunk."""
    vals = [_as_np(batch[s][0]) for s in range(1, num_slots + 1)]
    offs = [_as_np(batch[s][1]) for s in range(1, num_slots + 1)]
    n = len(offs[0]) - 1
    if any(len(o) != n + 1 for o in offs):
        raise ValueError("every slot needs offsets of length N+1")
    nchunks = 1 if not chunk_items or n <= chunk_items else -(-n // int(chunk_items))
    if nchunks > 1:
        for v, o in zip(vals, offs):
            if o[0] < 0 or o[-1] > len(v) or np.any(np.diff(o) < 0):
                raise ValueError("cutting a batch into chunks needs nondecreasing offsets within the "
                                 "values; pack it with chunk_items=None")
    bounds = [(k * n) // nchunks for k in range(nchunks + 1)]
    parts: List[np.ndarray] = []
    chunks: List[PackedChunk] = []
    pos = 0
    for c in range(nchunks):
        i0, i1 = bounds[c], bounds[c + 1]
        last = c == nchunks - 1
        lengths = []
        cv, co = [], []
        for v, o in zip(vals, offs):
            a = int(o[i0]) if nchunks > 1 else 0
            b = len(v) if last else int(o[i1])
            cv.append(v[a:b])
            co.append(o[i0:i1 + 1] - a if a else o[i0:i1 + 1])
        for p in cv + co:
            lengths.append(len(p))
            parts.append(p)
        chunks.append(PackedChunk(pos, lengths, i0, i1 - i0))
        pos += sum(lengths)
    flat = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
    if index_dtype not in ("auto", "int32", "int64"):
        raise ValueError("index_dtype must be 'auto', 'int32' or 'int64'")
    if index_dtype != "int64":
        fits = flat.size == 0 or (int(flat.min()) >= -(1 << 31) and int(flat.max()) < (1 << 31))
        if fits:
            flat = flat.astype(np.int32)
        elif index_dtype == "int32":
            raise ValueError("an id or offset does not fit in int32; pack with index_dtype='int64'")
    host = torch.from_numpy(flat)
    if pin:
        host = host.pin_memory()
    return PackedBatch(host, chunks, num_slots, n)


def unpack_device(flat: torch.Tensor, chunk: PackedChunk, num_slots: int) -> Dict[int, tuple]:
    """Batch dict of device views into a copied chunk."""
    views = torch.split(flat[chunk.start: chunk.start + chunk.size], chunk.lengths)
    S = num_slots
    return {s: (views[s - 1], views[S + s - 1]) for s in range(1, S + 1)}


class HostPipeline:
    """Runs packed host batches through ``rep`` with H2D / compute / D2H overlapped.

    ``max_ids`` and ``max_items`` bound the batches (ids summed over slots,
    items); ``max_chunks`` bounds the chunks per batch.  The last chunk of a
    run is computed in ``tail_parts`` item ranges, each copied out as soon as
    it is done, so that less of the final copy-out waits behind the kernels."""

    def __init__(self, rep: torch.nn.Module, max_ids: int, max_items: int, depth: int = 2,
                 max_chunks: int = 16, tail_parts: int = 4):
        dev = rep.emb.weight.device
        self.rep = rep
        self.tail_parts = tail_parts
        self._tail_events: List[torch.cuda.Event] = []
        self.device = dev
        self.depth = depth
        self.s_in = torch.cuda.Stream(dev)
        self.s_comp = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)
        S = rep.slot_num
        # raw bytes, viewed as each batch's index type (int32 or int64)
        self.in_bufs = [torch.empty(8 * (max_ids + S * (max_items + max_chunks)), dtype=torch.uint8, device=dev)
                        for _ in range(depth)]
        d_model = rep.linear.weight.shape[0] if hasattr(rep.linear, "weight") else rep.linear.qweight_t.shape[1]
        self.out_bufs = [torch.empty((max_items, d_model), dtype=rep.emb.weight.dtype, device=dev)
                         for _ in range(depth)]
        self.in_free = [torch.cuda.Event() for _ in range(depth)]   # compute finished reading in_bufs[k]
        self.out_free = [torch.cuda.Event() for _ in range(depth)]  # D2H finished reading out_bufs[k]
        self._chunk_events: Dict[tuple, tuple] = {}
        for k in range(depth):
            self.in_free[k].record(self.s_comp)
            self.out_free[k].record(self.s_out)

    def _events(self, k: int, c: int):
        ev = self._chunk_events.get((k, c))
        if ev is None:
            ev = (torch.cuda.Event(), torch.cuda.Event())  # copied, computed
            self._chunk_events[(k, c)] = ev
        return ev

    @staticmethod
    def _tail_bounds(pb: PackedBatch, ch: PackedChunk, parts: int):
        """Item ranges of the chunk and each slot's host offsets, or None when the
        chunk cannot be split: too few items, or offsets that decrease or leave
        their values (those are passed through whole, as given)."""
        n = ch.num_items
        parts = min(parts, n)
        if parts <= 1:
            return None
        S = pb.num_slots
        flat = pb.host[ch.start: ch.start + ch.size].numpy()
        pos = np.cumsum([0] + ch.lengths)
        offs = [flat[pos[S + s]: pos[S + s + 1]] for s in range(S)]
        for s, o in enumerate(offs):
            if len(o) != n + 1 or o[0] < 0 or o[-1] > ch.lengths[s] or np.any(np.diff(o) < 0):
                return None
        return [(j * n) // parts for j in range(parts + 1)], offs

    def run(self, batches: Sequence[PackedBatch], host_out: Sequence[torch.Tensor]) -> None:
        """Process ``batches``; result i goes to ``host_out[i]`` (pinned, [items_i, d_model]).
        Returns after the work is enqueued; synchronise the device (or ``self.s_out``) to wait."""
        for i, pb in enumerate(batches):
            k = i % self.depth
            inb, outb = self.in_bufs[k].view(pb.host.dtype), self.out_bufs[k]
            if pb.host.numel() > inb.numel() or pb.num_items > outb.shape[0]:
                raise ValueError("batch larger than the pipeline's max_ids / max_items / max_chunks")
            self.s_in.wait_event(self.in_free[k])
            self.s_comp.wait_event(self.out_free[k])
            for c, ch in enumerate(pb.chunks):
                copied, computed = self._events(k, c)
                i0, i1 = ch.item_begin, ch.item_begin + ch.num_items
                with torch.cuda.stream(self.s_in):
                    inb[ch.start: ch.start + ch.size].copy_(pb.host[ch.start: ch.start + ch.size],
                                                           non_blocking=True)
                    copied.record(self.s_in)
                self.s_comp.wait_event(copied)
                views = unpack_device(inb, ch, pb.num_slots)
                last = i == len(batches) - 1 and c == len(pb.chunks) - 1
                tail = self._tail_bounds(pb, ch, self.tail_parts) if last else None
                if tail is None:
                    with torch.cuda.stream(self.s_comp):
                        rep_encoder_forward(self.rep, views, out=outb[i0:i1])
                        computed.record(self.s_comp)
                    self.s_out.wait_event(computed)
                    with torch.cuda.stream(self.s_out):
                        host_out[i][i0:i1].copy_(outb[i0:i1], non_blocking=True)
                    continue
                # items [a, b) of the chunk: offsets stay absolute within the chunk's
                # values; the values end where item b starts (or at the chunk's end)
                bounds, offs = tail
                while len(self._tail_events) < len(bounds) - 1:
                    self._tail_events.append(torch.cuda.Event())
                for j in range(len(bounds) - 1):
                    a, b = bounds[j], bounds[j + 1]
                    part = {}
                    for s in range(1, pb.num_slots + 1):
                        v, o = views[s]
                        part[s] = (v if b == ch.num_items else v[: int(offs[s - 1][b])], o[a: b + 1])
                    ev = self._tail_events[j]
                    with torch.cuda.stream(self.s_comp):
                        rep_encoder_forward(self.rep, part, out=outb[i0 + a: i0 + b])
                        ev.record(self.s_comp)
                    self.s_out.wait_event(ev)
                    with torch.cuda.stream(self.s_out):
                        host_out[i][i0 + a: i0 + b].copy_(outb[i0 + a: i0 + b], non_blocking=True)
            self.in_free[k].record(self.s_comp)
            self.out_free[k].record(self.s_out)

    def synchronize(self) -> None:
        self.s_out.synchronize()
