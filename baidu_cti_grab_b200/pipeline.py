"""Host-resident batches through the RepEncoder with copies overlapped.

A serving loop hands the model one batch dict after another from host
memory.  ``HostPipeline`` packs each batch's 28 (values, offsets) pairs into
one pinned int64 buffer (the layout ``pack_batch`` produces), and runs, on
three CUDA streams,

    copy-in  (H2D of batch i+1)  |  compute (K1 + K2 of batch i)  |  copy-out (D2H of batch i-1)

so that PCIe traffic in both directions hides behind the kernels.  Each batch
has its own device input buffer and output buffer (double buffered), guarded
by CUDA events; results land in caller-visible pinned host tensors.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .rep_encoder import rep_encoder_forward


@dataclass
class PackedBatch:
    """One batch in a single pinned int64 buffer: 28 value arrays then 28 offset arrays."""

    host: torch.Tensor  # pinned int64
    lengths: List[int]  # per-part lengths (values of slots 1..S, then offsets of slots 1..S)
    num_slots: int
    num_items: int

    @property
    def nbytes(self) -> int:
        return self.host.numel() * 8


def pack_batch(batch: Dict[object, object], num_slots: int = 28, pin: bool = True) -> PackedBatch:
    """Pack a reference batch dict (numpy arrays or CPU tensors) into one pinned buffer."""
    parts = []
    for s in range(1, num_slots + 1):
        v = batch[s][0]
        parts.append(v.numpy() if torch.is_tensor(v) else np.asarray(v))
    for s in range(1, num_slots + 1):
        o = batch[s][1]
        parts.append(o.numpy() if torch.is_tensor(o) else np.asarray(o))
    flat = np.concatenate([p.astype(np.int64, copy=False) for p in parts])
    host = torch.from_numpy(flat)
    if pin:
        host = host.pin_memory()
    return PackedBatch(host, [len(p) for p in parts], num_slots, len(parts[num_slots]) - 1)


def unpack_device(flat: torch.Tensor, pb: PackedBatch) -> Dict[int, tuple]:
    """Batch dict of device views into a copied packed buffer."""
    views = torch.split(flat[: sum(pb.lengths)], pb.lengths)
    S = pb.num_slots
    return {s: (views[s - 1], views[S + s - 1]) for s in range(1, S + 1)}


class HostPipeline:
    """Runs packed host batches through ``rep`` with H2D / compute / D2H overlapped."""

    def __init__(self, rep: torch.nn.Module, max_ids: int, max_items: int, depth: int = 2):
        dev = rep.emb.weight.device
        self.rep = rep
        self.device = dev
        self.depth = depth
        self.s_in = torch.cuda.Stream(dev)
        self.s_comp = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)
        S = rep.slot_num
        self.in_bufs = [torch.empty(max_ids + S * (max_items + 1), dtype=torch.int64, device=dev)
                        for _ in range(depth)]
        d_model = rep.linear.weight.shape[0] if hasattr(rep.linear, "weight") else rep.linear.qweight_t.shape[1]
        self.out_bufs = [torch.empty((max_items, d_model), dtype=rep.emb.weight.dtype, device=dev)
                         for _ in range(depth)]
        self.in_free = [torch.cuda.Event() for _ in range(depth)]   # compute finished reading in_bufs[k]
        self.out_free = [torch.cuda.Event() for _ in range(depth)]  # D2H finished reading out_bufs[k]
        self.copied = [torch.cuda.Event() for _ in range(depth)]
        self.computed = [torch.cuda.Event() for _ in range(depth)]
        for k in range(depth):
            self.in_free[k].record(self.s_comp)
            self.out_free[k].record(self.s_out)

    def run(self, batches: Sequence[PackedBatch], host_out: Sequence[torch.Tensor]) -> None:
        """Process ``batches``; result i goes to ``host_out[i]`` (pinned, [items_i, d_model]).
        Returns after the work is enqueued; synchronise the device (or ``self.s_out``) to wait."""
        for i, pb in enumerate(batches):
            k = i % self.depth
            n = pb.num_items
            # copy-in
            self.s_in.wait_event(self.in_free[k])
            with torch.cuda.stream(self.s_in):
                d = self.in_bufs[k][: pb.host.numel()]
                d.copy_(pb.host, non_blocking=True)
                self.copied[k].record(self.s_in)
            # compute
            self.s_comp.wait_event(self.copied[k])
            self.s_comp.wait_event(self.out_free[k])
            with torch.cuda.stream(self.s_comp):
                batch = unpack_device(self.in_bufs[k], pb)
                rep_encoder_forward(self.rep, batch, out=self.out_bufs[k][:n])
                self.in_free[k].record(self.s_comp)
                self.computed[k].record(self.s_comp)
            # copy-out
            self.s_out.wait_event(self.computed[k])
            with torch.cuda.stream(self.s_out):
                host_out[i][:n].copy_(self.out_bufs[k][:n], non_blocking=True)
                self.out_free[k].record(self.s_out)

    def synchronize(self) -> None:
        self.s_out.synchronize()
