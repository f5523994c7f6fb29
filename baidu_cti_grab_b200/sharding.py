"""Multi-GPU partitioning of the RepEncoder path.

Two layouts (one process per GPU, ``torch.distributed`` for the plumbing):

* **User-partitioned** (tables fit in one GPU): a batch's users are split
  into contiguous ranges with about equal id counts; each rank runs K1 + K2 on
  its own items with a replicated table and weight.  Items are independent
  rows, so there is no collective on the data path.  ``partition_users`` and
  ``slice_items`` compute the split and the rebased per-rank batch.

* **Slot-sharded** (tables larger than one GPU's memory): rank r owns the
  slots s with (s-1) % world == r and only their table rows.  Every rank pools
  its slots for all items of the global batch (``rb_rep_gather_pool``), one
  ``all_to_all_single`` delivers to each rank the pooled rows of its own item
  range from every other rank, and the LayerNorm + int8 quantiser read the 28
  slot blocks in place through per-slot row pointers (``rb_layernorm_quant_slots``)
  before the local GEMM.  The exchange is in the row dtype (bf16), exactly
  what the reference's EmbeddingBag produces, so it loses nothing.

  With ``PeerExchange`` the pooling kernel does the exchange itself
  (``rb_rep_gather_pool_scatter``): every rank maps the other ranks' receive
  buffers (CUDA IPC) and stores each item's pooled rows straight into its
  owner's buffer over NVLink while it pools, so the transfer overlaps the
  gather; one small all-reduce per step then hands the rows over.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

NUM_SLOTS = 28
EMB_DIM = 512


# ----------------------------------------------------------- user partition
def partition_users(user_offsets: np.ndarray, world: int, item_weight: Optional[np.ndarray] = None
                    ) -> List[Tuple[int, int]]:
    """Contiguous user ranges per rank, balanced by total weight (default: items).

    Returns [(item_begin, item_end)] per rank; boundaries fall on user boundaries."""
    user_offsets = np.asarray(user_offsets, dtype=np.int64)
    n_users = len(user_offsets) - 1
    if item_weight is None:
        cum_items = user_offsets.astype(np.float64)
    else:
        w = np.concatenate([[0.0], np.cumsum(np.asarray(item_weight, dtype=np.float64))])
        cum_items = w[user_offsets]
    total = cum_items[-1]
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        u = int(np.searchsorted(cum_items, target, side="left"))
        u = min(max(u, bounds[-1]), n_users)
        bounds.append(u)
    bounds.append(n_users)
    return [(int(user_offsets[bounds[r]]), int(user_offsets[bounds[r + 1]])) for r in range(world)]


def item_weights_by_ids(batch: Dict[object, object], num_slots: int = NUM_SLOTS) -> np.ndarray:
    """Ids per item summed over slots (the gather's cost per item)."""
    n = len(batch[1][1]) - 1
    w = np.zeros(n, dtype=np.int64)
    for s in range(1, num_slots + 1):
        w += np.diff(np.asarray(batch[s][1], dtype=np.int64))
    return w


def slice_items(batch: Dict[object, object], i0: int, i1: int, num_slots: int = NUM_SLOTS
                ) -> Dict[object, object]:
    """Items [i0, i1) of a numpy batch dict, offsets rebased to the slice."""
    out: Dict[object, object] = {}
    uo = np.asarray(batch["user_offsets"], dtype=np.int64)
    u0 = int(np.searchsorted(uo, i0, side="left"))
    u1 = int(np.searchsorted(uo, i1, side="left"))
    out["user_offsets"] = uo[u0:u1 + 1] - i0
    for s in range(1, num_slots + 1):
        v, o = batch[s]
        o = np.asarray(o, dtype=np.int64)
        a, b = int(o[i0]), int(o[i1])
        out[s] = (np.asarray(v)[a:b], o[i0:i1 + 1] - a)
    return out


# ------------------------------------------------------------- slot shards
def slot_owner(slot: int, world: int) -> int:
    """Rank that owns 1-based slot ``slot``."""
    return (slot - 1) % world


def local_slots(rank: int, world: int, num_slots: int = NUM_SLOTS) -> List[int]:
    return [s for s in range(1, num_slots + 1) if slot_owner(s, world) == rank]


def max_local_slots(world: int, num_slots: int = NUM_SLOTS) -> int:
    return (num_slots + world - 1) // world


def received_slot_views(recv, world: int, items: int, num_slots: int = NUM_SLOTS):
    """Per-slot [items, 512] views of the all-to-all receive buffer.

    recv is [world, items, S_max*512]: block j holds rank j's local slots (in
    local order) for this rank's items; global slot s (1-based) owned by rank
    j = (s-1) % world sits in local column block k = (s-1) // world."""
    views = []
    for s in range(1, num_slots + 1):
        j = slot_owner(s, world)
        k = (s - 1) // world
        views.append(recv[j, :, k * EMB_DIM:(k + 1) * EMB_DIM])
    return views


@dataclass
class SlotShardPlan:
    rank: int
    world: int
    slots: List[int]          # global 1-based slots this rank owns
    s_max: int                # padded local slot count (exchange width in slots)
    item_ranges: List[Tuple[int, int]]  # item range of every rank

    @property
    def my_items(self) -> Tuple[int, int]:
        return self.item_ranges[self.rank]


def make_slot_plan(rank: int, world: int, user_offsets: np.ndarray,
                   item_weight: Optional[np.ndarray] = None) -> SlotShardPlan:
    return SlotShardPlan(rank, world, local_slots(rank, world), max_local_slots(world),
                         partition_users(user_offsets, world, item_weight))


def slot_sharded_rows(plan: SlotShardPlan, pooled_local, all_to_all: Callable, new_empty: Callable):
    """Exchange pooled rows and return the per-slot views of this rank's items.

    pooled_local: [N_total, S_max*512] rows of this rank's slots for all items
    (columns beyond the owned slots are padding).  all_to_all(out, inp,
    out_splits, in_splits) is a ``torch.distributed.all_to_all_single``-shaped
    callable; new_empty(shape) allocates the receive buffer."""
    i0, i1 = plan.my_items
    mine = i1 - i0
    width = plan.s_max * EMB_DIM
    recv = new_empty((plan.world, mine, width))
    in_splits = [b - a for a, b in plan.item_ranges]
    out_splits = [mine] * plan.world
    all_to_all(recv.view(plan.world * mine, width), pooled_local, out_splits, in_splits)
    return received_slot_views(recv, plan.world, mine)


# ----------------------------------------------------- slot-sharded module
class SlotShardedRepEncoder:
    """RepEncoder forward with the embedding table sharded by slot across ranks.

    ``local_table`` holds, after the padding row 0, the rows of this rank's
    slots one slot after another: global slot s = plan.slots[k] owns local
    rows 1 + k*R .. (k+1)*R, where R = rows_per_slot (the synthetic and
    reference layouts give slot s the global rows 1 + (s-1)*R .. s*R).  Ids
    are moved into the local block by subtracting ((s-1) - k)*R; an id outside
    its slot's block is clamped like any out-of-range id.

    ``forward(values, offsets)`` takes the global batch's per-slot id arrays
    (only the owned slots are read) and returns the [N_mine, d_model] output of
    this rank's item range ``plan.my_items``.
    """

    def __init__(self, plan: SlotShardPlan, local_table, rows_per_slot: int, gamma, beta, eps: float, w_nk,
                 w_scale, bias, all_to_all: Optional[Callable] = None):
        import torch

        self.plan = plan
        self.table = local_table
        self.R = rows_per_slot
        self.gamma, self.beta, self.eps = gamma, beta, eps
        self.w_nk, self.w_scale, self.bias = w_nk, w_scale, bias
        if all_to_all is None:
            import torch.distributed as dist

            def all_to_all(out, inp, out_splits, in_splits):
                dist.all_to_all_single(out, inp, out_splits, in_splits)
        self.all_to_all = all_to_all
        self._torch = torch

    def pool_local(self, values: Sequence, offsets: Sequence):
        """[N_total, S_max*512] pooled rows of this rank's slots (padding columns unset)."""
        from . import device_ops

        vals, offs = self._local_ids(values, offsets)
        return device_ops.rep_gather_pool(self.table, vals, offs, list(range(len(self.plan.slots))),
                                          self.plan.s_max)

    def forward(self, values: Sequence, offsets: Sequence):
        return self.finish(self.pool_local(values, offsets))

    def _local_ids(self, values: Sequence, offsets: Sequence):
        vals, offs = [], []
        for k, s in enumerate(self.plan.slots):
            shift = ((s - 1) - k) * self.R
            v = values[s - 1]
            vals.append(v - shift if shift else v)
            offs.append(offsets[s - 1])
        return vals, offs

    def pool_scatter(self, values: Sequence, offsets: Sequence, exchange: "PeerExchange", k: int) -> None:
        """Pool this rank's slots for all items straight into the owners' receive buffers k."""
        from . import device_ops

        vals, offs = self._local_ids(values, offsets)
        dest, begin, ld = exchange.dest_args(k)
        # start at the next rank's items: at any moment the ranks store into different owners
        n = begin[-1]
        shift = begin[(self.plan.rank + 1) % self.plan.world] % n if n else 0
        device_ops.rep_gather_pool_scatter(self.table, vals, offs, list(range(len(self.plan.slots))), dest, begin, ld,
                                           item_shift=shift)

    def finish_received(self, recv):
        """LayerNorm + int8 of this rank's items from its receive buffer [world, items, S_max*512], GEMM."""
        from . import device_ops

        torch = self._torch
        if recv.shape[1] == 0:
            return torch.empty((0, self.w_nk.shape[0]), dtype=recv.dtype, device=recv.device)
        views = received_slot_views(recv, self.plan.world, recv.shape[1])
        q, scale, _ = device_ops.layernorm_quant_slots(views, self.gamma, self.beta, self.eps)
        out = torch.empty((q.shape[0], self.w_nk.shape[0]), dtype=recv.dtype, device=recv.device)
        return device_ops.w8a8_gemm(q, self.w_nk, scale, self.w_scale, out, bias=self.bias)

    def forward_peer(self, values: Sequence, offsets: Sequence, exchange: "PeerExchange", barrier: Callable):
        """One step with the exchange done by the pooling kernel: pool into the
        owners' buffers, ``barrier()`` (a collective on the current stream, e.g. an
        NCCL all-reduce of one element), then LayerNorm + int8 + GEMM of this
        rank's items.  Alternates between the two receive buffers."""
        k = exchange.next_buffer()
        self.pool_scatter(values, offsets, exchange, k)
        barrier()
        return self.finish_received(exchange.received(k))

    def finish(self, pooled):
        """Exchange, LayerNorm + int8 of this rank's items, GEMM."""
        from . import device_ops

        torch = self._torch
        views = slot_sharded_rows(self.plan, pooled, self.all_to_all,
                                  lambda shape: torch.empty(shape, dtype=pooled.dtype, device=pooled.device))
        q, scale, _ = device_ops.layernorm_quant_slots(views, self.gamma, self.beta, self.eps)
        out = torch.empty((q.shape[0], self.w_nk.shape[0]), dtype=pooled.dtype, device=pooled.device)
        return device_ops.w8a8_gemm(q, self.w_nk, scale, self.w_scale, out, bias=self.bias)


class PeerExchange:
    """This rank's receive buffers, and every other rank's mapped into this process.

    bufs[k] is [world, N_mine, S_max*512] in the row dtype: block j receives the
    pooled rows of rank j's slots for this rank's items.  ``ptrs[k][d]`` is the
    address of rank d's buffer k here (its own tensor for d == rank, a CUDA IPC
    mapping otherwise).  Two buffers alternate: a rank stores step t+1's rows
    into buffer (t+1) % 2 while the owner may still read buffer t % 2; the
    owner's reads of buffer (t+1) % 2 from step t-1 precede its barrier of step
    t, which every rank passes before storing step t+1.

    ``all_gather_object(obj) -> list`` collects one picklable object per rank
    (``torch.distributed.all_gather_object``); ``remote`` = None maps nothing
    and takes ``peer_ptrs`` (for one process emulating several ranks)."""

    def __init__(self, plan: SlotShardPlan, dtype, device, all_gather_object: Optional[Callable] = None,
                 nbuf: int = 2, peer_ptrs: Optional[List[List[int]]] = None):
        import torch

        from . import device_ops

        self.plan = plan
        self.device = device
        self.width = plan.s_max * EMB_DIM
        self.esz = torch.empty((), dtype=dtype).element_size()
        self.sizes = [b - a for a, b in plan.item_ranges]
        mine = self.sizes[plan.rank]
        self.bufs = [torch.zeros((plan.world, max(mine, 1), self.width), dtype=dtype, device=device)
                     for _ in range(nbuf)]
        self._opened: List[tuple] = []
        self._step = -1
        if peer_ptrs is not None:
            self.ptrs = [list(p) for p in peer_ptrs]
            return
        if all_gather_object is None:
            raise ValueError("PeerExchange needs all_gather_object (or peer_ptrs)")
        exported = [device_ops.ipc_export(b) for b in self.bufs]
        everyone = all_gather_object(exported)
        self.ptrs = [[0] * plan.world for _ in range(nbuf)]
        for k in range(nbuf):
            for d in range(plan.world):
                if d == plan.rank:
                    self.ptrs[k][d] = self.bufs[k].data_ptr()
                else:
                    handle, off = everyone[d][k]
                    ptr = device_ops.ipc_import(handle, off, device)
                    self._opened.append((ptr, off))
                    self.ptrs[k][d] = ptr

    def received(self, k: int):
        """This rank's rows in buffer k: [world, N_mine, S_max*512]."""
        return self.bufs[k][:, : self.sizes[self.plan.rank]]

    def next_buffer(self) -> int:
        self._step += 1
        return self._step % len(self.bufs)

    def dest_args(self, k: int):
        """(dest, dest_begin, ld) for rb_rep_gather_pool_scatter from this rank into buffers k."""
        r = self.plan.rank
        dest = [self.ptrs[k][d] + r * max(self.sizes[d], 1) * self.width * self.esz for d in range(self.plan.world)]
        begin = [a for a, _ in self.plan.item_ranges] + [self.plan.item_ranges[-1][1]]
        return dest, begin, self.width

    def close(self) -> None:
        """Unmap the other ranks' buffers.  Call it on every rank after a barrier
        that follows the last step (no rank may still be storing into a buffer
        that its owner frees), and before the ranks exit."""
        from . import device_ops

        for ptr, off in self._opened:
            device_ops.ipc_close(ptr, off, self.device)
        self._opened = []


def build_local_table(full_table, plan: SlotShardPlan, rows_per_slot: int):
    """This rank's shard of a full [S*R+1, D] table (for tests and small runs)."""
    import torch

    R = rows_per_slot
    parts = [full_table[0:1]]
    for s in plan.slots:
        parts.append(full_table[1 + (s - 1) * R: 1 + s * R])
    return torch.cat(parts, dim=0).contiguous()
