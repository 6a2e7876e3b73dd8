"""The only collectives of multi-GPU self-play: replay-row gathering and counters.

Games shard across ranks with no exchange on the data path (rank r plays game
ids r*lanes + i, then + world*lanes per finished game, with randomness keyed
by game id). What crosses NVLink is what the reference's Trainer consumes in
one place (python/kingdom_ai/gpu_training.py:124-175 returns every game's
samples to the caller): the replay rows each rank wrote since the last
gather, appended in rank order to rank 0's FIFO, and the summed counters.

Both work on any torch.distributed backend (NCCL over NVLink on GPUs, gloo
for the CPU tests) and every rank must call them in the same order.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

# Packed row: features 810, mask 82, policy 82, value 1, to_play 1 (float32).
_FEATURES, _ACTIONS = 810, 82
ROW_FLOATS = _FEATURES + 2 * _ACTIONS + 2


def _unpack(packed: torch.Tensor):
    """features [n,10,9,9], masks, policy, value, to_play of packed rows."""
    n = packed.shape[0]
    return (packed[:, :_FEATURES].reshape(n, 10, 9, 9), packed[:, _FEATURES:_FEATURES + _ACTIONS] != 0,
            packed[:, _FEATURES + _ACTIONS:_FEATURES + 2 * _ACTIONS], packed[:, -2], packed[:, -1].to(torch.int8))


class ReplayGather:
    """Appends every rank's new rows of `ring` to `fifo` on rank 0.

    ``run(written)`` takes this rank's monotone count of rows written to its
    ring - the engine's device counters (``rows`` is entry 2), a 0-d tensor or
    an int - and never reads it on the host: each rank packs its oldest
    ungathered rows, at most `width`, into a fixed-size slab; the row counts
    and the slabs go to rank 0 only (two ``gather`` collectives); rank 0
    appends each rank's rows in rank order with device-side index arithmetic.
    Rows beyond `width` wait for the next call. Rows that the ring overwrote
    before they were gathered (more than `ring.capacity` behind) are skipped.
    `width` must be the same on every rank and at most the FIFO's capacity.
    """

    def __init__(self, ring, fifo=None, group=None, width: int = 8192):
        self.ring, self.fifo, self.group = ring, fifo, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.width = max(1, min(int(width), ring.capacity))
        device = ring.device
        self.sent = torch.zeros((), dtype=torch.int64, device=device)
        self._lanes = torch.arange(self.width, dtype=torch.int64, device=device)
        self._slab = torch.zeros((self.width, ROW_FLOATS), dtype=torch.float32, device=device)
        self._count = torch.zeros(1, dtype=torch.int64, device=device)
        if self.rank == 0:
            if fifo is None:
                raise ValueError("rank 0 needs a FIFO to gather into")
            if self.width > fifo.capacity:
                raise ValueError("width must not exceed the FIFO's capacity")
            self._fifo_rows = torch.zeros((), dtype=torch.int64, device=fifo.device)
            self._parts = [torch.empty_like(self._slab) for _ in range(self.world)]
            self._counts = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(self.world)]

    @property
    def fifo_rows(self) -> int:
        """Rows appended to the FIFO so far (rank 0; reads the device)."""
        return int(self._fifo_rows.item())

    def _pack(self, written: torch.Tensor) -> None:
        cap = self.ring.capacity
        start = torch.maximum(self.sent, written - cap)
        count = (written - start).clamp(0, self.width)
        idx = (start + self._lanes) % cap
        ring = self.ring
        slab = self._slab
        slab[:, :_FEATURES] = ring.features.reshape(cap, -1).index_select(0, idx)
        slab[:, _FEATURES:_FEATURES + _ACTIONS] = ring.masks.index_select(0, idx).to(torch.float32)
        slab[:, _FEATURES + _ACTIONS:_FEATURES + 2 * _ACTIONS] = ring.policy.index_select(0, idx)
        slab[:, -2] = ring.value.index_select(0, idx)
        slab[:, -1] = ring.to_play.index_select(0, idx).to(torch.float32)
        self._count.copy_(count.reshape(1))
        self.sent = start + count

    def run(self, written):
        """Gather; on rank 0 returns the rows appended (a 0-d device tensor), else None."""
        device = self.ring.device
        if isinstance(written, torch.Tensor):
            written = (written[2] if written.numel() == 8 else written.reshape(())).to(device, torch.int64)
        else:
            written = torch.tensor(int(written), dtype=torch.int64, device=device)
        self._pack(written)
        root = self.rank == 0
        dist.gather(self._count, self._counts if root else None, dst=0, group=self.group)
        dist.gather(self._slab, self._parts if root else None, dst=0, group=self.group)
        if not root:
            return None
        fifo = self.fifo
        cap = fifo.capacity
        counts = torch.cat(self._counts).to(fifo.device)
        offsets = torch.cumsum(counts, 0) - counts
        lanes = self._lanes.to(fifo.device)
        fields = (fifo.features, fifo.masks, fifo.policy, fifo.value, fifo.to_play)
        for r in range(self.world):
            # Positions of rank r's slab rows in the FIFO. The rows past its
            # count write back what is there, so the write needs no host-side
            # count; W <= capacity keeps the positions of one slab distinct,
            # and ranks are applied in order, so later rows win a wrap.
            pos = (self._fifo_rows + offsets[r] + lanes) % cap
            valid = lanes < counts[r]
            for field, new in zip(fields, _unpack(self._parts[r].to(fifo.device))):
                keep = valid.view((-1,) + (1,) * (new.dim() - 1))
                field.index_copy_(0, pos, torch.where(keep, new, field.index_select(0, pos)))
        total = counts.sum()
        self._fifo_rows += total
        return total


def total_counters(counters: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of every rank's counters (int64 [8]), returned on every rank."""
    out = counters.clone()
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out
