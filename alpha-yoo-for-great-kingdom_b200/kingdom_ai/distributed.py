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


def _pack(ring, start: int, count: int, width: int) -> torch.Tensor:
    feats, masks, policy, value, to_play = ring.rows(start, count)
    packed = torch.zeros((width, ROW_FLOATS), dtype=torch.float32, device=ring.device)
    if count:
        packed[:count, :_FEATURES] = feats.reshape(count, -1)
        packed[:count, _FEATURES:_FEATURES + _ACTIONS] = masks.to(torch.float32)
        packed[:count, _FEATURES + _ACTIONS:_FEATURES + 2 * _ACTIONS] = policy
        packed[:count, -2] = value
        packed[:count, -1] = to_play.to(torch.float32)
    return packed


class ReplayGather:
    """Appends every rank's new rows of `ring` to `fifo` on rank 0.

    `run(rows_written)` takes this rank's monotone count of rows written to its
    ring (the engine's ``rows`` counter). Rows that the ring overwrote before
    they were gathered (more than `ring.capacity` since the last call) are
    skipped: only the newest `ring.capacity` are sent.
    """

    def __init__(self, ring, fifo=None, group=None):
        self.ring, self.fifo, self.group = ring, fifo, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.sent = 0
        self.fifo_rows = 0  # rows appended to the FIFO so far (rank 0)
        if self.rank == 0 and fifo is None:
            raise ValueError("rank 0 needs a FIFO to gather into")

    def run(self, rows_written: int) -> int:
        """Gather; returns the number of rows appended on rank 0 (0 elsewhere)."""
        count = min(int(rows_written) - self.sent, self.ring.capacity)
        if count < 0:
            raise ValueError("rows_written went backwards")
        start = int(rows_written) - count
        device = self.ring.device
        sizes_t = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(self.world)]
        dist.all_gather(sizes_t, torch.tensor([count], dtype=torch.int64, device=device), group=self.group)
        sizes = [int(s.item()) for s in sizes_t]
        self.sent = int(rows_written)
        width = max(sizes)
        if width == 0:
            return 0
        packed = _pack(self.ring, start % self.ring.capacity, count, width)
        parts = [torch.empty_like(packed) for _ in range(self.world)]
        dist.all_gather(parts, packed, group=self.group)
        if self.rank != 0:
            return 0
        rows = torch.cat([parts[r][:sizes[r]] for r in range(self.world)])
        fifo = self.fifo
        if rows.shape[0] > fifo.capacity:  # only the newest rows survive a full lap
            self.fifo_rows += rows.shape[0] - fifo.capacity
            rows = rows[-fifo.capacity:]
        n = rows.shape[0]
        idx = (torch.arange(n, device=fifo.device) + self.fifo_rows) % fifo.capacity
        rows = rows.to(fifo.device)
        fifo.features.view(fifo.capacity, -1)[idx] = rows[:, :_FEATURES]
        fifo.masks[idx] = rows[:, _FEATURES:_FEATURES + _ACTIONS] != 0
        fifo.policy[idx] = rows[:, _FEATURES + _ACTIONS:_FEATURES + 2 * _ACTIONS]
        fifo.value[idx] = rows[:, -2]
        fifo.to_play[idx] = rows[:, -1].to(torch.int8)
        self.fifo_rows += n
        return n


def total_counters(counters: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of every rank's counters (int64 [8]), returned on every rank."""
    out = counters.clone()
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out
