"""GPU-resident replay buffer: validated bulk ingest and seeded sampling.

``DeviceReplayBuffer`` keeps the reference's ``ReplayBuffer`` contract
(python/kingdom_ai/replay.py:106-226) with its storage in device memory: a
FIFO ring measured in positions, atomic validated ``extend``, uniform
sampling with replacement from a caller-owned CPU generator, and the same
tensor-only checkpoint payload. Rows are validated by one CUDA kernel
(``gk_replay_validate``) instead of CPU tensor passes, and self-play rows can
be ingested straight from a device ``ReplayRing`` without a host round trip.
"""

from __future__ import annotations

from collections.abc import Iterable, Mapping

import torch

from . import _native as native
from .gpu_rules import _launch_scope
from .training import Cell, TrainingBatch, TrainingSample

ACTION_SIZE = 82
_STATE_VERSION = 1
_STATE_KEYS = {"version", "capacity", "size", "next_index", "features", "legal_mask", "policy", "value", "to_play"}
_SHAPES = {
    "features": ((10, 9, 9), torch.float32),
    "legal_mask": ((ACTION_SIZE,), torch.bool),
    "policy": ((ACTION_SIZE,), torch.float32),
    "value": ((), torch.float32),
    "to_play": ((), torch.int8),
}

# Messages of the reference's checks, in its order (replay.py:35-74); bit i of
# gk_replay_validate's result is check i.
MESSAGES = (
    "Replay features and policies must be finite",
    "Replay features must lie between zero and one",
    "Binary observation planes must contain only zero or one",
    "Scalar observation planes must be constant",
    "Replay actors must be Black or White",
    "Observation player perspective does not match its actor",
    "Replay observations must be taken before game termination",
    "Nonterminal replay observations must allow passing",
    "Observation legal placements do not match the action mask",
    "Stone observation planes cannot overlap",
    "An observation can contain at most one neutral stone",
    "Opposing territory observation planes cannot overlap",
    "Replay policies must assign non-negative mass to legal actions only",
    "Each replay policy must sum to one",
    "Completed-game replay values must be -1 or +1",
)


def _positive_integer(value, name):
    if isinstance(value, bool) or not isinstance(value, int) or value < 1:
        raise ValueError(f"{name} must be a positive integer")
    return value


def _rows(name, tensor, n, device):
    shape, dtype = _SHAPES[name]
    if not isinstance(tensor, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if tensor.layout != torch.strided or tuple(tensor.shape) != (n, *shape) or tensor.dtype != dtype:
        raise ValueError(f"{name} must have shape {(n, *shape)} and dtype {dtype}")
    return tensor.detach().to(device=device).contiguous()


def validate_rows(features, legal_mask, policy, value, to_play) -> None:
    """The reference's row checks (replay.py:35-74) on device tensors; raises
    ValueError with the reference's message for the first check that any row
    fails. The policy sum is taken in double (the reference sums in float32)."""
    n = features.shape[0]
    if n == 0:
        return
    flags = torch.empty(1, dtype=torch.int32, device=features.device)
    with torch.cuda.device(features.device):
        stream = _launch_scope(features.device, features, legal_mask, policy, value, to_play, flags)
        native.call("gk_replay_validate", native.ptr(features), native.ptr(legal_mask), native.ptr(policy),
                    native.ptr(value), native.ptr(to_play), n, native.ptr(flags), stream)
    code = int(flags.item()) & 0xFFFFFFFF
    if code:
        raise ValueError(MESSAGES[(code & -code).bit_length() - 1])


class DeviceReplayBuffer:
    """FIFO ring of training positions in device memory, sampled uniformly with
    replacement. Storage is ``capacity * 3655`` bytes of device memory."""

    def __init__(self, capacity: int, device="cuda"):
        self._capacity = _positive_integer(capacity, "Replay capacity")
        self.device = native.require_cuda(device)
        self._size = 0
        self._next_index = 0
        self._storage = {name: torch.empty((capacity, *shape), dtype=dtype, device=self.device)
                         for name, (shape, dtype) in _SHAPES.items()}

    @property
    def capacity(self) -> int:
        return self._capacity

    def __len__(self) -> int:
        return self._size

    def extend_rows(self, features, legal_mask, policy, value, to_play) -> None:
        """Validate every incoming row, then write them (all or nothing).
        Rows that a single call would evict at once are skipped, but their ring
        slots still advance, as ReplayBuffer.extend does (replay.py:133-161)."""
        n = features.shape[0] if isinstance(features, torch.Tensor) else -1
        if n < 0:
            raise TypeError("features must be a tensor")
        rows = {name: _rows(name, t, n, self.device)
                for name, t in zip(_SHAPES, (features, legal_mask, policy, value, to_play))}
        if n == 0:
            return
        validate_rows(*rows.values())
        skipped = max(0, n - self._capacity)
        index = (self._next_index + skipped) % self._capacity
        offset = skipped
        while offset < n:
            count = min(n - offset, self._capacity - index)
            for name, t in rows.items():
                self._storage[name][index:index + count].copy_(t[offset:offset + count])
            offset += count
            index = (index + count) % self._capacity
        self._next_index = index
        self._size = min(self._capacity, self._size + n)

    def extend(self, samples: Iterable[TrainingSample]) -> None:
        """ReplayBuffer.extend for TrainingSample objects (replay.py:133-161)."""
        incoming = list(samples)
        if not incoming:
            return
        for s in incoming:
            if not isinstance(s, TrainingSample):
                raise TypeError("Replay entries must be TrainingSample objects")
            if isinstance(s.value, bool) or not isinstance(s.value, (int, float)) or s.value not in (-1, 1):
                raise ValueError("Sample value must be -1 or +1")
            if not isinstance(s.to_play, Cell) or s.to_play not in (Cell.Black, Cell.White):
                raise ValueError("Sample actor must be Black or White")
        stacked = []
        for name in ("features", "legal_mask", "policy"):
            shape, dtype = _SHAPES[name]
            parts = []
            for s in incoming:
                t = getattr(s, name)
                if not isinstance(t, torch.Tensor) or tuple(t.shape) != shape or t.dtype != dtype:
                    raise ValueError(f"{name} must have shape {shape} and dtype {dtype}")
                parts.append(t.detach())
            home = parts[0].device
            stacked.append(torch.stack([p if p.device == home else p.to(home) for p in parts]).to(self.device))
        value = torch.tensor([float(s.value) for s in incoming], dtype=torch.float32, device=self.device)
        to_play = torch.tensor([1 if s.to_play == Cell.Black else 2 for s in incoming], dtype=torch.int8,
                               device=self.device)
        self.extend_rows(*stacked, value, to_play)

    def ingest(self, ring, start: int, count: int) -> None:
        """Append `count` rows of a self-play ReplayRing from ring row `start`."""
        if count <= 0:
            return
        self.extend_rows(*ring.rows(start, count))

    def sample(self, batch_size: int, *, generator: torch.Generator, device=None) -> TrainingBatch:
        """An independent batch drawn with replacement; the indices come from the
        caller's CPU generator exactly as in ReplayBuffer.sample (replay.py:163-177)."""
        _positive_integer(batch_size, "Batch size")
        if not isinstance(generator, torch.Generator) or generator.device.type != "cpu":
            raise ValueError("Replay sampling requires a caller-owned CPU torch.Generator")
        if self._size == 0:
            raise ValueError("Cannot sample an empty replay buffer")
        indices = torch.randint(self._size, (batch_size,), generator=generator, device="cpu").to(self.device)
        target = self.device if device is None else torch.device(device)
        s = self._storage
        return TrainingBatch(s["features"].index_select(0, indices).to(target),
                             s["legal_mask"].index_select(0, indices).to(target),
                             s["policy"].index_select(0, indices).to(target),
                             s["value"].index_select(0, indices).to(target))

    def state_dict(self) -> dict:
        """The reference's checkpoint payload (replay.py:179-191): CPU copies of
        the occupied slots, so a reference ReplayBuffer can load it."""
        payload = {"version": _STATE_VERSION, "capacity": self._capacity, "size": self._size,
                   "next_index": self._next_index}
        for name in _SHAPES:
            payload[name] = self._storage[name][:self._size].to("cpu", copy=True)
        return payload

    @classmethod
    def from_state_dict(cls, payload: Mapping, device="cuda") -> "DeviceReplayBuffer":
        """Restore a validated checkpoint (replay.py:193-226), rows checked on the GPU."""
        if not isinstance(payload, Mapping) or set(payload) != _STATE_KEYS:
            raise ValueError("Unexpected replay checkpoint fields")
        version = payload["version"]
        if isinstance(version, bool) or not isinstance(version, int) or version != _STATE_VERSION:
            raise ValueError("Unsupported replay checkpoint version")
        capacity = _positive_integer(payload["capacity"], "Replay capacity")
        size, next_index = payload["size"], payload["next_index"]
        if isinstance(size, bool) or not isinstance(size, int) or not 0 <= size <= capacity:
            raise ValueError("Replay checkpoint size is outside capacity")
        if (isinstance(next_index, bool) or not isinstance(next_index, int) or not 0 <= next_index < capacity
                or (size < capacity and next_index != size)):
            raise ValueError("Replay checkpoint ring index is inconsistent")
        restored = cls(capacity, device)
        rows = {name: _rows(name, payload[name], size, restored.device) for name in _SHAPES}
        validate_rows(*rows.values())
        for name, t in rows.items():
            restored._storage[name][:size].copy_(t)
        restored._size = size
        restored._next_index = next_index
        return restored
