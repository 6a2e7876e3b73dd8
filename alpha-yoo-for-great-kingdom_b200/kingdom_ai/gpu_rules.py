"""CUDA-resident game states in the reference's int32 [N,170] wire format.

Drop-in for ``kingdom_ai.gpu_rules`` (python/kingdom_ai/gpu_rules.py): the
same constants, the same ``GpuStateBatch`` methods, arguments, dtypes and
error behaviour. The kernels behind it are the bitboard rules of libgk.so
(``gk_initial_records``, ``gk_play_records``, ``gk_encode_records``), launched
on the current PyTorch stream.
"""

from __future__ import annotations

import torch

from . import _native as native

GPU_STATE_WIDTH = 170
GPU_CELL_COUNT = 81
GPU_ACTION_SIZE = 82
GPU_ACTOR = 162
GPU_BLACK_STOCK = 163
GPU_WHITE_STOCK = 164
GPU_PASSES = 165
GPU_REASON = 166
GPU_WINNER = 167
GPU_CAPTURED = 168
GPU_RESERVED = 169

GPU_NONE = 0
GPU_CAPTURE = 1
GPU_SUICIDE = 2
GPU_TWO_PASSES = 3

BITS_WIDTH = 16  # uint32 words per packed state (include/gk_common.h, gk_bits)

_REASON_BY_NAME = {"None_": GPU_NONE, "None": GPU_NONE, "Capture": GPU_CAPTURE, "Suicide": GPU_SUICIDE,
                   "TwoPasses": GPU_TWO_PASSES}


def _launch_scope(device, *tensors):
    """Current stream of `device`; marks tensors as used on it (allocator safety)."""
    stream = torch.cuda.current_stream(device)
    for tensor in tensors:
        if tensor is not None:
            tensor.record_stream(stream)
    return native.c_void_p(stream.cuda_stream)


def records_to_bits(records: torch.Tensor, check: bool = False) -> torch.Tensor:
    """Pack wire records into the engine's 64-byte bitboard states (int32 [N,16])."""
    n = records.shape[0]
    bits = torch.empty((n, BITS_WIDTH), dtype=torch.int32, device=records.device)
    status = torch.zeros(1, dtype=torch.int32, device=records.device) if check else None
    with torch.cuda.device(records.device):
        stream = _launch_scope(records.device, records, bits, status)
        native.call("gk_records_to_bits", native.ptr(records), native.ptr(bits), native.ptr(status), n, stream)
    if check and int(status.item()) != 0:
        raise ValueError("states hold values outside the [N,170] wire format's ranges")
    return bits


def bits_to_records(bits: torch.Tensor) -> torch.Tensor:
    n = bits.shape[0]
    records = torch.empty((n, GPU_STATE_WIDTH), dtype=torch.int32, device=bits.device)
    with torch.cuda.device(bits.device):
        stream = _launch_scope(bits.device, bits, records)
        native.call("gk_bits_to_records", native.ptr(bits), native.ptr(records), n, stream)
    return records


class GpuStateBatch:
    """CUDA int32 ``[N, 170]`` states using the confirmed default rules."""

    def __init__(self, states: torch.Tensor):
        if not isinstance(states, torch.Tensor):
            raise TypeError("states must be a torch Tensor")
        if states.device.type != "cuda" or states.dtype != torch.int32:
            raise ValueError("states must be CUDA int32 tensors")
        if states.ndim != 2 or states.shape[1] != GPU_STATE_WIDTH or states.shape[0] < 1:
            raise ValueError("states must have shape [N, 170] with N > 0")
        if not states.is_contiguous():
            raise ValueError("states must be contiguous")
        self.states = states

    @property
    def device(self):
        return self.states.device

    def __len__(self):
        return self.states.shape[0]

    @classmethod
    def initial(cls, n: int, device="cuda", neutral=(4, 4)):
        if type(n) is not int or n < 1:
            raise ValueError("n must be a positive integer")
        target = torch.device(device)
        if target.type != "cuda":
            raise ValueError("GpuStateBatch requires a CUDA device")
        if neutral is None:
            point = -1
        elif (isinstance(neutral, (tuple, list)) and len(neutral) == 2
              and all(type(value) is int and 0 <= value < 9 for value in neutral)):
            point = neutral[0] * 9 + neutral[1]
        else:
            raise ValueError("neutral must be None or a pair of coordinates in [0, 8]")
        states = torch.empty((n, GPU_STATE_WIDTH), device=target, dtype=torch.int32)
        result = cls(states)
        with torch.cuda.device(result.device):
            stream = _launch_scope(result.device, states)
            native.call("gk_initial_records", native.ptr(states), n, point, stream)
        return result

    @classmethod
    def from_records(cls, records, device="cuda"):
        """Import wire records (any int array-like [N,170]); values are range-checked."""
        target = torch.device(device)
        if target.type != "cuda":
            raise ValueError("GpuStateBatch requires a CUDA device")
        tensor = torch.as_tensor(records, dtype=torch.int32).to(device=target).contiguous()
        batch = cls(tensor)
        records_to_bits(batch.states, check=True)
        return batch

    @classmethod
    def from_engine(cls, states, device="cuda"):
        """Import CPU engine snapshots (``my_board_engine.State``), retaining ownership.

        Mirrors python/kingdom_ai/gpu_rules.py:376-413: default rules only,
        explicit reason translation (C++ EndReason orders TwoPasses before
        Suicide, the wire codes do not).
        """
        target = torch.device(device)
        if target.type != "cuda":
            raise ValueError("GpuStateBatch requires a CUDA device")
        snapshots = list(states)
        if not snapshots:
            raise ValueError("At least one engine State is required")
        records = []
        for state in snapshots:
            if not all(hasattr(state, name) for name in ("board", "ownership", "to_play", "result", "rules")):
                raise TypeError("Expected engine State snapshots")
            rules = state.rules
            if (getattr(rules.suicide_rule, "name", str(rules.suicide_rule)).split(".")[-1] != "Loses"
                    or rules.allow_own_territory_moves or not rules.allow_single_edge_territory
                    or rules.stones_per_player != 41):
                raise ValueError("Encoding v1 supports the confirmed default GameRules only")
            black, white = _engine_players(state)
            record = [int(cell) for cell in state.board.cells]
            record.extend(int(owner) for owner in state.ownership)
            reason = getattr(state.result.reason, "name", str(state.result.reason)).split(".")[-1]
            record.extend((
                int(state.to_play), state.remaining_stones(black), state.remaining_stones(white),
                state.consecutive_passes, _REASON_BY_NAME[reason], int(state.result.winner),
                state.result.captured_stones, 0,
            ))
            records.append(record)
        return cls(torch.tensor(records, dtype=torch.int32, device=target))

    def clone(self):
        return type(self)(self.states.clone())

    def play(self, actions):
        """Apply one action per state on-device; rejected states stay unchanged."""
        if isinstance(actions, torch.Tensor):
            action_tensor = actions
        else:
            action_tensor = torch.as_tensor(actions)
        if action_tensor.shape != (len(self),):
            raise ValueError("actions must have shape [N]")
        if action_tensor.dtype not in (torch.int32, torch.int64):
            raise TypeError("actions must be integer action indices")
        # int64 values outside [0, 82) are rejected by the kernel itself, so a
        # huge value never wraps into a legal int32 action.
        action_tensor = action_tensor.to(device=self.device).contiguous()
        accepted = torch.empty(len(self), device=self.device, dtype=torch.bool)
        with torch.cuda.device(self.device):
            stream = _launch_scope(self.device, self.states, action_tensor, accepted)
            native.call("gk_play_records", native.ptr(self.states), native.ptr(action_tensor),
                        action_tensor.element_size(), native.ptr(accepted), len(self), stream)
        return accepted

    def encode(self):
        """Return CUDA schema-1 features ``[N,10,9,9]`` and masks ``[N,82]``."""
        features = torch.empty((len(self), 10, 9, 9), device=self.device, dtype=torch.float32)
        masks = torch.empty((len(self), GPU_ACTION_SIZE), device=self.device, dtype=torch.bool)
        with torch.cuda.device(self.device):
            stream = _launch_scope(self.device, self.states, features, masks)
            native.call("gk_encode_records", native.ptr(self.states), native.ptr(features), native.ptr(masks),
                        len(self), stream)
        return features, masks

    def to_bits(self) -> torch.Tensor:
        """Packed 64-byte states (int32 [N,16]) for the search and self-play kernels."""
        return records_to_bits(self.states)

    def snapshot(self):
        """Synchronize and copy debug records to the CPU; never used in search."""
        return [{
            "cells": record[:GPU_CELL_COUNT],
            "ownership": record[GPU_CELL_COUNT:GPU_ACTOR],
            "actor": record[GPU_ACTOR],
            "black_stock": record[GPU_BLACK_STOCK],
            "white_stock": record[GPU_WHITE_STOCK],
            "passes": record[GPU_PASSES],
            "reason": record[GPU_REASON],
            "winner": record[GPU_WINNER],
            "captured_count": record[GPU_CAPTURED],
            "reserved": record[GPU_RESERVED],
        } for record in self.states.cpu().tolist()]


def _engine_players(state):
    """Black and White enum values of the engine module that made `state`."""
    cell_type = type(state.to_play)
    return cell_type.Black, cell_type.White
