"""Multi-rank host logic of sharded self-play on CPU (gloo, world size 2).

Games shard with no data-path exchange; the collectives are the replay-row
gather into rank 0's FIFO and the counter sum (kingdom_ai/distributed.py).
Two gloo ranks drive them here with rings of known rows: uneven per-rank
counts (padding), ring wrap-around, a rank that outran its ring (only the
newest rows survive), a rank with nothing new, and a FIFO that wraps.
"""

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
RING, FIFO = 8, 32
# Cumulative rows written per rank before each gather.
ROUNDS = [(5, 3), (11, 9), (23, 9), (23, 17)]


def _row_value(rank, i):
    return float(rank * 1000 + i)


def _write(ring, rank, first, last):
    for i in range(first, last):
        j = i % ring.capacity
        v = _row_value(rank, i)
        ring.features[j].fill_(v)
        ring.masks[j] = (torch.arange(82) + i + rank) % 3 == 0
        ring.policy[j].fill_(v / 7.0)
        ring.value[j] = 1.0 if (i + rank) % 2 == 0 else -1.0
        ring.to_play[j] = (i + rank) % 2


def _worker(rank, world, port, out):
    sys.path[:0] = [str(ROOT), str(ROOT / "alpha-yoo-for-great-kingdom_b200")]
    import torch.distributed as dist

    from kingdom_ai.distributed import ReplayGather, total_counters
    from kingdom_ai.selfplay import ReplayRing

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ring = ReplayRing(RING, "cpu")
        fifo = ReplayRing(FIFO, "cpu") if rank == 0 else None
        gather = ReplayGather(ring, fifo)
        written, appended = 0, []
        for counts in ROUNDS:
            _write(ring, rank, written, counts[rank])
            written = counts[rank]
            appended.append(gather.run(written))
        totals = total_counters(torch.arange(8, dtype=torch.int64) + 10 * rank)
        if rank == 0:
            torch.save({"appended": appended, "totals": totals, "fifo_rows": gather.fifo_rows,
                        "features": fifo.features.clone(), "masks": fifo.masks.clone(),
                        "policy": fifo.policy.clone(), "value": fifo.value.clone(),
                        "to_play": fifo.to_play.clone()}, out)
    finally:
        dist.destroy_process_group()


def _expected_rows():
    """(rank, row index) in FIFO order: per round, rank 0's new rows then rank 1's."""
    rows, sent = [], [0, 0]
    for counts in ROUNDS:
        for rank in (0, 1):
            first = max(sent[rank], counts[rank] - RING)  # overwritten rows are skipped
            rows += [(rank, i) for i in range(first, counts[rank])]
            sent[rank] = counts[rank]
    return rows


@pytest.fixture(scope="module")
def gathered(tmp_path_factory):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path_factory.mktemp("gather") / "rank0.pt"
    mp.spawn(_worker, args=(2, port, str(out)), nprocs=2, join=True)
    return torch.load(out)


def test_rows_arrive_in_rank_order_with_overwritten_rows_skipped(gathered):
    rows = _expected_rows()
    per_round = []
    sent = [0, 0]
    for counts in ROUNDS:
        n = sum(counts[r] - max(sent[r], counts[r] - RING) for r in (0, 1))
        per_round.append(n)
        sent = list(counts)
    assert gathered["appended"] == per_round
    assert gathered["fifo_rows"] == len(rows) == sum(per_round)
    # The FIFO wrapped: slot k holds the newest row whose position is k mod FIFO.
    for pos, (rank, i) in enumerate(rows):
        if pos + FIFO < len(rows):
            continue  # overwritten by a later row
        k = pos % FIFO
        v = _row_value(rank, i)
        assert torch.all(gathered["features"][k] == v), (pos, rank, i)
        assert torch.equal(gathered["masks"][k], (torch.arange(82) + i + rank) % 3 == 0)
        assert torch.allclose(gathered["policy"][k], torch.full((82,), v / 7.0))
        assert gathered["value"][k].item() == (1.0 if (i + rank) % 2 == 0 else -1.0)
        assert gathered["to_play"][k].item() == (i + rank) % 2


def test_counters_sum_over_ranks(gathered):
    assert torch.equal(gathered["totals"], 2 * torch.arange(8, dtype=torch.int64) + 10)
