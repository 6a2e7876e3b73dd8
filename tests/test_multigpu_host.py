"""Multi-rank host logic of sharded self-play on CPU (gloo, world size 2).

Games shard with no data-path exchange; the collectives are the replay-row
gather into rank 0's FIFO and the counter sum (kingdom_ai/distributed.py).
Two gloo ranks drive them here with rings of known rows: uneven per-rank
counts (padding), ring wrap-around, a rank that outran its ring (only the
newest rows survive), a rank with nothing new, and a FIFO that wraps; and
again with a slab narrower than a round's new rows, whose excess waits for
the next gather.
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


def _worker(rank, world, port, out, width):
    sys.path[:0] = [str(ROOT), str(ROOT / "alpha-yoo-for-great-kingdom_b200")]
    import torch.distributed as dist

    from kingdom_ai.distributed import ReplayGather, total_counters
    from kingdom_ai.selfplay import ReplayRing

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ring = ReplayRing(RING, "cpu")
        fifo = ReplayRing(FIFO, "cpu") if rank == 0 else None
        gather = ReplayGather(ring, fifo, width=width)
        written, appended = 0, []
        for counts in ROUNDS:
            _write(ring, rank, written, counts[rank])
            written = counts[rank]
            # The count goes in as a tensor, as the engine's device counters do.
            got = gather.run(torch.tensor(written))
            appended.append(None if got is None else int(got))
        totals = total_counters(torch.arange(8, dtype=torch.int64) + 10 * rank)
        if rank == 0:
            torch.save({"appended": appended, "totals": totals, "fifo_rows": gather.fifo_rows,
                        "features": fifo.features.clone(), "masks": fifo.masks.clone(),
                        "policy": fifo.policy.clone(), "value": fifo.value.clone(),
                        "to_play": fifo.to_play.clone()}, out)
    finally:
        dist.destroy_process_group()


def _expected_rounds(width):
    """Per round, the (rank, row index) pairs appended: rank 0's rows, then
    rank 1's, each rank sending its oldest rows not yet sent, at most `width`,
    after skipping rows its ring overwrote."""
    rounds, sent = [], [0, 0]
    for counts in ROUNDS:
        rows = []
        for rank in (0, 1):
            first = max(sent[rank], counts[rank] - RING)
            last = min(counts[rank], first + width)
            rows += [(rank, i) for i in range(first, last)]
            sent[rank] = last
        rounds.append(rows)
    return rounds


def _run(tmp_path_factory, width):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path_factory.mktemp("gather") / "rank0.pt"
    mp.spawn(_worker, args=(2, port, str(out), width), nprocs=2, join=True)
    return torch.load(out)


@pytest.fixture(scope="module")
def gathered(tmp_path_factory):
    return _run(tmp_path_factory, RING)


@pytest.fixture(scope="module")
def gathered_narrow(tmp_path_factory):
    return _run(tmp_path_factory, 3)


def _check(gathered, width):
    rounds = _expected_rounds(width)
    rows = [r for rnd in rounds for r in rnd]
    assert gathered["appended"] == [len(rnd) for rnd in rounds]
    assert gathered["fifo_rows"] == len(rows)
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


def test_rows_arrive_in_rank_order_with_overwritten_rows_skipped(gathered):
    _check(gathered, RING)


def test_a_narrow_slab_defers_rows_to_the_next_gather(gathered_narrow):
    _check(gathered_narrow, 3)


def test_counters_sum_over_ranks(gathered):
    assert torch.equal(gathered["totals"], 2 * torch.arange(8, dtype=torch.int64) + 10)
