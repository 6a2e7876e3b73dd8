"""GPU-resident replay buffer: the reference's ReplayBuffer tests (tests/replay_test.py)
replayed on DeviceReplayBuffer, and the CUDA row checks against the oracle's
restatement of replay.py:35-74."""

import re

import numpy as np
import pytest
import torch

from test_oracle import replay_corruptions, replay_sample

pytestmark = pytest.mark.gpu


def sample(oracle, index=0, white=False):
    from kingdom_ai import Cell, TrainingSample
    f, m, p, v, t = replay_sample(oracle, index, white)
    return TrainingSample(torch.from_numpy(f[0]), torch.from_numpy(m[0]), torch.from_numpy(p[0]), float(v[0]),
                          Cell.White if white else Cell.Black)


def generator(seed=17):
    return torch.Generator(device="cpu").manual_seed(seed)


def state_equal(a, b):
    assert set(a) == set(b)
    for key, before in a.items():
        if isinstance(before, torch.Tensor):
            assert torch.equal(before, b[key]), key
        else:
            assert before == b[key], key


def device_rows(row, copies=1):
    return [torch.from_numpy(np.repeat(np.asarray(row[k]), copies, axis=0)).cuda()
            for k in ("features", "legal_mask", "policy", "value", "to_play")]


def test_cuda_checks_report_the_reference_messages(oracle):
    from kingdom_ai import validate_rows
    from oracle.oracle import replay_violation
    f, m, p, v, t = replay_sample(oracle)
    good = dict(features=f, legal_mask=m, policy=p, value=v, to_play=t)
    validate_rows(*device_rows(good, 3000))
    for message, bad in replay_corruptions(oracle):
        assert replay_violation(**bad) == message
        rows = [torch.cat([a, b, a]) for a, b in zip(device_rows(good, 700), device_rows(bad))]
        with pytest.raises(ValueError, match=re.escape(message)):
            validate_rows(*rows)


def test_selfplay_rows_pass_and_mixed_corruptions_match_the_oracle(oracle):
    from kingdom_ai import validate_rows
    from kingdom_ai.model import random_network
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.selfplay import SelfPlayEngine
    from oracle.oracle import replay_violation

    engine = SelfPlayEngine(random_network(64, 2, 3), 128, GpuPUCTOptions(simulations=8, seed=3),
                            replay_capacity=1 << 14)
    engine.step(60)
    n = min(engine.stats()["rows"], engine.replay.capacity)
    assert n > 100
    rows = list(engine.replay.rows(0, n))
    validate_rows(*rows)
    host = [r.cpu().numpy() for r in rows]
    assert replay_violation(*host) is None
    rng = np.random.default_rng(4)
    corruptions = [
        lambda r, i: r[0].__setitem__((i, 3, 4, 4), 0.25),
        lambda r, i: r[0].__setitem__((i, 7, 2, 2), 0.125),
        lambda r, i: r[1].__setitem__((i, int(rng.integers(81))), True),
        lambda r, i: r[2].__setitem__((i, 5), r[2][i, 5] + 1e-3),
        lambda r, i: r[3].__setitem__(i, 0.5),
        lambda r, i: r[0].__setitem__((i, 2, 0, 0), 1.0),
        lambda r, i: r[4].__setitem__(i, 0),
    ]
    for trial in range(24):
        bad = [h.copy() for h in host]
        for _ in range(int(rng.integers(1, 4))):
            corruptions[int(rng.integers(len(corruptions)))](bad, int(rng.integers(n)))
        expected = replay_violation(*bad)
        tensors = [torch.from_numpy(b).cuda() for b in bad]
        if expected is None:
            validate_rows(*tensors)
        else:
            with pytest.raises(ValueError, match=re.escape(expected)):
                validate_rows(*tensors)


def test_capacity_fifo_order_and_bulk_equals_sequential(oracle):
    from kingdom_ai import Cell, DeviceReplayBuffer
    buffer = DeviceReplayBuffer(3)
    assert buffer.capacity == 3 and len(buffer) == 0
    buffer.extend(sample(oracle, i) for i in range(5))
    saved = buffer.state_dict()
    assert saved["next_index"] == 2 and saved["policy"].argmax(dim=1).tolist() == [3, 4, 2]
    buffer.extend([sample(oracle, 5)])
    saved = buffer.state_dict()
    assert saved["next_index"] == 0 and saved["policy"].argmax(dim=1).tolist() == [3, 4, 5]
    bulk, sequential = DeviceReplayBuffer(3), DeviceReplayBuffer(3)
    first = sample(oracle, 20, white=True)
    bulk.extend([first])
    sequential.extend([first])
    incoming = [sample(oracle, i) for i in range(9)]
    bulk.extend(incoming)
    for s in incoming:
        sequential.extend([s])
    state_equal(bulk.state_dict(), sequential.state_dict())
    assert bulk.state_dict()["to_play"].tolist() == [1, 1, 1]
    for capacity in (0, -1, True, 3.0, "3"):
        with pytest.raises(ValueError):
            DeviceReplayBuffer(capacity)
    assert Cell.White == 2


def test_atomic_bulk_validation_and_wrapped_overcapacity_append(oracle):
    from dataclasses import replace
    from kingdom_ai import DeviceReplayBuffer
    entries = [sample(oracle, i) for i in range(5)] * 820
    buffer = DeviceReplayBuffer(3)
    buffer.extend(entries)
    saved = buffer.state_dict()
    assert saved["next_index"] == len(entries) % 3 and saved["policy"].argmax(dim=1).tolist() == [3, 4, 2]
    with pytest.raises(ValueError):
        buffer.extend([sample(oracle, 0)] * 4096 + [replace(sample(oracle, 1), value=0.0)])
    state_equal(saved, buffer.state_dict())
    capacity = 4099
    bulk, incremental = DeviceReplayBuffer(capacity), DeviceReplayBuffer(capacity)
    initial = [sample(oracle, i) for i in range(73)]
    bulk.extend(initial)
    incremental.extend(initial)
    incoming = [sample(oracle, i + 7) for i in range(capacity + 19)]
    bulk.extend(incoming)
    for start in range(0, len(incoming), 97):
        incremental.extend(incoming[start:start + 97])
    state_equal(bulk.state_dict(), incremental.state_dict())


def test_seeded_sampling_and_checkpoint_round_trip(oracle):
    from kingdom_ai import DeviceReplayBuffer
    buffer = DeviceReplayBuffer(7)
    with pytest.raises(ValueError):
        buffer.sample(1, generator=generator())
    buffer.extend(sample(oracle, i, white=i % 3 == 0) for i in range(11))
    with pytest.raises(ValueError):
        buffer.sample(0, generator=generator())
    with pytest.raises(ValueError):
        buffer.sample(2, generator=None)
    batch = buffer.sample(33, generator=generator())
    saved = buffer.state_dict()
    indices = torch.randint(len(buffer), (33,), generator=generator())
    assert torch.equal(batch.features.cpu(), saved["features"][indices])
    assert torch.equal(batch.legal_mask.cpu(), saved["legal_mask"][indices])
    assert torch.equal(batch.policy.cpu(), saved["policy"][indices])
    assert torch.equal(batch.value.cpu(), saved["value"][indices])
    restored = DeviceReplayBuffer.from_state_dict(saved)
    again = restored.sample(33, generator=generator(), device="cpu")
    assert torch.equal(again.features, batch.features.cpu()) and torch.equal(again.value, batch.value.cpu())
    small = DeviceReplayBuffer(3)
    small.extend([sample(oracle, 0), sample(oracle, 1)])
    payload = small.state_dict()
    invalid = [None, {}, dict(payload, extra=1), dict(payload, version=True), dict(payload, version=2),
               dict(payload, capacity=0), dict(payload, capacity=True), dict(payload, size=-1),
               dict(payload, size=4), dict(payload, size=True), dict(payload, next_index=0),
               dict(payload, next_index=3), dict(payload, next_index=True),
               dict(payload, features=payload["features"].double()),
               dict(payload, to_play=payload["to_play"].long())]
    for field, index, value in (("features", (0, 0, 0, 0), float("nan")), ("policy", (0, 40), 1.0),
                                ("value", 0, 0.0), ("to_play", 0, 0)):
        bad = dict(payload)
        bad[field] = payload[field].clone()
        bad[field][index] = value
        invalid.append(bad)
    for checkpoint in invalid:
        with pytest.raises((TypeError, ValueError)):
            DeviceReplayBuffer.from_state_dict(checkpoint)


def test_ingest_from_selfplay_ring(oracle):
    from kingdom_ai import DeviceReplayBuffer
    from kingdom_ai.model import random_network
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.selfplay import SelfPlayEngine
    engine = SelfPlayEngine(random_network(64, 2, 5), 64, GpuPUCTOptions(simulations=8, seed=9),
                            replay_capacity=1 << 12)
    engine.step(50)
    n = min(engine.stats()["rows"], engine.replay.capacity)
    buffer = DeviceReplayBuffer(1 << 12)
    buffer.ingest(engine.replay, 0, n)
    assert len(buffer) == n
    rows = engine.replay.rows(0, n)
    saved = buffer.state_dict()
    assert torch.equal(saved["features"], rows[0].cpu()) and torch.equal(saved["to_play"], rows[4].cpu())
