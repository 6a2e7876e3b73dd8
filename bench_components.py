"""Per-kernel benchmarks behind `bench.py --workload ...` (one JSON line each).

    network  leaf evaluation: `--net CxR --batch B` (default 10 x 128ch, 8192 positions)
    rules    4096 uniform-random complete playouts, and one transition of 2^22 packed states
    encode   observation planes + legal masks for 65,536 and 2^20 generated positions
    puct     1024 trees x 800 simulations with the injected evaluator
    replay   replay-row checks of DeviceReplayBuffer ingest on 2^20 rows (3.66 GB)
    batched  the evaluation searcher (BatchedPUCT) for 4096 games x 128 simulations, leaf batch 8
    selfplay_reference  self-play with the reference's 32 x 2 GroupNorm network and its 128 simulations
    evaluation  a 512-game evaluation match between two 6 x 64 networks (evaluate_models_gpu)
    collect  the Trainer's hook: collect_gpu_puct_games for --games games, --lanes in flight

Every timed launch is bracketed by CUDA events on the launching stream; an L2
flush (a 256 MB write) separates timed launches so each one reads its inputs
from HBM.
"""

from __future__ import annotations

import json

import torch

from kingdom_ai import _native as native

L2_FLUSH_BYTES = 256 << 20


class Flusher:
    def __init__(self, device):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    def __call__(self):
        self.buf.fill_(1)


def timed(fn, steps, warmup, flush):
    """Average milliseconds of `fn` over `steps` launches (events per launch)."""
    for _ in range(warmup):
        fn()
    total = 0.0
    for _ in range(steps):
        flush()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        stop.record()
        stop.synchronize()
        total += start.elapsed_time(stop)
    return total / steps


def positions(n, seed, device):
    bits = torch.empty((n, 16), dtype=torch.int32, device=device)
    native.call("gk_gen_positions", seed, 0, n, native.ptr(bits), native.stream_of(device))
    return bits


def emit(line):
    print(json.dumps(line), flush=True)


def host_cores():
    import os
    return len(os.sched_getaffinity(0))


def _reference():
    """The reference engine compiled from its sources (oracle/_ref), or None."""
    try:
        from oracle.oracle import Reference
        return Reference()
    except Exception:  # noqa: BLE001 - the caller reports the baseline as unavailable
        return None


def network_error(model, net, bits):
    """Max |native bf16 - PyTorch fp32| on logits and values over `bits`
    positions (TF32 off, so the reference forward is true fp32)."""
    from kingdom_ai.gpu_puct import encode_packed

    features, _ = encode_packed(bits)
    tf32 = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            ref_logits, ref_values = model.to(bits.device).float().eval()(features)
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = tf32
    logits, values = net.forward_states(bits)
    net.check()
    return {"positions": int(bits.shape[0]),
            "fp32_max_abs_logit": float((logits - ref_logits).abs().max()),
            "fp32_max_abs_value": float((values - ref_values).abs().max()),
            "fp32_max_logit_magnitude": float(ref_logits.abs().max())}


def bench_network(args, peaks):
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import (NativePolicyValueNet, calibrate_batchnorm, random_groupnorm_network,
                                  random_network)

    device = torch.device("cuda", 0)
    channels, blocks = (int(x) for x in args.net.split("x"))
    n = args.batch
    group = args.norm == "group"
    model = (random_groupnorm_network if group else random_network)(channels, blocks, 1234).to(device)
    bits = positions(n, 4321, device)
    features, _ = encode_packed(bits)
    if not group:
        calibrate_batchnorm(model, features)
    net = NativePolicyValueNet(model.cpu(), device)
    flush = Flusher(device)
    ms = timed(lambda: net.forward_states(bits), args.steps, args.warmup, flush)
    net.check()
    hidden = channels if group else 64
    flops = 2 * 81 * 9 * 10 * channels + 2 * blocks * 2 * 81 * 9 * channels * channels + 2 * 81 * (
        channels * 3 + 162 * 82 + 81 * hidden + hidden)
    tflops = n * flops / (ms / 1e3) / 1e12
    error = network_error(model, net, bits)
    model = model.to(device)
    with torch.no_grad():
        t_ref = timed(lambda: model(features), max(1, args.steps // 2), 1, flush)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            t_amp = timed(lambda: model(features), max(1, args.steps // 2), 1, flush)
    cpu = None
    try:
        import time
        cores = host_cores()
        threads = torch.get_num_threads()
        torch.set_num_threads(cores)
        cpu_model, sample = model.cpu().float().eval(), features[:128].cpu()
        with torch.no_grad():
            cpu_model(sample[:8])
            start, reps = time.perf_counter(), 0
            while reps < 1 or time.perf_counter() - start < 3.0:
                cpu_model(sample)
                reps += 1
        elapsed = time.perf_counter() - start
        torch.set_num_threads(threads)
        cpu = {"value": reps * len(sample) / elapsed, "unit": "positions/s", "cores": cores, "kind": "port",
               "sample": f"{reps} fp32 PyTorch CPU forwards of {len(sample)} positions ({cores} threads), "
                         f"{elapsed:.1f} s"}
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        cpu = {"value": None, "unavailable": str(exc)}
    kind = "GroupNorm (the reference's PolicyValueNet)" if group else "batch norm folded"
    return {"workload": f"network forward {channels}ch x {blocks} blocks, {kind}, batch {n}", "metric": "positions/s",
            "value": n / (ms / 1e3), "unit": "positions/s", "ms_per_batch": ms, "dtype": "bf16",
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks[3], "unit": "TFLOP/s",
                         "frac": tflops / peaks[3], "peak_kind": f"{peaks[2]} bf16 burst (kernel timed alone)",
                         "flops_per_position": flops},
            "error_vs_fp32": error, "pytorch_fp32_ms": t_ref, "pytorch_bf16_autocast_ms": t_amp,
            "cpu_baseline": cpu}


def bench_rules(args, peaks):
    import time

    device = torch.device("cuda", 0)
    flush = Flusher(device)
    n = 4096
    boards = torch.empty((n, 81), dtype=torch.int8, device=device)
    infos = torch.empty((n, 5), dtype=torch.int32, device=device)
    stream = native.stream_of(device)
    ms = timed(lambda: native.call("gk_random_playouts", 2024, 0, n, 40, native.ptr(boards), native.ptr(infos),
                                   stream), args.steps, args.warmup, flush)
    plies = int(infos[:, 4].sum().item())
    big = args.states
    bits = positions(big, 99, device)
    work = bits.clone()
    actions = torch.randint(0, 82, (big,), dtype=torch.int32, device=device)
    accepted = torch.empty(big, dtype=torch.bool, device=device)
    # A copy restores the inputs before each launch; the transition alone is timed.
    total = 0.0
    for i in range(args.warmup + args.steps):
        work.copy_(bits)
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        native.call("gk_play_bits", native.ptr(work), native.ptr(actions), 4, native.ptr(accepted), big, stream)
        e.record()
        e.synchronize()
        if i >= args.warmup:
            total += s.elapsed_time(e)
    play_ms = total / args.steps
    bytes_per_state = 64 + 4 + 64 + 1
    gbs = big * bytes_per_state / (play_ms / 1e3) / 1e9
    ref, cpu = _reference(), None
    if ref is not None:
        cores = host_cores()
        rates = {}
        for fast, name in ((0, "legal_moves"), (1, "candidates")):
            start = time.perf_counter()
            _, ref_infos = ref.random_playouts(2024, n, fast=bool(fast), threads=cores)
            rates[name] = int(ref_infos[:, 4].sum()) / (time.perf_counter() - start)
        cpu = {"value": rates["legal_moves"], "unit": "moves/s", "cores": cores, "kind": "reference",
               "candidates_moves_per_s": rates["candidates"],
               "sample": f"the same {n} playouts through kingdom::State::play on {cores} threads, legal moves "
                         "from State::legal_moves() (value) and from the MCTS::candidates rule"}
    return {"workload": f"rules: 4096 uniform-random complete playouts; one transition of {big} packed states",
            "metric": "playout moves/s", "value": plies / (ms / 1e3), "unit": "moves/s",
            "games_per_s": n / (ms / 1e3), "playout_ms": ms, "mean_plies": plies / n,
            "play_kernel": {"states": big, "ms": play_ms, "states_per_s": big / (play_ms / 1e3)},
            "roofline": {"bound": "hbm", "kernel": "play_bits_kernel", "achieved": gbs, "peak": peaks[1],
                         "unit": "GB/s", "frac": gbs / peaks[1], "bytes_per_state": bytes_per_state},
            "cpu_baseline": cpu}


def bench_encode(args, peaks):
    device = torch.device("cuda", 0)
    flush = Flusher(device)
    stream = native.stream_of(device)
    out = {}
    small, big = args.positions, 1 << 20
    for n in (small, big):
        bits = positions(n, 11, device)
        feats = torch.empty((n, 10, 9, 9), dtype=torch.float32, device=device)
        masks = torch.empty((n, 82), dtype=torch.bool, device=device)
        ms = timed(lambda: native.call("gk_encode_bits", native.ptr(bits), native.ptr(feats), native.ptr(masks), n,
                                       stream), args.steps, args.warmup, flush)
        out[n] = ms
    bytes_per_pos = 64 + 3240 + 82
    n = small
    gbs = n * bytes_per_pos / (out[n] / 1e3) / 1e9
    gbs_big = big * bytes_per_pos / (out[big] / 1e3) / 1e9
    ref, cpu = _reference(), None
    if ref is not None:
        cores = host_cores()
        seconds, _, _ = ref.encode_timed(11, n, threads=cores)
        cpu = {"value": n / seconds, "unit": "positions/s", "cores": cores, "kind": "reference",
               "sample": f"kingdom::encode_puct_position over the same {n} generated positions on {cores} threads "
                         "(generation excluded)"}
    return {"workload": f"encode {n} generated positions (and 2^20)", "metric": "positions/s",
            "value": n / (out[n] / 1e3), "unit": "positions/s", "ms": out[n], "ms_2pow20": out[big],
            "roofline": {"bound": "hbm", "kernel": "encode_bits_kernel", "achieved": gbs, "peak": peaks[1],
                         "unit": "GB/s", "frac": gbs / peaks[1], "bytes_per_position": bytes_per_pos,
                         "achieved_2pow20": gbs_big, "frac_2pow20": gbs_big / peaks[1]},
            "cpu_baseline": cpu}


def puct_bytes_per_simulation(mean_depth: float) -> float:
    """Algorithmic HBM bytes of one simulation: every level of the descent
    reads the node's 82 edges (N i32, W f64, P f64 = 20 B each) and writes a
    12-byte backup; the leaf's expansion writes one 20-byte row of 82 edges;
    the new child state and its scalars take 96 B."""
    return mean_depth * (82 * 20 + 12) + 82 * 20 + 96


def bench_puct(args, peaks):
    import time

    from kingdom_ai.gpu_puct import SearchWorkspace, search_hash

    device = torch.device("cuda", 0)
    flush = Flusher(device)
    n, sims = args.trees, args.sims
    bits = positions(n, 4242, device)
    ws = SearchWorkspace(n, sims + 1, device)
    holder = {}

    def run():
        holder["r"] = search_hash(bits, sims, workspace=ws)

    ms = timed(run, max(1, args.steps // 3), 1, flush)
    r = holder["r"]
    assert int(r.simulations.sum().item()) == n * sims
    # Mean selection depth: each simulation adds one visit to every non-root
    # node on its path, so the visits of all non-root nodes sum to the total depth.
    live = torch.arange(sims + 1, device=device)[None, :] < r.nodes[:, None]
    depth_total = (ws.node_visits * live)[:, 1:].sum().item()
    mean_depth = depth_total / (n * sims)
    bps = puct_bytes_per_simulation(mean_depth)
    gbs = n * sims * bps / (ms / 1e3) / 1e9
    ref, cpu = _reference(), None
    if ref is not None:
        cores = host_cores()
        m = min(n, 8 * cores)
        start = time.perf_counter()
        visits, best = ref.puct_positions(4242, m, sims, threads=cores)
        elapsed = time.perf_counter() - start
        assert (visits == r.visits[:m].cpu().numpy()).all(), "reference visits differ from the device search"
        cpu = {"value": m * sims / elapsed, "unit": "simulations/s", "cores": cores, "kind": "reference",
               "sample": f"kingdom::PUCT::search over the first {m} of the same roots ({sims} simulations, injected "
                         f"evaluator) on {cores} threads, {elapsed:.2f} s; visit counts equal the device's"}
    return {"workload": f"PUCT {n} trees x {sims} simulations, injected evaluator, c_puct 1.5",
            "metric": "simulations/s", "value": n * sims / (ms / 1e3), "unit": "simulations/s",
            "ms_per_search": ms, "nodes_mean": float(r.nodes.float().mean().item()),
            "roofline": {"bound": "hbm", "kernel": "puct_search_hash_kernel", "achieved": gbs, "peak": peaks[1],
                         "unit": "GB/s", "frac": gbs / peaks[1], "mean_depth": mean_depth,
                         "bytes_per_simulation": bps,
                         "bytes_rule": "d*(82*20+12) + 82*20 + 96 with d the measured mean selection depth"},
            "cpu_baseline": cpu}


def bench_replay(args, peaks):
    """gk_replay_validate over `--rows` valid replay rows (the reference's
    ReplayBuffer ingest checks, replay.py:35-74); CPU baseline: the numpy
    restatement of the same checks on a bounded sample, one thread."""
    import time

    device = torch.device("cuda", 0)
    flush = Flusher(device)
    stream = native.stream_of(device)
    n = args.rows
    bits = positions(n, 29, device)
    feats = torch.empty((n, 10, 9, 9), dtype=torch.float32, device=device)
    masks = torch.empty((n, 82), dtype=torch.bool, device=device)
    native.call("gk_encode_bits", native.ptr(bits), native.ptr(feats), native.ptr(masks), n, stream)
    del bits
    policy = masks.float() / masks.sum(dim=1, keepdim=True).float()
    value = torch.where(torch.arange(n, device=device) % 3 == 0, 1.0, -1.0).float()
    to_play = torch.where(feats[:, 5, 0, 0] == 1.0, 1, 2).to(torch.int8)
    flags = torch.zeros(1, dtype=torch.int32, device=device)
    args_ = (native.ptr(feats), native.ptr(masks), native.ptr(policy), native.ptr(value), native.ptr(to_play), n,
             native.ptr(flags), stream)
    ms = timed(lambda: native.call("gk_replay_validate", *args_), args.steps, args.warmup, flush)
    assert int(flags.item()) == 0, "generated rows must be valid"
    row_bytes = 3240 + 82 + 328 + 4 + 1
    gbs = n * row_bytes / (ms / 1e3) / 1e9
    cpu = None
    try:
        from oracle.oracle import replay_violation
        m = min(n, 1 << 16)
        host = [t[:m].cpu().numpy() for t in (feats, masks, policy, value, to_play)]
        start = time.perf_counter()
        reps = 0
        while True:
            assert replay_violation(*host) is None
            reps += 1
            if time.perf_counter() - start > 10.0:
                break
        elapsed = time.perf_counter() - start
        cpu = {"value": reps * m / elapsed, "unit": "rows/s", "cores": 1, "kind": "port",
               "sample": f"{reps} passes over {m} rows (numpy restatement of replay.py:35-74), {elapsed:.1f} s"}
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        cpu = {"value": None, "unavailable": str(exc)}
    return {"workload": f"replay row checks, {n} generated positions with masked-uniform policies",
          "metric": "rows/s", "value": n / (ms / 1e3), "unit": "rows/s", "ms": ms, "dtype": "f32",
          "roofline": {"bound": "hbm", "kernel": "replay_validate_kernel", "achieved": gbs, "peak": peaks[1],
                       "unit": "GB/s", "frac": gbs / peaks[1], "bytes_per_row": row_bytes},
          "cpu_baseline": cpu}


def bench_batched(args, peaks):
    """The evaluation searcher (kingdom::BatchedPUCT, mcts/src/BatchedPUCT.cpp)
    for `--searchers` games at once: `--sims` simulations in leaf batches of
    `--leaf`, from generated positions, new trees every search. Two evaluators:
    the injected one (the whole search is one launch) and the native 64ch x 6
    block network (one network batch per wave over every game). CPU baseline:
    the reference's own BatchedPUCT (oracle/_ref) with the injected evaluator
    on a bounded sample, one thread."""
    import time

    from kingdom_ai import HashEvaluator
    from kingdom_ai.batched_puct import GpuBatchedPUCT, PUCTOptions
    from kingdom_ai.model import random_network

    device = torch.device("cuda", 0)
    flush = Flusher(device)
    T, S, L = args.searchers, args.sims_batched, args.leaf
    bits = positions(T, 4343, device)
    search = GpuBatchedPUCT(T, PUCTOptions(simulations=S), L, reuse_tree=False)
    hold = {}

    def run(evaluator):
        hold["r"] = search.search(bits, evaluator)

    ms_hash = timed(lambda: run(HashEvaluator()), args.steps, args.warmup, flush)
    r = hold["r"]
    assert int(r.simulations.sum().item()) == T * S
    nodes = float(r.nodes.float().mean().item())
    net = random_network(64, 6, 1)
    ms_net = timed(lambda: run(net), max(1, args.steps // 2), 1, flush)
    r = hold["r"]
    assert int(r.simulations.sum().item()) == T * S
    batches = float(search.stats["inference_batches"].float().mean().item())
    cpu = None
    try:
        from oracle.oracle import Reference, RefState
        ref = Reference()
        searcher = ref.batched(S, 1.5, L, False, "hash")
        start, done = time.perf_counter(), 0
        while time.perf_counter() - start < 10.0:
            searcher.search(RefState.generated(ref, 4343, done))
            done += 1
        elapsed = time.perf_counter() - start
        cpu = {"value": done * S / elapsed, "unit": "simulations/s", "cores": 1, "kind": "reference",
               "sample": f"{done} searches of {S} simulations, leaf batch {L}, injected evaluator, "
                         f"reference kingdom::BatchedPUCT, {elapsed:.1f} s"}
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        cpu = {"value": None, "unavailable": str(exc)}
    return {"workload": f"batched evaluation search: {T} games x {S} simulations, leaf batch {L}, c_puct 1.5, "
                      "generated positions, new trees every search",
          "metric": "simulations/s", "unit": "simulations/s",
          "value": T * S / (ms_hash / 1e3), "ms_per_search": ms_hash, "evaluator": "injected (one launch)",
          "nodes_mean": nodes,
          "network": {"value": T * S / (ms_net / 1e3), "ms_per_search": ms_net,
                      "evaluator": "native 64ch x 6-block bf16 network, one batch per wave",
                      "waves_per_search": batches},
          "cpu_baseline": cpu}


def bench_selfplay_reference(args, peaks):
    """Self-play as the reference's Trainer configures it (loop.py:36-57:
    128 simulations per move, the 32 x 2 GroupNorm PolicyValueNet,
    model.py:30-84), on `--lanes` games of one GPU at once: the device engine
    runs one ply of every game per step. Reported with the same counters as
    the headline line; no CPU baseline is run for this line."""
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.model import random_groupnorm_network
    from kingdom_ai.selfplay import SelfPlayEngine

    device = torch.device("cuda", 0)
    opts = GpuPUCTOptions(simulations=128, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=7)
    engine = SelfPlayEngine(random_groupnorm_network(32, 2, 1234), args.lanes, opts, temperature=1.0,
                            temperature_moves=10, final_temperature=0.0, replay_capacity=1 << 20, device=device)
    for _ in range(args.warmup):
        engine.step(1)
    torch.cuda.synchronize(device)
    engine.check()
    before = engine.stats()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        engine.step(1)
    stop.record()
    stop.synchronize()
    engine.check()
    after = engine.stats()
    ms = start.elapsed_time(stop)
    moves = after["moves"] - before["moves"]
    return {"workload": f"self-play, the reference's 32ch x 2-block GroupNorm network, {args.lanes} games, "
                      "128 sims/move, c_puct 1.5, Dirichlet 0.3/0.25",
          "metric": "simulations/s", "unit": "simulations/s", "value": moves * 128 / (ms / 1e3),
          "moves_per_s": moves / (ms / 1e3), "ms_per_step": ms / args.steps, "steps": args.steps,
          "warmup": args.warmup, "games_finished": after["games"] - before["games"]}


def bench_evaluation(args, peaks):
    """A whole evaluation match on one GPU (python/kingdom_ai/evaluation.py:
    235-360 with its defaults: 128 simulations, c_puct 1.5, leaf batch 8, six
    sampled opening moves): `--games` games between two different 6 x 64
    networks, every game stepped at once. Timed with CUDA events around the
    match, after one warm-up match of 16 games; no CPU baseline is run."""
    import time

    from kingdom_ai import evaluate_models_gpu
    from kingdom_ai.model import random_network

    candidate, reference = random_network(64, 6, 31), random_network(64, 6, 32)
    evaluate_models_gpu(candidate, reference, games=16, simulations=128)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall = time.perf_counter()
    start.record()
    result = evaluate_models_gpu(candidate, reference, games=args.games, simulations=128, seed=5)
    stop.record()
    stop.synchronize()
    wall = time.perf_counter() - wall
    seconds = start.elapsed_time(stop) / 1e3
    return {"workload": f"evaluation match: {args.games} games between two 64ch x 6-block networks, 128 sims/move, "
                      "leaf batch 8, 6 sampled opening moves, subtree reuse",
          "metric": "games/s", "unit": "games/s", "value": args.games / seconds,
          "moves_per_s": result.total_plies / seconds, "simulations_per_s": result.total_plies * 128 / seconds,
          "seconds": seconds, "wall_seconds": wall, "total_plies": result.total_plies,
          "candidate_win_rate": result.win_rate, "endings": result.endings}


def bench_collect(args, peaks):
    """The Trainer's self-play hook end to end (python/kingdom_ai/loop.py:
    524-541 calling collect_gpu_puct_games): `--games` complete games with
    `--lanes` in flight, the 6 x 64 network, 400 simulations, Dirichlet 0.3 /
    0.25, T = 1 for 10 plies then the best action. Wall clock around the whole
    call, which returns GameData built on the host; after one warm-up call."""
    import time

    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.model import random_network
    from kingdom_ai.training import collect_gpu_puct_games

    model = random_network(64, 6, 1234)
    opts = GpuPUCTOptions(simulations=400, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=7)
    kw = dict(options=opts, temperature=1.0, temperature_moves=10, final_temperature=0.0, seed=11)
    collect_gpu_puct_games(model, 8, batch_size=8, **kw)
    torch.cuda.synchronize()
    start = time.perf_counter()
    games = collect_gpu_puct_games(model, args.games, batch_size=args.lanes, **kw)
    seconds = time.perf_counter() - start
    moves = sum(len(g.samples) for g in games)
    return {"workload": f"collect_gpu_puct_games: {args.games} games, {args.lanes} in flight, 64ch x 6-block bf16 net, "
                        "400 sims/move, Dirichlet 0.3/0.25, T=1 for 10 plies then best",
            "metric": "simulations/s", "unit": "simulations/s", "value": moves * 400 / seconds,
            "moves_per_s": moves / seconds, "games_per_s": len(games) / seconds, "seconds": seconds,
            "moves": moves, "timing": "wall clock around the call, GameData returned on the host"}
