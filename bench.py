"""Batched self-play benchmark: PUCT simulations/s and self-play moves/s per B200.

Workload (per GPU): 4096 concurrent games from the default start, a 6-block x
64-channel policy/value net in bf16 (Kaiming-normal weights from the seed,
batch norms calibrated on generated positions, folded), 400 PUCT simulations
per move, c_puct 1.5, root Dirichlet noise alpha 0.3 / epsilon 0.25,
temperature 1 for the first 10 plies of each game then the search's best
move; finished games write (obs, visit policy, outcome) rows to a 1M-row FIFO
and restart. One step = one ply in every game (4096 moves, 4096 x 400
simulations). Inputs are synthetic (no datasets exist for this game).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU over NCCL; games are sharded by
game id (no data-path collective); new replay rows are gathered to rank 0's
FIFO every step and counters are all-reduced. Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "alpha-yoo-for-great-kingdom_b200"))

LANES = 4096
SIMULATIONS = 400
CHANNELS, BLOCKS = 64, 6
# Algorithmic FLOPs of one leaf evaluation in the tower kernel (81 cells, no
# padding): stem 3x3 10->C, 2R convs 3x3 C->C, the 1x1 head convs C->3.
TOWER_FLOPS_PER_EVAL = (2 * 81 * 9 * 10 * CHANNELS + 2 * BLOCKS * 2 * 81 * 9 * CHANNELS * CHANNELS
                        + 2 * 81 * CHANNELS * 3)  # 72.63 MFLOP
# DRAM bytes of one tower launch (dram__bytes_read.sum + dram__bytes_write.sum)
# from an ncu capture of net_tower_cols_kernel on 4096 positions: the bf16
# weights streamed once per image group plus the packed input states;
# activations never leave shared memory and the head features stay in L2.
TOWER_DRAM_BYTES_PER_LAUNCH = 1_257_216
# Kernel launches per ply: begin, noise, finish, advance; (compact, tower,
# heads, expand/backup) per evaluation; select per simulation.
LAUNCHES_PER_PLY = 4 + 4 * (SIMULATIONS + 1) + SIMULATIONS
METRIC = "PUCT simulations/sec and self-play moves/sec at 1/2/4/8 B200"


def make_network(seed: int):
    import torch

    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import calibrate_batchnorm, random_network

    model = random_network(CHANNELS, BLOCKS, seed).cuda()
    bits = torch.empty((4096, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", seed, 0, 4096, native.ptr(bits), native.stream_of(bits.device))
    features, _ = encode_packed(bits)
    calibrate_batchnorm(model, features)
    return model.cpu().eval()


class ClockSampler:
    """nvidia-smi clock/throttle samples (200 ms) during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        self.file.seek(0)
        rows = [line.strip().split(", ") for line in self.file if line.strip()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "", 1).isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def peaks():
    """(bf16 sustained TFLOP/s, HBM GB/s, source, bf16 burst TFLOP/s).

    The sustained GEMM figure is the denominator for the tower timed inside a
    seconds-long self-play step; the burst figure is for a kernel timed alone.
    """
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return (data.get("bf16_tflops_sustained", 1378.6), data.get("hbm_gbs", 6543.4), "measured",
                data.get("bf16_tflops", 1619.6))
    return 1400.0, 6650.0, "fallback", 1590.0


REF_INSTALL = ROOT / "baseline" / "_ref"  # the reference package, installed offline with pip


def _reference_imports():
    """Put the installed reference first on sys.path (its package is also
    named kingdom_ai, so this runs only in processes that never import ours)."""
    if not (REF_INSTALL / "kingdom_ai").exists():
        raise FileNotFoundError("the reference is not installed under baseline/_ref")
    sys.path.insert(0, str(REF_INSTALL))


def reference_cpu_selfplay(steps: int, warmup: int):
    """The reference's own CPU self-play path on every host core.

    It is the pattern of examples/gpu_puct_benchmark.py:57-77 and of the
    "CPU PUCT + CPU batch inference" row of docs/performance.md:292, run through
    the reference's public API: one kingdom::PUCT (my_board_engine.PUCT,
    400 simulations, c_puct 1.5, Dirichlet 0.3 / 0.25) and one game per worker
    thread, `cores` workers; leaves from all workers are batched into one
    fp32 CPU forward of the reference's PolicyValueNet(64, 6) by its
    BatchedEvaluator (1 ms batch deadline); moves are sampled from the visits
    at T = 1 for 10 plies, then the best move (sample_visits). torch runs
    cores / 2 intra-op threads, set explicitly so torchrun's
    OMP_NUM_THREADS=1 cannot change it (the fastest split measured on the
    B200 host). One step = one move in every worker's game.
    """
    from concurrent.futures import ThreadPoolExecutor

    _reference_imports()
    import torch
    import my_board_engine as engine
    from kingdom_ai import BatchedEvaluator, PolicyValueNet
    from kingdom_ai.puct import sample_visits

    cores = len(os.sched_getaffinity(0))
    workers, threads = cores, max(1, cores // 2)
    torch.set_num_threads(threads)
    torch.manual_seed(1234)
    model = PolicyValueNet(CHANNELS, BLOCKS).eval()
    states = [engine.State() for _ in range(workers)]
    plies = [0] * workers
    generators = [torch.Generator().manual_seed(100 + i) for i in range(workers)]
    searchers = [engine.PUCT(engine.PUCTOptions(simulations=SIMULATIONS, c_puct=1.5, seed=1000 + i,
                                                dirichlet_alpha=0.3, dirichlet_epsilon=0.25))
                 for i in range(workers)]
    with BatchedEvaluator(model, device="cpu", max_batch_size=workers, max_wait_ms=1.0) as evaluator, \
            ThreadPoolExecutor(workers) as pool:
        def move(i):
            result = searchers[i].search(states[i], evaluator)
            choice = sample_visits(result, 1.0 if plies[i] < 10 else 0.0, generators[i])
            if not states[i].play(choice).accepted():
                raise RuntimeError("the reference played an illegal move")
            plies[i] += 1
            if states[i].result.finished():
                states[i], plies[i] = engine.State(), 0
            return result.simulations

        for _ in range(warmup):
            sum(pool.map(move, range(workers)))
        sims, seconds = 0, []
        for _ in range(steps):
            start = time.perf_counter()
            sims += sum(pool.map(move, range(workers)))
            seconds.append(time.perf_counter() - start)
    total = sum(seconds)
    return {"value": sims / total, "unit": "simulations/s", "moves_per_s": steps * workers / total,
            "ms_per_step": 1000.0 * total / steps, "cores": cores, "kind": "reference",
            "sample": f"{steps} steps x {workers} concurrent games x {SIMULATIONS} simulations after {warmup} "
                      f"warm-up steps: the reference's my_board_engine.PUCT per worker thread + "
                      f"kingdom_ai.BatchedEvaluator (PolicyValueNet({CHANNELS}, {BLOCKS}) fp32, batch <= "
                      f"{workers}, {threads} torch threads), {total:.1f} s"}


def reference_nvrtc_selfplay(plies: int, warmup: int, lanes: int = LANES):
    """The reference's own GPU path (NVRTC kernels) on this B200.

    The per-ply loop of _collect_chunk (python/kingdom_ai/gpu_training.py:
    59-87) through its public classes: GpuStateBatch.encode, GpuPUCT.search
    (400 simulations, c_puct 1.5, Dirichlet 0.3 / 0.25) with the reference's
    PolicyValueNet(64, 6) in fp32 as leaf evaluator, visit sampling at T = 1
    for 10 plies then the best move, GpuStateBatch.play; `lanes` games from
    the opening. The stock collect_gpu_puct_games plays every chunk to the
    end of its longest game (about 100 plies of 3.4 s at 4096 lanes), so the
    loop is timed over a bounded number of plies after `warmup` plies, with
    CUDA synchronisation before each clock read (gpu_puct_benchmark.py:87-90).
    Compilation and model transfer happen in the warm-up.
    """
    _reference_imports()
    import torch
    from kingdom_ai import PolicyValueNet
    from kingdom_ai.gpu_puct import GpuPUCT, GpuPUCTOptions
    from kingdom_ai.gpu_rules import GPU_REASON, GpuStateBatch
    from kingdom_ai.gpu_runtime import nvrtc_version
    from kingdom_ai.gpu_training import _visit_sampling_weights

    torch.manual_seed(1234)
    searcher = GpuPUCT(PolicyValueNet(CHANNELS, BLOCKS), GpuPUCTOptions(
        simulations=SIMULATIONS, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=7))
    state = GpuStateBatch.initial(lanes)
    generator = torch.Generator(device="cuda").manual_seed(11)
    sims = torch.zeros((), dtype=torch.int64, device="cuda")

    def ply(index):
        alive = state.states[:, GPU_REASON] == 0
        state.encode()
        result = searcher.search(state)
        if index < 10:
            weights = _visit_sampling_weights(result.visits, 1.0)
            weights[:, -1] += (~alive).to(weights.dtype)
            actions = torch.where(alive, torch.multinomial(weights, 1, generator=generator).flatten(),
                                  result.actions)
        else:
            actions = result.actions
        state.play(actions)
        sims.add_(result.simulations.sum())

    for i in range(warmup):
        ply(i)
    torch.cuda.synchronize()
    sims.zero_()
    start = time.perf_counter()
    for i in range(warmup, warmup + plies):
        ply(i)
    torch.cuda.synchronize()
    seconds = time.perf_counter() - start
    return {"value": int(sims.item()) / seconds, "unit": "simulations/s", "moves_per_s": lanes * plies / seconds,
            "ms_per_ply": 1000.0 * seconds / plies, "lanes": lanes, "plies": plies, "warmup_plies": warmup,
            "nvrtc": "%d.%d" % nvrtc_version(),
            "path": "reference GpuStateBatch / GpuPUCT (NVRTC kernels) + PolicyValueNet(64, 6) fp32, "
                    "the per-ply loop of collect_gpu_puct_games"}


def _subprocess_json(argv, timeout):
    """Run bench.py in a fresh interpreter and return its last JSON line."""
    env = dict(os.environ)
    for key in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
                "TORCHELASTIC_RUN_ID", "GROUP_RANK", "ROLE_RANK"):
        env.pop(key, None)
    try:
        out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *argv], capture_output=True, text=True,
                             timeout=timeout, env=env)
    except subprocess.TimeoutExpired:
        return {"value": None, "unavailable": f"timed out after {timeout} s"}
    lines = [line for line in out.stdout.splitlines() if line.startswith("{")]
    if out.returncode != 0 or not lines:
        return {"value": None, "unavailable": (out.stderr.strip().splitlines() or ["no output"])[-1][:300]}
    return json.loads(lines[-1])


def reference_arm(args):
    """`--impl reference`: the reference's CPU self-play on the host cores,
    K timed steps after W warm-up steps, rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    try:
        base = reference_cpu_selfplay(args.steps, args.warmup)
    except Exception as exc:  # noqa: BLE001 - the line says why
        print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
        return
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "simulations/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "moves_per_s": base["moves_per_s"],
        "config": {"workload": f"self-play, {CHANNELS}ch x {BLOCKS}-block net (the reference's PolicyValueNet), "
                               f"{SIMULATIONS} sims/move, c_puct 1.5, Dirichlet 0.3/0.25, T=1 for 10 plies "
                               "then best", "concurrent_games": base["cores"],
                   "path": "CPU: my_board_engine.PUCT per worker thread + kingdom_ai.BatchedEvaluator"},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "simulations/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def nvrtc_arm(args):
    """`--impl nvrtc`: the reference's NVRTC GPU path on cuda:0 (one JSON line)."""
    try:
        line = reference_nvrtc_selfplay(args.steps, args.warmup)
    except Exception as exc:  # noqa: BLE001 - the line says why
        line = {"value": None, "unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    line["impl"] = "nvrtc"
    print(json.dumps(line), flush=True)


class HostPly:
    """One self-play ply driven from host memory through the engine's public
    API: the lanes' positions are copied in from pinned host records, the
    ply runs (search, temperature sampling, history, replay flush), and the
    new positions, the moves played, the visit-share targets and the replay
    rows of games that finished cross back to pinned host buffers."""

    def __init__(self, engine):
        import torch

        self.engine = engine
        n = engine.lanes
        self.records = engine.records().cpu().pin_memory()
        self.records_dev = torch.empty_like(self.records, device=engine.device)
        self.actions = torch.empty(n, dtype=torch.int32).pin_memory()
        self.policy = torch.empty((n, 82), dtype=torch.float32).pin_memory()
        self.counters = torch.empty(engine.counters.numel(), dtype=torch.int64).pin_memory()
        cap = 4 * n
        ring = engine.replay
        self.rows = [torch.empty((cap,) + tuple(t.shape[1:]), dtype=t.dtype).pin_memory()
                     for t in (ring.features, ring.masks, ring.policy, ring.value, ring.to_play)]
        self.row_bytes = sum(t[0].numel() * t.element_size() for t in self.rows)
        self.rows_seen = int(engine.stats()["rows"])
        self.rows_out = 0
        self.h2d = self.records.numel() * 4
        self.d2h_fixed = (self.records.numel() * 4 + self.actions.numel() * 4 + self.policy.numel() * 4
                          + self.counters.numel() * 8)

    def __call__(self):
        import torch

        e = self.engine
        e.load_records(self.records)
        e.step()
        e.records(self.records_dev)
        self.records.copy_(self.records_dev, non_blocking=True)
        self.actions.copy_(e.last_action, non_blocking=True)
        self.policy.copy_(e.last_policy, non_blocking=True)
        self.counters.copy_(e.counters, non_blocking=True)
        torch.cuda.current_stream(e.device).synchronize()
        written = int(self.counters[2])
        ring = e.replay
        while self.rows_seen < written:
            count = min(written - self.rows_seen, self.rows[0].shape[0], ring.capacity - self.rows_seen % ring.capacity)
            lo = self.rows_seen % ring.capacity
            for host, dev in zip(self.rows, (ring.features, ring.masks, ring.policy, ring.value, ring.to_play)):
                host[:count].copy_(dev[lo:lo + count], non_blocking=True)
            torch.cuda.current_stream(e.device).synchronize()
            self.rows_seen += count
            self.rows_out += count


def component_lines(args):
    """Compact C1-C4 measurements for the headline line (rank 0, one GPU)."""
    import bench_components

    small = argparse.Namespace(**vars(args))
    small.steps, small.warmup = 5, 2
    lines = {}
    for name in ("rules", "encode", "puct", "network"):
        try:
            lines[name] = getattr(bench_components, f"bench_{name}")(small, peaks())
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            lines[name] = {"value": None, "unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return lines


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference", "nvrtc"], default="ours",
                        help="reference: the reference's CPU self-play; nvrtc: the reference's NVRTC GPU path")
    parser.add_argument("--preroll-plies", type=int, default=150,
                        help="plies played at --preroll-sims before warm-up, so games are spread over all phases")
    parser.add_argument("--preroll-sims", type=int, default=16)
    parser.add_argument("--no-extras", action="store_true",
                        help="skip the component lines, the CPU baseline and the NVRTC figure")
    parser.add_argument("--workload", choices=["selfplay", "network", "rules", "encode", "puct", "replay", "batched",
                                                   "selfplay_reference", "evaluation", "collect"],
                        default="selfplay",
                        help="selfplay is the headline; the others time one kernel family each")
    parser.add_argument("--net", default="128x10", help="network workload: CHANNELSxBLOCKS")
    parser.add_argument("--norm", choices=["batch", "group"], default="batch",
                        help="network workload: batch norm folded, or the reference's GroupNorm network")
    parser.add_argument("--batch", type=int, default=8192, help="network workload batch")
    parser.add_argument("--states", type=int, default=1 << 22, help="rules workload: states per play launch")
    parser.add_argument("--positions", type=int, default=65536, help="encode workload: positions")
    parser.add_argument("--trees", type=int, default=1024, help="puct workload: trees")
    parser.add_argument("--sims", type=int, default=800, help="puct workload: simulations per tree")
    parser.add_argument("--rows", type=int, default=1 << 20, help="replay workload: rows validated per launch")
    parser.add_argument("--searchers", type=int, default=4096, help="batched workload: games searched together")
    parser.add_argument("--sims-batched", type=int, default=128, help="batched workload: simulations per search")
    parser.add_argument("--leaf", type=int, default=8, help="batched workload: leaf batch per tree")
    parser.add_argument("--lanes", type=int, default=4096,
                        help="selfplay_reference and collect workloads: games at once")
    parser.add_argument("--games", type=int, default=512, help="evaluation and collect workloads: games")
    args = parser.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.impl == "nvrtc":
        nvrtc_arm(args)
        return
    if args.workload != "selfplay":
        import bench_components
        bench_components.emit(getattr(bench_components, f"bench_{args.workload}")(args, peaks()))
        return

    import torch
    import torch.distributed as dist

    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.distributed import ReplayGather
    from kingdom_ai.selfplay import ReplayRing, SelfPlayEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))

    model = make_network(1234)
    opts = GpuPUCTOptions(simulations=SIMULATIONS, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=7)
    fifo_capacity = 1 << 20
    engine = SelfPlayEngine(model, LANES, opts, temperature=1.0, temperature_moves=10, final_temperature=0.0,
                            replay_capacity=fifo_capacity if world == 1 else 1 << 18, rank=rank, world_size=world,
                            device=device)
    fifo = engine.replay if world == 1 else (ReplayRing(fifo_capacity, device) if rank == 0 else None)
    gather = ReplayGather(engine.replay, fifo) if world > 1 else None

    def step():
        engine.step(1)
        if gather is not None:
            gather.run(engine.counters)

    # Steady state: a short pre-roll at a few simulations per move lets games
    # end and restart at different plies, so the timed plies see every phase
    # of a game (openings, middle games, endings, restarts) as a long run does.
    engine.set_simulations(max(1, min(args.preroll_sims, SIMULATIONS)))
    for _ in range(args.preroll_plies):
        step()
    engine.set_simulations(SIMULATIONS)
    for _ in range(args.warmup):
        step()
    # Each ply replays one captured CUDA graph of its launches; a second
    # graph's tower launches also record CUDA events (the roofline sample).
    timer = engine.enable_timer(1)
    engine.capture()
    torch.cuda.synchronize(device)
    engine.check()
    before = engine.stats()
    sampled_evals = torch.zeros((), dtype=torch.int64, device=device)
    start_ev, stop_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        start_ev.record()
        for i in range(args.steps):
            # CUDA events bracket every tower launch of the last timed ply: a
            # live sample (the timer keeps the last replay's times). The
            # evaluations of that ply are counted on the device.
            sampled_ply = i == args.steps - 1
            engine.timer = timer if sampled_ply else None
            if sampled_ply:
                evals_before = engine.counters[7].clone()
            step()
            if sampled_ply:
                sampled_evals += engine.counters[7] - evals_before
        stop_ev.record()
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    elapsed_ms = start_ev.elapsed_time(stop_ev)
    engine.check()
    after = engine.stats()
    tower_ms, tower_launches = timer.read()
    engine.timer = None
    clock = clocks.summary()
    local_counts = torch.tensor([after[k] - before[k] for k in ("moves", "evaluations", "games", "rows")],
                                dtype=torch.float64, device=device)
    ms = torch.tensor([elapsed_ms, tower_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(local_counts, op=dist.ReduceOp.SUM)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    moves, evals, games, rows = local_counts.tolist()
    elapsed_s = ms[0].item() / 1000.0
    sims = moves * SIMULATIONS
    tower_s = tower_ms / 1000.0
    tflops = int(sampled_evals.item()) * TOWER_FLOPS_PER_EVAL / tower_s / 1e12 if tower_s > 0 else None
    peak_tf, hbm, peak_kind, _ = peaks()

    # e2e: the same number of plies, continuing the same games, driven from
    # host memory through the engine's public API (HostPly).
    host_ply = HostPly(engine)
    for _ in range(min(args.warmup, 2)):
        host_ply()
        if gather is not None:
            gather.run(engine.counters)
    e2e_before = engine.stats()
    rows_out_before = host_ply.rows_out
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    wall = time.perf_counter()
    for _ in range(args.steps):
        host_ply()
        if gather is not None:
            gather.run(engine.counters)
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - wall
    engine.check()
    e2e_moves = engine.stats()["moves"] - e2e_before["moves"]
    e2e_rows = host_ply.rows_out - rows_out_before
    t = torch.tensor([float(e2e_moves), float(e2e_rows)], dtype=torch.float64, device=device)
    w = torch.tensor([wall], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        dist.all_reduce(w, op=dist.ReduceOp.MAX)
    e2e_moves, e2e_rows = t.tolist()
    wall = w.item()
    e2e = {"value": e2e_moves * SIMULATIONS / wall, "unit": "simulations/s", "moves_per_s": e2e_moves / wall,
           "h2d_bytes_per_step": host_ply.h2d,
           "d2h_bytes_per_step": host_ply.d2h_fixed + int(round(host_ply.row_bytes * e2e_rows / world / args.steps)),
           "steps": args.steps,
           "api": "SelfPlayEngine driven from pinned host records: load_records (H2D) -> step (search, T=1 "
                  "sampling for 10 plies then best, history, replay flush) -> records, last_action, last_policy, "
                  "counters and the new replay rows (D2H), two host synchronisations per ply",
           "replay_rows_per_step": e2e_rows / world / args.steps}

    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        net_error = None
        try:
            import bench_components
            from kingdom_ai.model import NativePolicyValueNet

            net_error = bench_components.network_error(
                model, NativePolicyValueNet(model, device), bench_components.positions(LANES, 4321, device))
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            net_error = {"unavailable": str(exc)}
        extras["network_error"] = net_error
        extras["components"] = component_lines(args)
        extras["nvrtc"] = _subprocess_json(["--impl", "nvrtc", "--steps", "2", "--warmup", "1"], timeout=600)
        cpu = _subprocess_json(["--impl", "reference", "--steps", "3", "--warmup", "1"], timeout=600)
        extras["cpu_baseline"] = cpu.get("cpu_baseline", cpu)
    if rank == 0:
        line = {
            "metric": METRIC, "value": sims / elapsed_s, "unit": "simulations/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms[0].item() / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (continuous self-play at steady state; random-init network)",
            "moves_per_s": moves / elapsed_s, "games_finished": games, "replay_rows": rows,
            "network_evaluations_per_s": evals / elapsed_s,
            "config": {"workload": f"batched self-play, {LANES} games/GPU, {CHANNELS}ch x {BLOCKS}-block bf16 net, "
                                   f"{SIMULATIONS} PUCT sims/move, c_puct 1.5, Dirichlet 0.3/0.25, T=1 for 10 "
                                   "plies then best, 1M-row replay FIFO",
                       "lanes_per_gpu": LANES, "simulations": SIMULATIONS, "parallelism": f"games sharded x{world}",
                       "steady_state": f"{args.preroll_plies} pre-roll plies at {args.preroll_sims} sims/move, "
                                       f"then {args.warmup} warm-up plies at {SIMULATIONS}",
                       "launch": f"each ply replays a captured CUDA graph of its {LAUNCHES_PER_PLY} kernel launches",
                       "l2": "working set (search trees 3.2 GB/GPU) far larger than L2"},
            "roofline": {"bound": "tensor", "kernel": "net_tower_cols_kernel",
                         "achieved": tflops, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": (tflops / peak_tf) if tflops else None, "traffic": TOWER_DRAM_BYTES_PER_LAUNCH,
                         "peak_kind": f"{peak_kind} bf16 sustained",
                         "flops_per_eval": TOWER_FLOPS_PER_EVAL, "launches": tower_launches,
                         "sampled": "every tower launch of the last timed ply",
                         "avg_launch_ms": tower_ms / max(tower_launches, 1)},
            "cpu_baseline": extras.get("cpu_baseline"),
            "nvrtc": extras.get("nvrtc"),
            "e2e": e2e,
            "network_error": extras.get("network_error"),
            "components": extras.get("components"),
            "gpu_launches": int(args.steps * LAUNCHES_PER_PLY),
            "clocks": clock,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
