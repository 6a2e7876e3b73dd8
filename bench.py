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


def cpu_baseline_sample(seconds: float = 15.0):
    """Reference C++ PUCT (compiled from its sources) + fp32 CPU network, batch 1.

    Mirrors the reference's CPU self-play (collect_puct_game: kingdom::PUCT with
    a NeuralAgent-style single-position evaluator) on the same network and
    search settings; runs searches from the opening until `seconds` elapse.
    """
    import ctypes

    import numpy as np
    import torch

    from oracle.oracle import Reference, RefState

    from kingdom_ai.model import calibrate_batchnorm, random_network
    from oracle.oracle import Oracle

    ref = Reference()
    # Same network as the GPU arm: same seed, batch norms calibrated on the
    # same generated positions (here produced by the CPU oracle).
    oracle = Oracle()
    features, _ = oracle.encode(oracle.gen_positions(1234, 4096))
    model = calibrate_batchnorm(random_network(CHANNELS, BLOCKS, 1234), torch.from_numpy(features)).float().eval()
    ref.lib.gkr_puct_search_cb.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_double,
                                           ctypes.c_double, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p,
                                           np.ctypeslib.ndpointer(np.int32), np.ctypeslib.ndpointer(np.int32)]
    ref.lib.gkr_puct_search_cb.restype = ctypes.c_int
    threads = torch.get_num_threads()
    EVAL = ctypes.CFUNCTYPE(None, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint8),
                            ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), ctypes.c_void_p)

    def evaluate(features, mask, policy, value, ctx):
        f = torch.from_numpy(np.ctypeslib.as_array(features, shape=(810,)).copy()).view(1, 10, 9, 9)
        m = torch.from_numpy(np.ctypeslib.as_array(mask, shape=(82,)).astype(bool))
        with torch.inference_mode():
            logits, v = model(f)
            p = torch.softmax(logits[0].masked_fill(~m, -torch.inf), 0).masked_fill(~m, 0.0)
        out = np.ctypeslib.as_array(policy, shape=(82,))
        out[:] = p.double().numpy()
        value[0] = float(v[0])

    callback = EVAL(evaluate)
    state = RefState.initial(ref, 40)
    visits = np.zeros(82, np.int32)
    stats = np.zeros(4, np.int32)
    sims = moves = 0
    start = time.perf_counter()
    while time.perf_counter() - start < seconds:
        status = ref.lib.gkr_puct_search_cb(state.h, SIMULATIONS, 1.5, 0.3, 0.25, 42 + moves,
                                            ctypes.cast(callback, ctypes.c_void_p), None, visits, stats)
        if status != 0:
            raise RuntimeError("reference PUCT failed")
        sims += int(stats[1])
        moves += 1
        if not state.play(int(stats[0])) or state.record()[166] != 0:
            state = RefState.initial(ref, 40)
    elapsed = time.perf_counter() - start
    return {"value": sims / elapsed, "unit": "simulations/s", "cores": threads, "kind": "reference",
            "moves_per_s": moves / elapsed,
            "sample": f"{moves} moves x {SIMULATIONS} simulations from the opening (reference kingdom::PUCT "
                      f"compiled from source, fp32 PyTorch CPU network at batch 1, {threads} threads), "
                      f"{elapsed:.1f} s"}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        base = cpu_baseline_sample(max(5.0, min(60.0, 4.0 * args.steps)))
    except FileNotFoundError as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"reference engine not built: {exc}"}))
        return
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "simulations/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * LANES * SIMULATIONS / base["value"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "moves_per_s": base["moves_per_s"],
        "config": {"workload": f"self-play, {CHANNELS}ch x {BLOCKS} blocks net, {SIMULATIONS} sims/move, "
                               "c_puct 1.5, Dirichlet 0.3/0.25", "lanes": 1},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "simulations/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def e2e_arm(model, steps: int, warmup: int, device):
    """The same self-play ply through the public API with host buffers.

    Every step copies the 4096 current wire records from pinned host memory,
    runs GpuPUCT.search (native network, 400 simulations), plays the chosen
    actions with GpuStateBatch.play and reads the actions, visit policies and
    new records back to the host; finished games restart on the host.
    """
    import torch

    import kingdom_ai
    from kingdom_ai.gpu_rules import GPU_REASON

    opts = kingdom_ai.GpuPUCTOptions(simulations=SIMULATIONS, c_puct=1.5, dirichlet_alpha=0.3,
                                     dirichlet_epsilon=0.25, seed=7)
    searcher = kingdom_ai.GpuPUCT(model, opts, device=device)
    initial = kingdom_ai.GpuStateBatch.initial(1, device=device).states.cpu()
    host = initial.repeat(LANES, 1).pin_memory()
    actions_h = torch.empty(LANES, dtype=torch.int64).pin_memory()
    policy_h = torch.empty((LANES, 82), dtype=torch.float32).pin_memory()
    h2d = host.numel() * 4
    d2h = actions_h.numel() * 8 + policy_h.numel() * 4 + host.numel() * 4

    def step():
        states = host.to(device, non_blocking=True)
        batch = kingdom_ai.GpuStateBatch(states)
        result = searcher.search(batch)
        batch.play(result.actions)
        actions_h.copy_(result.actions, non_blocking=True)
        policy_h.copy_(result.policy, non_blocking=True)
        host.copy_(batch.states, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        done = host[:, GPU_REASON] != 0
        if bool(done.any()):
            host[done] = initial

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    start = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize(device)
    elapsed = time.perf_counter() - start
    return {"value": steps * LANES * SIMULATIONS / elapsed, "unit": "simulations/s",
            "moves_per_s": steps * LANES / elapsed, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "GpuStateBatch + GpuPUCT.search + GpuStateBatch.play with pinned host records",
            "_moves": steps * LANES, "_elapsed": elapsed}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--e2e-steps", type=int, default=3)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--workload", choices=["selfplay", "network", "rules", "encode", "puct", "replay", "batched",
                                                   "selfplay_reference", "evaluation"],
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
    parser.add_argument("--lanes", type=int, default=4096, help="selfplay_reference workload: games at once")
    parser.add_argument("--games", type=int, default=512, help="evaluation workload: games in the match")
    args = parser.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.workload != "selfplay":
        import bench_components
        getattr(bench_components, f"bench_{args.workload}")(args, peaks())
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
            gather.run(int(engine.counters[2].item()))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    engine.check()
    before = engine.stats()
    timer = engine.enable_timer(args.steps)
    start_ev, stop_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        start_ev.record()
        for _ in range(args.steps):
            step()
        stop_ev.record()
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    elapsed_ms = start_ev.elapsed_time(stop_ev)
    engine.check()
    after = engine.stats()
    tower_ms, tower_launches = timer.read()
    engine.timer = None
    local_counts = torch.tensor([after[k] - before[k] for k in ("moves", "evaluations", "games", "rows")],
                                dtype=torch.float64, device=device)
    ms = torch.tensor([elapsed_ms, tower_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(local_counts, op=dist.ReduceOp.SUM)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    moves, evals, games, rows = local_counts.tolist()
    elapsed_s = ms[0].item() / 1000.0
    sims = moves * SIMULATIONS
    my_evals = after["evaluations"] - before["evaluations"]
    tower_s = tower_ms / 1000.0
    tflops = my_evals * TOWER_FLOPS_PER_EVAL / tower_s / 1e12 if tower_s > 0 else None
    peak_tf, hbm, peak_kind, _ = peaks()

    e2e = None
    if args.e2e_steps > 0:
        e2e = e2e_arm(model, args.e2e_steps, 1, device)
        e2e_moves, e2e_elapsed = float(e2e.pop("_moves")), e2e.pop("_elapsed")
        if world > 1:
            # Whole job: every rank's moves over the slowest rank's time.
            t = torch.tensor([e2e_moves], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            e2e_moves = t.item()
            t = torch.tensor([e2e_elapsed], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_elapsed = t.item()
        e2e["value"] = e2e_moves * SIMULATIONS / e2e_elapsed
        e2e["moves_per_s"] = e2e_moves / e2e_elapsed
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_sample(15.0)
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            cpu = {"value": None, "unavailable": str(exc)}
    clock = clocks.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": sims / elapsed_s, "unit": "simulations/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms[0].item() / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (self-play from the opening; random-init network)",
            "moves_per_s": moves / elapsed_s, "games_finished": games, "replay_rows": rows,
            "network_evaluations_per_s": evals / elapsed_s,
            "config": {"workload": f"batched self-play, {LANES} games/GPU, {CHANNELS}ch x {BLOCKS}-block bf16 net, "
                                   f"{SIMULATIONS} PUCT sims/move, c_puct 1.5, Dirichlet 0.3/0.25, T=1 for 10 "
                                   "plies then best, 1M-row replay FIFO",
                       "lanes_per_gpu": LANES, "simulations": SIMULATIONS, "parallelism": f"games sharded x{world}",
                       "l2": "working set (search trees 3.2 GB/GPU) far larger than L2"},
            "roofline": {"bound": "tensor", "kernel": "net_tower_cols_kernel",
                         "achieved": tflops, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": (tflops / peak_tf) if tflops else None, "traffic": TOWER_DRAM_BYTES_PER_LAUNCH,
                         "peak_kind": f"{peak_kind} bf16 sustained",
                         "flops_per_eval": TOWER_FLOPS_PER_EVAL, "launches": tower_launches,
                         "avg_launch_ms": tower_ms / max(tower_launches, 1)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(args.steps * LAUNCHES_PER_PLY),
            "clocks": clock,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
