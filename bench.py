"""Benchmark of the self-play hot path on B200: the BASELINE configs' metrics.

Default run (one JSON line):

* headline: batched legal move generation + FNN feature
  encoding of 262,144 positions per GPU from the seeded random-playout
  generator (all expansions, stop ply U[0, 120]); one step = one pass of
  ``generate_legal_moves_and_fnn_features_batch`` over the batch (moves
  [P,256,6] u8, num_legal [P] i32, features [P,122] f32).  Inputs (898 MB per
  GPU) are larger than L2, so no flush is needed between steps.  Beside the
  K-step region, a second region of >= 2 s of the same steps, and each
  rank's time and clocks;
* ``mcts``: Gumbel-root MCTS, 512 games per GPU, 4,096
  simulations per move, FNN large; one step = one searched move of every
  game through ``FNNMCTSOrchestrator.self_play_batch`` (host states in,
  training examples out); simulations/s, an FP32 roofline, the reference's
  CPU player beside it, and at N > 1 the replay-sample all-gather over NCCL;
* ``hybrid``: PUCT with the FNN-transformer evaluator,
  256 games per GPU, 1,024 simulations per move; simulations/s and a tensor
  roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload all|movegen|mcts|hybrid|fnn]

N > 1 runs one process per GPU under torch.distributed (weak scaling: every
rank owns its own games, no data-path collective); timing is the max over
ranks of CUDA-event time.  ``--impl reference`` times the reference's own
CPU implementation (its hive_gpu/csrc headers compiled on the host,
oracle/_ref) on all host cores for the same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "movegen+encode positions/sec"
UNIT = "positions/s"
POSITIONS = 262144
POSITIONS_DEFAULT = POSITIONS
MAX_PLY = 120
EXPANSIONS = 7
SEED = 20260101
STATE_BYTES = 3424
MOVE_BYTES = 6
MAX_MOVES = 256
FEAT = 122


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": "config2: movegen+FNN-encode, 262144 positions/GPU, all expansions, ply U[0,120]",
        "positions_per_gpu": POSITIONS,
        "global_positions": POSITIONS * n_gpus,
        "expansion_mask": EXPANSIONS,
        "max_ply": MAX_PLY,
        "seed": SEED,
        "parallelism": f"games sharded dp{n_gpus}" if n_gpus > 1 else "single GPU",
        "l2": "inputs (898 MB/GPU) larger than the 126 MB L2; no flush",
    }


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# --------------------------------------------------------------------------
# CPU legs (reference build of the reference headers, or the C oracle)
# --------------------------------------------------------------------------
def _cpu_lib():
    from oracle import oracle as O
    if not O.ref_available() and O.reference_available():
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref",
                        f"HIVE_REFERENCE={O.reference_dir()}"], check=False)
    if O.ref_available():
        return O.ref(), "reference"
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "liboracle.so"], check=True)
    return O.oracle(), "port"


def cpu_rate(states_np, threads: int, target_s: float = 12.0):
    """positions/s of the CPU implementation over a bounded sample: repeated
    passes over the given positions until about target_s of work is done."""
    lib, kind = _cpu_lib()
    lib.legal_moves_features(states_np[:2048], threads)  # warm-up
    done, passes = 0, 0
    t0 = time.perf_counter()
    while True:
        lib.legal_moves_features(states_np, threads)
        done += len(states_np)
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= target_s or passes >= 1000:
            break
    return done / dt, kind, done, dt


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}

        def mhz(s):
            try:
                return float(s.split()[0])
            except Exception:
                return None

        sm = [mhz(r[1]) for r in rows if mhz(r[1]) is not None]
        mx = [mhz(r[2]) for r in rows if mhz(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------
# roofline helpers
# --------------------------------------------------------------------------
def staged_upload_bytes(states):
    """Host->device bytes of hv_stage_host_states for these states: bytes
    2645..3423 of each, and per stack level L the 16-byte words spanning the
    board rows that hold a cell higher than L."""
    import torch
    n = states.shape[0]
    rowmax = states[:, 2645:2645 + 529].reshape(n, 23, 23).amax(2).long()
    rows = torch.arange(23, device=states.device)
    total = n * (STATE_BYTES - 2645)
    for lv in range(5):
        has = rowmax > lv
        r0 = torch.where(has, rows, 23).amin(1)
        r1 = torch.where(has, rows + 1, 0).amax(1)
        w0 = (lv * 529 + r0 * 23) // 16
        w1 = (lv * 529 + r1 * 23 + 15) // 16
        total += int((16 * (w1 - w0) * has.any(1)).sum().item())
    return total


def measured_peak_gbs():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic_per_position():
    """DRAM bytes per position of the movegen kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "movegen_features_config2.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_position:"):
                    return float(line.split(":", 1)[1].split()[0])
    except Exception:
        pass
    return None


# --------------------------------------------------------------------------
# reference arm
# --------------------------------------------------------------------------
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lib, kind = _cpu_lib()
    cores = host_cores()
    # the same generator recipe, run by the CPU implementation itself
    sample_n = 16384
    states = lib.generate_positions(SEED, 0, sample_n, MAX_PLY, EXPANSIONS, cores)
    rates = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        lib.legal_moves_features(states, cores)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            rates.append((sample_n, dt))
    total_n = sum(n for n, _ in rates)
    total_t = sum(t for _, t in rates)
    value = total_n / total_t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / len(rates),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"{sample_n} positions of the workload per step, {cpu_model()}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload in ("all", "mcts"):
        # the reference's CPU player on config 4's kind of roots (base game, ply U[0, 30])
        roots = lib.generate_positions(SEED + 97, 0, 4 * cores, 30, 0, cores)
        roots = roots[roots[:, 3415] == 0]
        rec = mcts_cpu_player_baseline(roots, args.sims)
        line["mcts"] = {"impl": "reference", "metric": "MCTS simulations/sec", "value": rec["value"],
                        "unit": "simulations/s", "cpu_baseline": rec,
                        "e2e": {"value": rec["value"], "unit": "simulations/s", "h2d_bytes_per_step": 0,
                                "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# B200 arm
# --------------------------------------------------------------------------
class Ranks:
    """One process per GPU: the rank's device and the process group (None at N = 1)."""

    def __init__(self, timeout_s: int = 300):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=self.dev)
            self.dist = dist
            # the communicator's setup on its first collective, done here and
            # not in the barrier that opens the first timed region (after a
            # first collective the next step ran late by several ms)
            self.barrier()
            self.gather(0.0)
            torch.cuda.synchronize(self.dev)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier(device_ids=[self.local])

    def gather(self, x: float) -> list[float]:
        """x of every rank, in rank order."""
        import torch
        t = torch.tensor([float(x)], device=self.dev, dtype=torch.float64)
        if self.dist is None:
            return [float(x)]
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [float(o.item()) for o in out]

    def gather_obj(self, obj) -> list:
        if self.dist is None:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.dist is not None:
            self.dist.barrier(device_ids=[self.local])
            self.dist.destroy_process_group()


def timed_region(ranks: Ranks, fn, steps: int, step_times: list | None = None) -> tuple[float, list[float]]:
    """CUDA-event time (ms) of `steps` calls of fn on the current stream,
    bracketed by a barrier and a synchronize on both sides: (max over ranks,
    every rank's time).  step_times: filled with this rank's time of each
    step (an event after every step; the region's time is unchanged)."""
    import torch
    stream = torch.cuda.current_stream(ranks.dev)
    ranks.barrier()
    torch.cuda.synchronize(ranks.dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1 if step_times is not None else 2)]
    ev[0].record(stream)
    for i in range(steps):
        fn()
        if step_times is not None:
            ev[i + 1].record(stream)
    ev[-1].record(stream)
    torch.cuda.synchronize(ranks.dev)
    ranks.barrier()
    if step_times is not None:
        step_times[:] = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    per_rank = ranks.gather(ev[0].elapsed_time(ev[-1]))
    return max(per_rank), per_rank


def bench_movegen(args, ranks: Ranks) -> dict:
    """BASELINE config 2, the headline line."""
    import torch
    dev, rank, world = ranks.dev, ranks.rank, ranks.world

    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    P = POSITIONS
    states = ext.generate_positions(SEED, rank * P, P, MAX_PLY, EXPANSIONS, device=dev)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    box = {}

    def step():
        box["out"] = ext.generate_legal_moves_and_fnn_features_batch(states, P)

    # ---- device-resident throughput: exactly K timed steps ----
    # the clock sampler starts first; the warm-up steps then run right before
    # the timed region, so the GPU does not enter it from an idle spell (a
    # GPU idle for a fraction of a second runs its first steps slower)
    sampler = ClockSampler(ranks.local)
    sampler.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    own_steps: list = []
    ms_max, per_rank_ms = timed_region(ranks, step, args.steps, own_steps)
    value = world * P * args.steps / (ms_max / 1e3)
    rank_steps = ranks.gather_obj(own_steps)
    # ---- the same steps over a region of >= --long-s seconds (every rank the same count) ----
    long_steps = max(args.steps, int(math.ceil(1000.0 * args.long_s / (ms_max / args.steps))))
    long_max, long_per_rank = timed_region(ranks, step, long_steps) if args.long_s > 0 else (None, None)
    clocks = sampler.stop()
    out = box["out"]
    mean_legal = float(out[1].float().mean().item())

    # ---- end to end through the public API with host buffers ----
    host_states = torch.empty((P, STATE_BYTES), dtype=torch.uint8, pin_memory=True)
    host_states.copy_(states)
    h_moves = torch.empty((P, MAX_MOVES, MOVE_BYTES), dtype=torch.uint8, pin_memory=True)
    h_nl = torch.empty((P,), dtype=torch.int32, pin_memory=True)
    h_feat = torch.empty((P, FEAT), dtype=torch.float32, pin_memory=True)
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_step():
        # host states in, host results out; chunked and overlapped over three streams
        ext.generate_legal_moves_and_fnn_features_host(host_states, P, out=(h_moves, h_nl, h_feat),
                                                       chunk=args.e2e_chunk, device=dev)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    e2e_ms, e2e_per_rank = timed_region(ranks, e2e_step, e2e_steps)
    e2e_value = world * P * e2e_steps / (e2e_ms / 1e3)
    h2d = staged_upload_bytes(states)
    n_tall = int((states[:, 2645:2645 + 529].amax(1) >= 3).sum().item())
    # bytes that crossed the link: with the pinned buffers (and enough host
    # threads to clear the row tails) each row's first HOST_MOVE_PREFIX moves
    # (pitched copy) and, for longer lists, the moves past them in 16-byte
    # stores; the rest of each row is cleared on the host.  Else whole rows.
    from hive_neuralnet_b200.hive_gpu import HOST_CLEAR_MIN_THREADS, HOST_MOVE_PREFIX
    split = torch.get_num_threads() >= HOST_CLEAR_MIN_THREADS
    if split:
        nl64 = h_nl.to(torch.int64).clamp(0, MAX_MOVES)
        tail = torch.where(nl64 > HOST_MOVE_PREFIX,
                           (nl64 * MOVE_BYTES + 15) // 16 * 16 - HOST_MOVE_PREFIX * MOVE_BYTES, torch.zeros_like(nl64))
        d2h = P * (HOST_MOVE_PREFIX * MOVE_BYTES + 4 + FEAT * 4) + int(tail.sum())
        moves_path = (f"moves: the first {HOST_MOVE_PREFIX} of each row by a pitched copy, longer lists' rest "
                      f"stored into the mapped rows, the row tails cleared on {torch.get_num_threads()} host "
                      f"threads (hv_download_moves)")
    else:
        d2h = P * (MAX_MOVES * MOVE_BYTES + 4 + FEAT * 4)
        moves_path = f"moves: whole rows ({torch.get_num_threads()} host threads per rank: too few to clear tails)"
    # the host results equal the device-resident step's (same positions)
    host_equal = (torch.equal(h_nl, out[1].cpu()) and torch.equal(h_moves, out[0].cpu())
                  and torch.equal(h_feat.view(torch.int32), out[2].cpu().view(torch.int32)))

    # ---- the host link the e2e leg runs against: plain pinned copies of the
    # step's state bytes, each direction alone, CUDA events on this stream
    dev_buf = torch.empty_like(states)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def link_gbs(copy, nbytes):
        for _ in range(2):
            copy()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(3):
            copy()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return 3 * nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9

    side = torch.cuda.Stream(dev)

    def both_ways():
        # the state upload and the move-list download at once, on two streams
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            h_moves.copy_(out[0], non_blocking=True)
        dev_buf.copy_(host_states, non_blocking=True)
        stream.wait_stream(side)

    h2d_gbs = link_gbs(lambda: dev_buf.copy_(host_states, non_blocking=True), P * STATE_BYTES)
    d2h_gbs = link_gbs(lambda: host_states.copy_(dev_buf, non_blocking=True), P * STATE_BYTES)
    bidir_gbs = link_gbs(both_ways, P * (STATE_BYTES + MAX_MOVES * MOVE_BYTES))
    del dev_buf
    e2e_step_s = e2e_ms / 1e3 / e2e_steps
    # the step moves bytes both ways at once: its bound is the link's combined rate
    link = {"h2d_gbs_measured": h2d_gbs, "d2h_gbs_measured": d2h_gbs, "bidir_gbs_measured": bidir_gbs,
            "h2d_gbs_achieved": h2d / e2e_step_s / 1e9, "d2h_gbs_achieved": d2h / e2e_step_s / 1e9,
            "frac": (h2d + d2h) / e2e_step_s / 1e9 / bidir_gbs}

    # ---- roofline of the dominant kernel: the step's move generator
    # k_root<1,1,0,1,0>, timed alone with CUDA events on the launching stream
    # through hv_generate_legal_moves_linked (the first half of the step's
    # entry: a 16-byte memset of the position counters, then the generator);
    # algorithmic bytes per position = state read + move list (6 bytes per
    # legal move) + num_legal written.  The standalone generator entry
    # (static position stride) is timed beside it.
    peak, peak_kind = measured_peak_gbs()
    lib = ext._lib
    mv_t, nl_t, ft_t = out[0], out[1], out[2]

    # Only the generator half is timed on its own: the feature half
    # (hv_fnn_features_linked) consumes the working data that its own
    # generator half leaves in the feature rows, so it cannot run alone.
    def linked_gen():
        rc = lib.hv_generate_legal_moves_linked(states.data_ptr(), P, mv_t.data_ptr(), nl_t.data_ptr(),
                                                ft_t.data_ptr(), stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"hv_generate_legal_moves_linked: {lib.hv_status_string(rc)}")

    def time_reps(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(reps):
            fn()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        return g0.elapsed_time(g1) / reps / 1e3

    reps = max(5, min(args.steps, 20))
    gen_s = time_reps(linked_gen, reps)
    static_s = time_reps(lambda: ext.generate_legal_moves_batch(states, P), reps)
    alg_bytes = P * (STATE_BYTES + 4 + MOVE_BYTES * mean_legal)
    achieved = alg_bytes / gen_s / 1e9
    tpp = profiled_traffic_per_position()
    step_bytes = P * (STATE_BYTES + 4 + FEAT * 4 + MOVE_BYTES * mean_legal)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind,
                "traffic": (tpp * P) if tpp else None,
                "algorithmic_bytes_per_launch": alg_bytes,
                "kernel": f"k_root<1,1,0,1,0> move generator (the step's first launch, positions claimed "
                          f"from a counter), {gen_s * 1e3:.3f} ms per launch",
                "standalone_generator_ms": static_s * 1e3,
                "step": {"algorithmic_bytes": step_bytes,
                         "achieved_gbs": step_bytes / ((ms_max / args.steps) / 1e3) / 1e9,
                         "launches": ["k_root<1,1,0,1> (legal moves)", "k_root<0,0,1,1,1> (FNN features, positions 1..)",
                                      "k_root<0,0,1,1> (FNN features, position 0)"]}}
    rank_clocks = ranks.gather_obj(clocks)
    cpu_sample = states[:65536].cpu().numpy() if (rank == 0 and world == 1 and not args.no_cpu) else None
    del states, host_states, h_moves, h_nl, h_feat, box, out, mv_t, nl_t, ft_t
    torch.cuda.empty_cache()
    if rank != 0:
        return {}
    cpu = None
    if cpu_sample is not None:
        cores = host_cores()
        rate, kind, n, dt = cpu_rate(cpu_sample, cores)
        cpu = {"value": rate, "unit": UNIT, "cores": cores, "kind": kind,
               "sample": f"first {n} positions of the workload ({dt:.1f} s), {cpu_model()}"}
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": workload_config(world),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "per_rank_ms_per_step": [t / e2e_steps for t in e2e_per_rank],
                "path": f"generate_legal_moves_and_fnn_features_host, pinned host buffers, "
                        f"staged upload (hv_stage_host_states: stack levels over occupied rows; "
                        f"{n_tall} states with a 3-high stack), "
                        f"{args.e2e_chunk}-position chunks over 3 streams; {moves_path}",
                "host_results_equal_device": host_equal,
                "link": link},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "per_rank": {"ms_per_step": [t / args.steps for t in per_rank_ms],
                     "first_step_ms": [st[0] for st in rank_steps],
                     "median_step_ms": [sorted(st)[len(st) // 2] for st in rank_steps],
                     "clocks": [{"sm_mhz": c.get("sm_mhz"), "reasons": c.get("reasons"),
                                 "samples": c.get("samples")} for c in rank_clocks]},
        "long_run": {"steps": long_steps, "ms_per_step": long_max / long_steps,
                     "value": world * P * long_steps / (long_max / 1e3),
                     "per_rank_ms_per_step": [t / long_steps for t in long_per_rank],
                     "timed_s": long_max / 1e3} if long_max is not None else None,
        "gpu_launches": 3 * args.steps,  # per step: generator, features, features of position 0
        "mean_legal_moves": mean_legal,
    }


# --------------------------------------------------------------------------
# BASELINE configs 4 (Gumbel MCTS + FNN) and 5 (PUCT + FNN-transformer)
# --------------------------------------------------------------------------
MCTS_GAMES = 512
MCTS_SIMS = 4096
# FLOPs of the FNN large evaluation (multiply-add = 2): per evaluated position
# encode 2*(122*64 + 64*64) + value head 2*64; per successor row the same
# encode and value head (child Q) + the action tower 2*(128*64) + 2*64
FNN_FLOP_PER_LEAF = 2 * (122 * 64 + 64 * 64) + 2 * 64
FNN_FLOP_PER_ROW = 2 * (122 * 64 + 64 * 64) + 2 * 64 + 2 * (128 * 64) + 2 * 64
SMS = 148
FP32_LANES_PER_SM = 128


def fp32_peak_tflops() -> tuple[float, str]:
    """FP32 FMA peak: 148 SMs x 128 lanes x 2 FLOP x the max SM clock (MEASURED_PEAKS.json's)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f)["sm_max_mhz"])
    except Exception:
        mhz = 1965.0
    return SMS * FP32_LANES_PER_SM * 2 * mhz * 1e6 / 1e12, f"computed: {SMS} SMs x {FP32_LANES_PER_SM} lanes x 2 x {mhz:.0f} MHz"


def bf16_peak_tflops(sustained: bool) -> tuple[float, str]:
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key]), f"measured ({key})"
    except Exception:
        return (1400.0 if sustained else 1590.0), "fallback"


def _mcts_start_states(ext, n, seed, device, no_immediate_end=False):
    """Seeded in-progress base-game positions (ply U[0, 30]) as search roots.
    ``no_immediate_end`` keeps only positions where no legal move ends the game
    (the PUCT driver skips the whole batch's search when any game can win at
    once, fnn_puct_orchestrator.py:203-208)."""
    m = n * 4
    st = ext.generate_positions(seed, 0, m, 30, 0, device=device)
    ok = ext.check_results_batch(st, m) == 0
    if no_immediate_end:
        legal, nl = ext.generate_legal_moves_batch(st, m)
        res, _, _ = ext.child_probe_batch(st, legal, nl, m, False)
        ok &= (res == 0).all(dim=1) & (nl > 0)
    keep = torch_nonzero(ok)[:n]
    if keep.numel() < n:
        raise RuntimeError(f"only {keep.numel()} of {n} start positions qualified")
    return st[keep].contiguous()


def torch_nonzero(mask):
    import torch
    return torch.nonzero(mask, as_tuple=False).squeeze(1)


def _search_steps(ranks: Ranks, orch, starts, warmup: int, steps: int):
    """Warm-up and timed searched moves: (ms max over ranks, per-rank ms,
    simulations of all ranks, evaluated positions and rows of all ranks,
    clocks, the last step's examples)."""
    import torch
    sampler = ClockSampler(ranks.local)
    sampler.start()
    for i in range(warmup):
        orch.self_play_batch(starts[i])
    torch.cuda.synchronize(ranks.dev)
    orch.sims_done.zero_()
    orch.rows_evaluated.zero_()
    orch.leaves_evaluated = 0
    box = {}

    it = iter(range(warmup, warmup + steps))

    def step():
        box["ex"] = orch.self_play_batch(starts[next(it)])  # host states in, training examples out

    ms, per_rank = timed_region(ranks, step, steps)
    clocks = sampler.stop()
    sims = sum(ranks.gather(float(orch.sims_done.item())))
    rows = sum(ranks.gather(float(orch.rows_evaluated.item())))
    leaves = sum(ranks.gather(float(orch.leaves_evaluated)))
    return ms, per_rank, sims, leaves, rows, clocks, box["ex"]


def _replay_gather(ranks: Ranks, examples) -> dict | None:
    """The once-per-iteration replay exchange at N > 1: every rank's examples
    of the last searched move all-gathered over NCCL (replay.gather_examples)."""
    if ranks.dist is None:
        return None
    import torch

    from hive_neuralnet_b200.replay import gather_examples, pack_examples
    flat = [e for games in examples for e in games]
    nbytes = int(pack_examples(flat).size)
    ranks.barrier()
    torch.cuda.synchronize(ranks.dev)
    t0 = time.perf_counter()
    got = gather_examples(flat)
    torch.cuda.synchronize(ranks.dev)
    ms = (time.perf_counter() - t0) * 1e3
    per_rank_ms = ranks.gather(ms)
    total = sum(ranks.gather(float(nbytes)))
    return {"examples_per_rank": len(flat), "examples_gathered": len(got), "bytes_per_rank": nbytes,
            "bytes_total": int(total), "ms": max(per_rank_ms), "per_rank_ms": per_rank_ms,
            "path": "replay.gather_examples: sizes then padded byte buffers, two NCCL all_gathers, "
                    "host pack / unpack included"}


def bench_mcts(args, ranks: Ranks) -> dict:
    """Gumbel-root MCTS, 512 games/GPU, 4,096 simulations
    per move, 16 considered actions, wave schedule (2, 4, 8, 16), FNN large
    random init (seed 0), seeded Philox Gumbel noise, Dirichlet off, root
    tactical probe on (the trainer's default).  One step = one searched move
    of every game; metric = simulations per second."""
    import torch

    from hive_neuralnet_b200.fnn import HiveFNN
    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    dev, rank, world = ranks.dev, ranks.rank, ranks.world
    ext = load_extension()
    torch.manual_seed(0)
    net = HiveFNN()
    games = args.games
    cfg = FNNMCTSConfig(num_simulations=args.sims, batch_size=games, max_game_length=1, dirichlet_epsilon=0.0,
                        seed=1234 + rank, max_tree_nodes=65536, expansion_mask=0,
                        short_forced_win_probe=True)
    orch = FNNMCTSOrchestrator(net, cfg, device=dev)
    W, K = args.mcts_warmup, args.mcts_steps
    starts = [_mcts_start_states(ext, games, SEED + 97 * (rank * 1000 + i), dev).cpu() for i in range(W + K)]
    ms, per_rank, sims, leaves, rows, clocks, examples = _search_steps(ranks, orch, starts, W, K)
    value = sims / (ms / 1e3)
    flops = leaves * FNN_FLOP_PER_LEAF + rows * FNN_FLOP_PER_ROW
    peak, peak_src = fp32_peak_tflops()
    achieved = flops / world / (ms / 1e3) / 1e12
    gather = _replay_gather(ranks, examples)
    rank_clocks = ranks.gather_obj(clocks)
    cpu_states = starts[0].numpy() if (rank == 0 and world == 1 and not args.no_cpu) else None
    del orch, starts
    torch.cuda.empty_cache()
    if rank != 0:
        return {}
    cpu = mcts_cpu_player_baseline(cpu_states, args.sims) if cpu_states is not None else None
    return {"metric": "MCTS simulations/sec", "value": value, "unit": "simulations/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config4: Gumbel MCTS {games} games/GPU x {args.sims} sims/move, k=16, "
                                   "waves (2,4,8,16), FNN large random init",
                       "simulations": sims, "games_per_gpu": games,
                       "parallelism": f"games sharded dp{world}" if world > 1 else "single GPU",
                       "l2": "tree arrays (1.6 GB/GPU) larger than L2"},
            "e2e": {"value": value, "unit": "simulations/s", "h2d_bytes_per_step": games * STATE_BYTES,
                    "d2h_bytes_per_step": games * (STATE_BYTES + MAX_MOVES * 4 + 4 + 1 + 1),
                    "note": "the timed steps are end to end: start states come from pinned-less host memory and "
                            "the move's states, policy targets, move counts and flags return to the host in every "
                            "step (self_play_batch's public API)"},
            "roofline": {"bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": peak_src, "traffic": None,
                         "algorithmic_flop": flops / world,
                         "formula": f"{FNN_FLOP_PER_LEAF} FLOP per evaluated position + {FNN_FLOP_PER_ROW} per "
                                    f"successor row (FNN large), per GPU per step time",
                         "evaluated_positions": leaves, "successor_rows": rows},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "per_rank": {"ms_per_step": [t / K for t in per_rank],
                         "clocks": [{"sm_mhz": c.get("sm_mhz"), "reasons": c.get("reasons")} for c in rank_clocks]},
            "replay_gather": gather}


def mcts_cpu_player_baseline(roots_np, sims: int, seconds: float = 15.0) -> dict:
    """The reference's CPU player for the Gumbel search (FNNNativeCPUPlayer,
    hive_fnn/fnn_native_cpu_player.py:211-281), restated in oracle/cpu_player.py
    over the reference's own cpu_native backend built into oracle/_ref: one
    game per process on every host core, torch on one thread per process."""
    from oracle import cpu_player as CP
    if CP.backend_path() is None:
        return {"value": None, "unit": "simulations/s", "cores": 0, "kind": "port",
                "sample": "oracle/_ref cpu_native backend not built"}
    cores = host_cores()
    rate, done, wall, moves = CP.timed_rate(roots_np, sims, cores, seconds)
    return {"value": rate, "unit": "simulations/s", "cores": cores, "kind": "port",
            "sample": f"FNNNativeCPUPlayer's Gumbel search (restated in oracle/cpu_player.py, pinned to the "
                      f"reference player by tests/test_cpu_player.py) over the reference's compiled cpu_native "
                      f"backend, {sims} simulations per move, one game per process x {cores} processes for "
                      f"{wall:.1f} s ({done} simulations, {moves} moves finished), {cpu_model()}"}


def mcts_cpu_baseline(net, roots_np, sims, wave, c_puct, hybrid):
    """CPU restatement of the search (oracle tree ops, oracle successor features,
    fp32 torch CPU network on every host thread) timed on a bounded sample."""
    import torch

    from oracle import cpu_search as CS
    from oracle import oracle as O
    orc = O.oracle()
    cores = host_cores()
    torch.set_num_threads(cores)
    net_cpu = net.cpu().eval()
    ev = ((lambda s, m, n, f: CS.hybrid_eval(net_cpu, orc, s, m, n, f)) if hybrid
          else (lambda s, m, n, f: CS.fnn_eval(net_cpu, orc, s, m, n, f)))
    rate, done, dt = CS.timed_search(ev, roots_np, sims, wave, c_puct, min_seconds=10.0)
    return {"value": rate, "unit": "simulations/s", "cores": cores, "kind": "port",
            "sample": f"{len(roots_np)} of the timed roots x {sims} PUCT simulations in waves of {wave}, repeated "
                      f"for {dt:.1f} s ({done} simulations): C oracle tree ops / move generation / successor "
                      f"features + fp32 torch CPU {'hybrid' if hybrid else 'FNN'} evaluator, {cpu_model()}"}


def run_fnn(args) -> None:
    """Config 3: leaf evaluation of 65,536 roots (all legal successors)
    with FNN large (fp32, random init seed 0)."""
    import torch

    from hive_neuralnet_b200.fnn import FusedFNNEvaluator, HiveFNN
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    ev = FusedFNNEvaluator(HiveFNN(), dev)
    P = 65536 if args.positions == POSITIONS_DEFAULT else args.positions
    st = ext.generate_positions(SEED + 3, 0, P, MAX_PLY, EXPANSIONS, device=dev)
    legal, nl, feats = ext.generate_legal_moves_and_fnn_features_batch(st, P)
    for _ in range(args.warmup):
        ev.eval_states(st, legal, nl, P, feats)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ev.eval_states(st, legal, nl, P, feats)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    succ = int(nl.sum().item())
    flops = P * FNN_FLOP_PER_LEAF + succ * FNN_FLOP_PER_ROW
    peak, peak_src = fp32_peak_tflops()
    cpu = None
    if not args.no_cpu:
        from oracle import cpu_search as CS
        from oracle import oracle as O
        orc = O.oracle()
        cores = host_cores()
        torch.set_num_threads(cores)
        net_cpu = ev.net.cpu().eval()
        sample = st[:2048].cpu().numpy()
        smv, snl, sft = (x[:2048].cpu().numpy() for x in (legal, nl, feats))
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            CS.fnn_eval(net_cpu, orc, sample, smv, snl, sft)
            done += len(sample)
        dt = time.perf_counter() - t0
        cpu = {"value": done / dt, "unit": "roots/s", "cores": cores, "kind": "port",
               "sample": f"first 2048 roots of the workload, repeated for {dt:.1f} s: C oracle successor "
                         f"features + fp32 torch CPU HiveFNN, {cpu_model()}"}
    print(json.dumps({"metric": "FNN leaf evaluations/sec", "value": P / (ms / 1e3), "unit": "roots/s",
                      "successors_per_s": succ / (ms / 1e3), "ms_per_step": ms, "steps": args.steps,
                      "warmup": args.warmup, "n_gpus": 1, "dtype": "f32", "data": "synthetic",
                      "config": {"workload": f"config3: {P} roots x all legal successors, FNN large fp32",
                                 "successors": succ},
                      "roofline": {"bound": "fp32", "achieved": flops / (ms / 1e3) / 1e12, "peak": peak,
                                   "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / peak,
                                   "peak_source": peak_src, "traffic": None},
                      "cpu_baseline": cpu}), flush=True)


HYBRID_GAMES = 256
HYBRID_SIMS = 1024
HYBRID_WAVE = 32  # 256 games x 32 = 8,192 leaves per wave
TRUNK_FLOP_PER_LEAF = 7.61e6  # algorithmic trunk FLOPs per position (29 tokens, 4 blocks)
# tensor FLOPs of the hybrid evaluation: per position the trunk, the value
# head and the root FNN encode (~7.65 MFLOP); per legal action the FNN
# successor encode, graph and move projections and the action layer (68.9 KFLOP)
HYBRID_FLOP_PER_LEAF = 7.65e6
HYBRID_FLOP_PER_ROW = 68.9e3


def bench_hybrid(args, ranks: Ranks) -> dict:
    """Config 5: PUCT MCTS with the hybrid FNN-transformer evaluator, 256
    games/GPU, 1,024 simulations per move, c_puct 1.5, 8,192 leaves per wave,
    HybridGNNConfig() random init (seed 0), fp16-operand tensor-core trunk
    (fp32 accumulation; the reference runs this network under fp16 autocast).  One step
    = one searched move of every game; metric = simulations per second."""
    import torch

    from hive_neuralnet_b200.hive_gpu import load_extension
    from hive_neuralnet_b200.hybrid import HiveHybridGNN, HybridPieceTensorBatch
    from hive_neuralnet_b200.orchestrator import HybridPUCTConfig, HybridPUCTOrchestrator
    dev, rank, world = ranks.dev, ranks.rank, ranks.world
    ext = load_extension()
    torch.manual_seed(0)
    net = HiveHybridGNN().eval()
    games = args.games if args.games != MCTS_GAMES else HYBRID_GAMES
    sims = args.sims if args.sims != MCTS_SIMS else HYBRID_SIMS
    cfg = HybridPUCTConfig(num_simulations=sims, batch_size=games, max_game_length=1, dirichlet_epsilon=0.0,
                           seed=4321 + rank, max_tree_nodes=65536, wave_size=HYBRID_WAVE, c_puct=1.5)
    orch = HybridPUCTOrchestrator(net, cfg, device=dev)
    W, K = args.hybrid_warmup, args.hybrid_steps
    starts = [_mcts_start_states(ext, games, SEED + 131 * (rank * 1000 + i), dev, no_immediate_end=True).cpu()
              for i in range(W + K)]
    ms, per_rank, done, leaves, rows, clocks, _ = _search_steps(ranks, orch, starts, W, K)
    value = done / (ms / 1e3)
    flops = leaves * HYBRID_FLOP_PER_LEAF + rows * HYBRID_FLOP_PER_ROW
    peak_s, peak_s_src = bf16_peak_tflops(sustained=True)
    achieved = flops / world / (ms / 1e3) / 1e12

    # trunk kernel alone on one wave's worth of leaves (8,192 positions)
    L = games * HYBRID_WAVE
    st = ext.generate_positions(SEED + 5, 0, L, MAX_PLY, 0, device=dev)
    mv, nl = ext.generate_legal_moves_batch(st, L)
    pb = HybridPieceTensorBatch(*ext.hybrid_transformer_encode_with_moves_batch(st, mv, nl, L))
    trunk = orch.evaluator.trunk
    for _ in range(3):
        trunk(pb)
    torch.cuda.synchronize(dev)
    reps = 20
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(reps):
        trunk(pb)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    trunk_ms = t0.elapsed_time(t1) / reps
    peak_b, peak_b_src = bf16_peak_tflops(sustained=False)
    trunk_tf = L * TRUNK_FLOP_PER_LEAF / (trunk_ms / 1e3) / 1e12
    rank_clocks = ranks.gather_obj(clocks)
    cpu_roots = starts[0][:32].numpy() if (rank == 0 and world == 1 and not args.no_cpu) else None
    del orch, starts, st, mv, nl, pb
    torch.cuda.empty_cache()
    if rank != 0:
        return {}
    cpu = None
    if cpu_roots is not None:
        cpu = mcts_cpu_baseline(net, cpu_roots, sims=128, wave=HYBRID_WAVE, c_puct=1.5, hybrid=True)
    return {"metric": "MCTS simulations/sec", "value": value, "unit": "simulations/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"config5: PUCT {games} games/GPU x {sims} sims/move, c_puct 1.5, "
                                   f"{games * HYBRID_WAVE} leaves/wave, HybridGNNConfig() random init "
                                   f"({net.count_parameters()} params)",
                       "simulations": done, "games_per_gpu": games,
                       "parallelism": f"games sharded dp{world}" if world > 1 else "single GPU"},
            "e2e": {"value": value, "unit": "simulations/s", "h2d_bytes_per_step": games * STATE_BYTES,
                    "d2h_bytes_per_step": games * (STATE_BYTES + MAX_MOVES * 4 + 4 + 1),
                    "note": "the timed steps are end to end: start states come from host memory and training "
                            "examples return to it inside every step (self_play_batch's public API)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_s, "unit": "TFLOP/s",
                         "frac": achieved / peak_s, "peak_source": peak_s_src, "traffic": None,
                         "formula": f"{HYBRID_FLOP_PER_LEAF:.3g} FLOP per evaluated position + "
                                    f"{HYBRID_FLOP_PER_ROW:.3g} per legal action, per GPU per step time",
                         "evaluated_positions": leaves, "successor_rows": rows,
                         "trunk_kernel": {"kernel": f"k_hybrid_trunk on {L} positions ({trunk_ms:.3f} ms, alone)",
                                          "achieved": trunk_tf, "peak": peak_b, "peak_source": peak_b_src,
                                          "frac": trunk_tf / peak_b,
                                          "algorithmic_flop_per_position": TRUNK_FLOP_PER_LEAF}},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "per_rank": {"ms_per_step": [t / K for t in per_rank],
                         "clocks": [{"sm_mhz": c.get("sm_mhz"), "reasons": c.get("reasons")} for c in rank_clocks]}}


def run_gpu(args) -> None:
    import torch
    ranks = Ranks()
    line = {}
    if args.workload in ("all", "movegen"):
        line = bench_movegen(args, ranks)
    if args.workload in ("all", "mcts"):
        rec = bench_mcts(args, ranks)
        line = rec if args.workload == "mcts" else {**line, "mcts": rec}
    if args.workload in ("all", "hybrid"):
        rec = bench_hybrid(args, ranks)
        line = rec if args.workload == "hybrid" else {**line, "hybrid": rec}
    torch.cuda.synchronize(ranks.dev)
    ranks.close()
    if ranks.rank == 0:
        print(json.dumps(line), flush=True)


def main() -> None:
    global POSITIONS
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["all", "movegen", "mcts", "fnn", "hybrid"], default="all",
                    help="all: the headline (config 2) line with the config-4 and config-5 records in it")
    ap.add_argument("--games", type=int, default=MCTS_GAMES)
    ap.add_argument("--sims", type=int, default=MCTS_SIMS)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--mcts-steps", type=int, default=5, help="timed searched moves of the config-4 record")
    ap.add_argument("--mcts-warmup", type=int, default=3)
    ap.add_argument("--hybrid-steps", type=int, default=10, help="timed searched moves of the config-5 record")
    ap.add_argument("--hybrid-warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline legs")
    ap.add_argument("--e2e-chunk", type=int, default=32768, help="positions per pipelined chunk of the e2e leg")
    ap.add_argument("--long-s", type=float, default=2.0,
                    help="seconds of the config-2 steps' second, long timed region (0: none; profiling runs)")
    ap.add_argument("--positions", type=int, default=POSITIONS,
                    help="positions per GPU (profiling runs use a smaller case)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.mcts_warmup = max(args.mcts_warmup, 3)
    args.hybrid_warmup = max(args.hybrid_warmup, 3)
    POSITIONS = args.positions
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "fnn":
        run_fnn(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
