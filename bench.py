"""Benchmark: dense-constant fold GB/s (in+out) and pass wall time on B200.

Workload (one step): configuration 2, the 4096x4096 f32 fold chain — four
dense constants A, B, C, D (uniform[-4,4), 0.5% exact zeros in the divisor)
folded through addf, mulf, subf, divf, maximumf, minimumf: six elementwise
folds of 16,777,216 elements, 192 MiB of algorithmic traffic each (two
64 MiB operands in, one 64 MiB result out), 1.125 GiB per step.

  value  GB/s of algorithmic bytes with the constants resident in HBM: the
         six fold kernels back to back through the device entry points,
         timed per step with CUDA events on the launch stream (each fold
         pays the write-back of the previous one); a 256 MiB write evicts
         L2 between steps;
  roofline  each fold kernel alone (a 256 MiB read evicts L2 before it),
         achieved = bytes per launch / mean launch time, against the
         measured HBM copy bandwidth;
  e2e    the same configuration end to end through the pass driver's C ABI
         (dcf_opt_run): its MLIR text (537 MB of dense<"0x..."> literals)
         in pageable host memory, `canonicalize`, the run phase timed as
         the reference's bench does (fuzz/src/bench.rs:55-66): every fold,
         with the literals' copies to the GPU and every folded constant
         back in host memory; GB/s = the six folds' algorithmic bytes per
         run.  Every printed module is checked against the expected results
         (tests/golden/config_digests.json) before the line is printed;
  pass_config5  configuration 5 (4096 functions + the 16384^2 bf16
         transpose, 5.4 GB of text in page-locked memory; the pageable
         figure beside it) through
         builtin.module(func.func(tosa-layerwise-constant-fold,canonicalize)),
         same timing and check;
  cpu_baseline  the oracle (the scalar C restatement of the reference's
         fold loop, which runs single-threaded in the reference) timed on
         this host on a bounded sample.

Multi-GPU (strong scaling: one module, fixed total work): one process per
GPU (torchrun).  For `value` each rank folds one contiguous element range
of every constant — the split the pass driver makes for a bare
canonicalize — with no data-path collective; value = the step's bytes over
the slowest rank's time.  For `e2e` and `pass_config5` rank 0 runs the
module through the pass driver on all N GPUs while the other ranks wait on
the host.

`--impl reference` times the reference's CPU fold path instead: the oracle
port with all host threads (the reference cannot be built here: no Rust
toolchain, and its arithmetic crate is not vendored).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SIDE = 4096
N = SIDE * SIDE
FOLD_BYTES = 3 * 4 * N                 # two f32 operands in, one f32 result out
CHAIN = [("addf", "A", "B", "t1"), ("mulf", "t1", "C", "t2"), ("subf", "t2", "D", "t3"),
         ("divf", "t3", "D", "t4"), ("maximumf", "t4", "A", "t5"), ("minimumf", "t5", "B", "t6")]
STEP_BYTES = FOLD_BYTES * len(CHAIN)
# config 5: 4096 functions x (addf 12 + mulf 12 + reciprocal 8 bytes per
# element of 65,536 f32) + the 16384^2 bf16 transpose (4 bytes per element)
CONFIG5_BYTES = 4096 * 65536 * (12 + 12 + 8) + 16384 * 16384 * 4
METRIC = "dense-constant fold GB/s (in+out)"
CONFIG = {
    "workload": "4x 4096x4096 f32 dense constants folded by the chain addf, mulf, subf, divf, maximumf, "
                "minimumf under canonicalize (6 folds x 16,777,216 elements, 1.125 GiB algorithmic per step)",
    "elements_per_fold": N,
    "folds_per_step": len(CHAIN),
    "bytes_per_step": STEP_BYTES,
    "l2": "operands (256 MiB) exceed L2; before every timed fold a 256 MiB read-only pass evicts L2 "
          "(a read, so no dirty lines are left to write back inside the timed kernel)",
    "unit_per_gpu": "one isolated function (the fold chain) per GPU",
}


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """dram bytes per launch of the fold kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ew_binary_f32_chain4096.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus):
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------- our arm

def row_block(world: int, rank: int) -> tuple[int, int]:
    """This rank's element range of each constant: the module's folds split
    into one contiguous range per GPU (boundaries on multiples of 4096
    elements), as the pass driver splits a bare canonicalize's constants."""
    lo = (N * rank // world) // 4096 * 4096
    hi = N if rank == world - 1 else (N * (rank + 1) // world) // 4096 * 4096
    return lo, hi


def wait_for_rank0(world: int, rank: int, key: str):
    """Ranks other than 0 wait, on the host, while rank 0 drives every GPU
    through the pass driver (no kernel of theirs runs meanwhile)."""
    if world == 1:
        return
    import datetime
    import torch.distributed as dist
    store = dist.distributed_c10d._get_default_store()
    if rank == 0:
        store.set(key, "1")
    else:
        store.wait([key], datetime.timedelta(seconds=900))


def digests():
    with open(os.path.join(ROOT, "tests", "golden", "config_digests.json")) as fh:
        return json.load(fh)


def verify_module(out, config: str) -> bool:
    """Check a printed module's returned values against the committed
    digests of the configuration's expected results (computed from the
    oracle by tests/golden/make_config_digests.py); a mismatch ends the run
    without a bench line."""
    for d in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
        if d not in sys.path:
            sys.path.insert(0, d)
    from full_module import returns_digest, scan
    got = returns_digest(scan(bytes(out)))
    if got != digests()[config]:
        raise SystemExit(f"{config}: the printed module differs from the expected results ({got})")
    return True


def pass_runs(opt, text, pipeline, n_gpus, warmup, steps, config):
    """Run a pipeline over pageable module text `warmup + steps` times; the
    run phases of the last `steps` are kept; the last output is checked."""
    runs, out = [], None
    for r in range(warmup + steps):
        t0 = time.perf_counter()
        out, st = opt.run(text, pipeline, n_gpus=n_gpus, as_array=True)
        st["wall_ms"] = (time.perf_counter() - t0) * 1e3
        if r >= warmup:
            runs.append(st)
        if r + 1 < warmup + steps:
            del out
    ok = verify_module(out, config)
    del out
    return runs, ok


def pass_summary(runs, algo_bytes, config, pipeline, text_bytes, n_gpus, ok, memory="pageable"):
    mean = lambda k: statistics.mean(s[k] for s in runs)
    run_ms = mean("run_ms")
    return {"config": config, "pipeline": pipeline, "n_gpus": n_gpus, "text_bytes": text_bytes,
            "text_memory": memory, "runs": len(runs),
            "run_ms": round(run_ms, 3), "run_ms_best": round(min(s["run_ms"] for s in runs), 3),
            "call_ms": round(mean("call_ms"), 2), "parse_ms": round(mean("parse_ms"), 2),
            "print_ms": round(mean("print_ms"), 2), "upload_ms": round(mean("upload_ms"), 2),
            "fold_ms": round(mean("fold_ms"), 2), "download_ms": round(mean("download_ms"), 2),
            "folds": runs[-1]["folds"], "refused": runs[-1]["refused"],
            "h2d_bytes": runs[-1]["h2d_bytes"], "d2h_bytes": runs[-1]["d2h_bytes"],
            "algorithmic_bytes": algo_bytes,
            "GB/s": round(algo_bytes / (run_ms * 1e-3) / 1e9, 2) if algo_bytes else None,
            "verified": ok}


def run_gpu(args):
    import torch
    import mlirpass_b200 as dcf
    from mlirpass_b200 import mlir_gen as G
    from mlirpass_b200 import opt
    from mlirpass_b200 import workloads as W

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    os.environ["DCF_DEVICES"] = str(local)
    dcf.init(1)
    dev = torch.device("cuda", local)

    d = W.config2(SIDE)
    lo, hi = row_block(world, rank)
    n = hi - lo
    fold_bytes = 3 * 4 * n
    host = {k: d[k] for k in "ABCD"}
    # device-resident operands (this rank's rows) and results
    res = {k: torch.from_numpy(host[k][lo:hi].copy()).to(dev) for k in "ABCD"}
    for _, _, _, t in CHAIN:
        res[t] = torch.empty(n, dtype=torch.float32, device=dev)
    status = torch.empty(len(CHAIN) * 2, dtype=torch.int64, device=dev)
    flush = torch.ones(32 << 20, dtype=torch.int64, device=dev)   # 256 MiB (L2 is 126 MB)
    stream = torch.cuda.current_stream(dev)

    def chain(fold_events=None, read_flush=False, on=None):
        on = on or stream
        if not read_flush:
            status.fill_(-1)          # the six statuses at once (all bytes 0xFF)
        for i, (op, a, b, t) in enumerate(CHAIN):
            st = status[2 * i:2 * i + 2]
            if read_flush:
                flush.sum()
                dcf.status_reset(st, on)
            if fold_events is not None:
                fold_events[i][0].record(on)
            dcf.binary_async(op, "f32", res[a], res[b], res[t], st, n=n, stream=on)
            if fold_events is not None:
                fold_events[i][1].record(on)

    for _ in range(args.warmup):
        chain(read_flush=True)
    torch.cuda.synchronize()
    for i in range(len(CHAIN)):
        r = dcf.status_read(status[2 * i:2 * i + 2], stream)
        if not r.folded:
            raise SystemExit(f"fold {CHAIN[i][0]} refused at {r.first_fail_index}")

    # The step's six launches are captured once in a CUDA graph and replayed:
    # at small per-GPU sizes (2M elements at 8 GPUs, ~7 us a fold) the host
    # cannot issue launches as fast as the GPU runs them.
    graph = None
    if not args.no_graph:
        try:
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            with torch.cuda.graph(g, stream=cap):
                chain(on=cap)
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            graph = g
        except Exception as e:  # noqa: BLE001 - fall back to launching from the host
            sys.stderr.write(f"graph capture of the chain failed ({e}); launching from the host\n")
            torch.cuda.synchronize()
    step = graph.replay if graph is not None else chain

    clocks = Clocks(local)
    clocks.start()
    launches0 = dcf.kernel_launches()
    # ---- value: whole steps (the six folds back to back, each paying the
    # write-back of the one before); between steps a 256 MiB write evicts L2.
    barrier(world)
    torch.cuda.synchronize()
    step_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for s in range(args.steps):
        flush.add_(1)
        step_ev[s][0].record(stream)
        step()
        step_ev[s][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    step_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in step_ev)
    # ---- roofline: each fold alone, a 256 MiB read evicting L2 before it
    fold_ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in CHAIN] for _ in range(args.steps)]
    for s in range(args.steps):
        chain(fold_ev[s], read_flush=True)
    torch.cuda.synchronize()
    barrier(world)
    value_launches = dcf.kernel_launches() - launches0 + (len(CHAIN) * args.steps if graph is not None else 0)
    fold_ms = [[fold_ev[s][i][0].elapsed_time(fold_ev[s][i][1]) for i in range(len(CHAIN))]
               for s in range(args.steps)]
    kernel_ms = sum(sum(x) for x in fold_ms) / (args.steps * len(CHAIN))
    per_fold_us = {CHAIN[i][0]: round(1000.0 * sum(fold_ms[s][i] for s in range(args.steps)) / args.steps, 2)
                   for i in range(len(CHAIN))}
    step_ms_max = allreduce_max(step_ms, world)
    kernel_ms_max = allreduce_max(kernel_ms, world)

    # ---- e2e: the whole configuration through the pass driver, from its MLIR
    # text in pageable host memory (and, as a second figure, in page-locked
    # memory); rank 0 drives all `world` GPUs (the module's constants split
    # into one element range per GPU) while the other ranks wait on the host.
    e2e = e2e_pinned = p5 = p5_pageable = None
    launches1 = dcf.kernel_launches()
    if rank == 0:
        text2 = G.config2_module().tobytes()
        runs2, ok2 = pass_runs(opt, text2, "canonicalize", world, args.warmup, args.steps, "config2")
        e2e = pass_summary(runs2, STEP_BYTES, "config2", "canonicalize", len(text2), world, ok2)
        pin2 = opt.pinned_text(text2)
        runs2p, ok2p = pass_runs(opt, pin2, "canonicalize", world, args.warmup, args.steps, "config2")
        e2e_pinned = pass_summary(runs2p, STEP_BYTES, "config2", "canonicalize", len(text2), world, ok2p, "pinned")
        del text2, pin2
        if not args.no_config5:
            text5 = G.config5_module(4096).tobytes()
            reps = max(1, min(args.steps, 3))
            pin5 = opt.pinned_text(text5)
            runs5, ok5 = pass_runs(opt, pin5, G.LAYERWISE, world, 1, reps, "config5")
            p5 = pass_summary(runs5, CONFIG5_BYTES, "config5", G.LAYERWISE, len(text5), world, ok5, "pinned")
            del pin5
            runs5q, ok5q = pass_runs(opt, text5, G.LAYERWISE, world, 1, reps, "config5")
            p5_pageable = pass_summary(runs5q, CONFIG5_BYTES, "config5", G.LAYERWISE, len(text5), world, ok5q)
            del text5
    pass_launches = dcf.kernel_launches() - launches1
    wait_for_rank0(world, rank, "pass_done")
    barrier(world)
    clk = clocks.stop()

    # ---- the host C ABI on raw operands (pinned host buffers): each fold
    # copies its operands in and its result out
    pin = {k: torch.from_numpy(host[k][lo:hi].copy()).pin_memory() for k in "ABCD"}
    for _, _, _, t in CHAIN:
        pin[t] = torch.empty(n, dtype=torch.float32).pin_memory()
    npv = {k: v.numpy() for k, v in pin.items()}

    def host_step():
        for op, a, b, t in CHAIN:
            f = dcf.binary(op, "f32", npv[a], npv[b], out=npv[t].view(np.uint32))
            if not f.folded:
                raise SystemExit(f"host fold {op} refused")

    for _ in range(max(1, args.warmup)):
        host_step()
    launches2 = dcf.kernel_launches()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_step()
    cabi_s = time.perf_counter() - t0
    barrier(world)
    cabi_launches = dcf.kernel_launches() - launches2
    same = all(torch.equal(res[t].cpu(), pin[t]) for _, _, _, t in CHAIN)
    cabi_ms_max = allreduce_max(cabi_s * 1000.0 / args.steps, world)
    launches = allreduce_max(float(value_launches + cabi_launches), world) + pass_launches

    if rank != 0:
        return
    peak, peak_kind = load_peaks()
    gbs = STEP_BYTES / (step_ms_max * 1e-3) / 1e9
    achieved = fold_bytes / (kernel_ms_max * 1e-3) / 1e9
    traffic = load_traffic() if world == 1 else None
    line = {
        "metric": METRIC,
        "value": round(gbs, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms_max, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (SplitMix64-seeded dense constants; no dataset)",
        "config": dict(CONFIG, parallelism=f"one module over {world} GPU(s): each constant split into "
                                            f"{world} element range(s), one per GPU",
                       elements_per_gpu=n, results_bit_identical_device_vs_host_path=same),
        "e2e": {"value": e2e["GB/s"], "unit": "GB/s", "ms_per_step": e2e["run_ms"],
                "h2d_bytes_per_step": e2e["h2d_bytes"], "d2h_bytes_per_step": e2e["d2h_bytes"],
                "path": "dcf_opt_run (the pass driver's C ABI) on the configuration's MLIR text in pageable "
                        "host memory, canonicalize: the run phase (every fold, with the literals' host->device "
                        "copies and decode and every folded constant back in host memory), as the "
                        "reference's bench times it; the printed module is checked against the expected "
                        "results every run",
                "pass": e2e,
                "pinned_text": e2e_pinned,
                "c_abi_pinned": {"value": round(STEP_BYTES / (cabi_ms_max * 1e-3) / 1e9, 2), "unit": "GB/s",
                                 "ms_per_step": round(cabi_ms_max, 3),
                                 "path": "dcf_binary (host C ABI) on raw operands in pinned host buffers, this "
                                         "rank's rows, 6 calls per step"}},
        "pass_config5": p5,
        "pass_config5_pageable": p5_pageable,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "ew_tma_kernel<FArith/FMinMax f32>: cp.async.bulk 16 KB tiles, 2 stages, "
                               "3 CTAs/SM; fused fold + refusal + splat test",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "timing": "each fold alone, a 256 MiB read evicting L2 before it (part of its result is "
                               "still in L2 when it ends); value times the six folds back to back",
                     "value_frac": round(gbs / world / peak, 4),
                     "kernel_ms": round(kernel_ms_max, 5), "per_fold_us": per_fold_us,
                     "bytes_per_launch": fold_bytes},
        "gpu_launches": int(launches),
        "gpu_launches_detail": {"value_and_roofline": int(value_launches), "value_launch": "CUDA graph replay"
                                if graph is not None else "host launches", "pass_runs": int(pass_launches),
                                "c_abi": int(cabi_launches)},
        "clocks": clk,
    }
    if traffic:
        line["roofline"]["dram_rate_GBs"] = round(traffic / (kernel_ms_max * 1e-3) / 1e9, 1)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(host, budget_s=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def cpu_baseline(host, budget_s=12.0, threads=1):
    """Time the oracle on the same chain: whole chains until `budget_s`."""
    import oracle
    from concurrent.futures import ThreadPoolExecutor

    oracle.lib()
    env = {k: host[k] for k in "ABCD"}
    outs = {t: np.empty(N, dtype=np.uint32) for _, _, _, t in CHAIN}

    def fold(op, a, b, t, lo, hi):
        oracle.binary(op, "f32", env_v[a][lo:hi], env_v[b][lo:hi], out=outs[t][lo:hi])

    env_v = {k: v.view(np.uint32) for k, v in env.items()}
    for t in outs:
        env_v[t] = outs[t]
    bounds = [(N * i // threads, N * (i + 1) // threads) for i in range(threads)]
    pool = ThreadPoolExecutor(threads) if threads > 1 else None
    chains = 0
    folds = 0
    t0 = time.perf_counter()
    while True:
        for op, a, b, t in CHAIN:
            if pool:
                list(pool.map(lambda lh: fold(op, a, b, t, *lh), bounds))
            else:
                fold(op, a, b, t, 0, N)
            folds += 1
        chains += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    if pool:
        pool.shutdown()
    return {"value": round(folds * FOLD_BYTES / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{chains} full chains ({folds} folds of 16,777,216 f32) of the same workload, "
                      f"{dt:.1f} s, oracle C restatement (scalar, -O2)",
            "seconds": round(dt, 2)}


# ---------------------------------------------------------- reference arm

def run_reference(args):
    world, rank, _ = env_int("WORLD_SIZE", 1), env_int("RANK", 0), env_int("LOCAL_RANK", 0)
    if rank != 0:
        return
    from mlirpass_b200 import workloads as W
    import oracle
    from concurrent.futures import ThreadPoolExecutor

    oracle.lib()
    threads = os.cpu_count() or 1
    d = W.config2(SIDE)
    env = {k: d[k].view(np.uint32) for k in "ABCD"}
    for _, _, _, t in CHAIN:
        env[t] = np.empty(N, dtype=np.uint32)
    bounds = [(N * i // threads, N * (i + 1) // threads) for i in range(threads)]
    pool = ThreadPoolExecutor(threads)

    def step():
        for op, a, b, t in CHAIN:
            list(pool.map(lambda lh: oracle.binary(op, "f32", env[a][lh[0]:lh[1]], env[b][lh[0]:lh[1]],
                                                   out=env[t][lh[0]:lh[1]]), bounds))

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    pool.shutdown()
    ms = dt * 1000.0 / args.steps
    gbs = STEP_BYTES / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (SplitMix64-seeded dense constants; no dataset)",
        "config": dict(CONFIG, parallelism="host threads over row blocks (one process)"),
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "the full fold chain per step (the reference itself cannot be built here: "
                                   "no Rust toolchain, mlirformat 0.9.0 not vendored), oracle C restatement "
                                   f"on {threads} threads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------- per-configuration kernels

def run_kernels(args):
    """Every configuration's fold kernels on device-resident operands: one
    JSON line per kernel with its time and fraction of the HBM roof."""
    import torch
    import mlirpass_b200 as dcf
    from mlirpass_b200 import workloads as W

    torch.cuda.set_device(0)
    os.environ["DCF_DEVICES"] = "0"
    dcf.init(1)
    dev = torch.device("cuda", 0)
    peak, _ = load_peaks()
    flush = torch.ones(32 << 20, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    st = torch.empty(2, dtype=torch.int64, device=dev)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    def timeit(launch, nbytes, label, reps=None, in_bytes=None):
        # A fold that ends "not folded" counts its input bytes only.
        reps = reps or args.steps
        times = []
        for r in range(args.warmup + reps):
            flush.sum()
            dcf.status_reset(st, stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launch()
            e1.record(stream)
            torch.cuda.synchronize()
            if r >= args.warmup:
                times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        folded = dcf.status_read(st).folded
        if not folded and in_bytes is not None:
            nbytes = in_bytes
        gbs = nbytes / (ms * 1e-3) / 1e9
        line = {"workload": label[0], "fold": label[1], "us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                "frac": round(gbs / peak, 3), "bytes": nbytes, "folded": bool(folded)}
        print(json.dumps(line), flush=True)

    # config 1 / 2 (f32 binary)
    c1 = W.config1()
    a, b = T(c1["A"]), T(c1["B"])
    o = torch.empty_like(a)
    timeit(lambda: dcf.binary_async("addf", "f32", a, b, o, st), 12 * a.numel(), ("config1 1024x1024 f32", "addf"))
    # config 3 (integers)
    for dt in ("i8", "i32", "i64"):
        c = W.config3(dt)
        X, Y, S, Xd, Yd = (T(c[k].view({"i8": np.int8, "i32": np.int32, "i64": np.int64}[dt]))
                           for k in ("X", "Y", "S", "Xd", "Yd"))
        o = torch.empty_like(X)
        es = X.element_size()
        for op, l, r in (("addi", X, Y), ("muli", X, Y), ("subi", X, Y), ("andi", X, Y), ("xori", X, Y),
                         ("shli", X, S), ("divsi", Xd, Yd), ("remsi", Xd, Yd)):
            timeit(lambda op=op, l=l, r=r: dcf.binary_async(op, dt, l, r, o, st), 3 * es * X.numel(),
                   (f"config3 8192x2048 {dt}", op), in_bytes=2 * es * X.numel())
    # config 4 (conversions)
    c = W.config4()
    cp = W.config4(prerounded=True)
    x, xr, inr, ints = T(c["x"]), T(cp["x"]), T(c["inrange"]), T(c["ints"])
    n = x.numel()
    o16 = torch.empty(n, dtype=torch.int16, device=dev)
    o32 = torch.empty(n, dtype=torch.int32, device=dev)
    o8 = torch.empty(n, dtype=torch.uint8, device=dev)
    timeit(lambda: dcf.convert_async("truncf", "f32", "bf16", x, o16, st), 6 * n, ("config4 16M", "truncf f32->bf16 (refuses)"), in_bytes=4 * n)
    timeit(lambda: dcf.convert_async("truncf", "f32", "bf16", xr, o16, st), 6 * n, ("config4b 16M", "truncf f32->bf16"), in_bytes=4 * n)
    timeit(lambda: dcf.convert_async("truncf", "f32", "f16", x, o16, st), 6 * n, ("config4 16M", "truncf f32->f16 (refuses)"), in_bytes=4 * n)
    timeit(lambda: dcf.convert_async("extf", "bf16", "f32", o16, o32, st), 6 * n, ("config4b 16M", "extf bf16->f32"), in_bytes=2 * n)
    timeit(lambda: dcf.convert_async("fptosi", "f32", "i32", inr, o32, st), 8 * n, ("config4 16M", "fptosi f32->i32"), in_bytes=4 * n)
    timeit(lambda: dcf.convert_async("sitofp", "i32", "f32", ints, o32, st), 8 * n, ("config4 16M", "sitofp i32->f32"), in_bytes=4 * n)
    timeit(lambda: dcf.binary_async("cmpf", "f32", x, inr, o8, st, flags=4 << 8), 9 * n,
           ("config4 16M", "cmpf olt (kernel only; dense cmpf is not folded)"))
    # config 5: 4096 functions per step, batched; and the 16384^2 bf16 transpose
    funcs = [W.config5_func(i) for i in range(args.funcs)]
    A = [T(f[0]) for f in funcs]
    B = [T(f[1]) for f in funcs]
    O = [torch.empty_like(t) for t in A]

    def tables(op, unary=False):
        # job tables built once, outside the timed region
        return [dcf.device_jobs([{"op": op, "dtype": "f32", "lhs": A[i], "out": O[i],
                                  **({} if unary else {"rhs": B[i]})}
                                 for i in range(k, min(k + dcf.NOALLOC_MAX_JOBS, len(A)))])
                for k in range(0, len(A), dcf.NOALLOC_MAX_JOBS)]

    def batched(tabs):
        for t in tabs:
            dcf.run_device_jobs(t, stream)
    per = A[0].numel()
    t_add, t_rec = tables("addf"), tables("reciprocal", True)
    timeit(lambda: batched(t_add), 12 * per * len(A), (f"config5 {len(A)} funcs 256x256", "addf (batched)"), reps=5)
    timeit(lambda: batched(t_rec), 8 * per * len(A), (f"config5 {len(A)} funcs 256x256", "reciprocal (batched)"),
           reps=5)
    w = T(W.config5_weight().view(np.int16))
    wo = torch.empty_like(w)
    kind = "bulk-tensor pipeline" if os.environ.get("DCF_TRANSPOSE") == "tma" else "tiled loads, prefetched"
    timeit(lambda: dcf.permute_async(2, (16384, 16384), (1, 0), w, wo, st), 4 * w.numel(),
           ("config5 16384x16384 bf16", f"transpose (dcf_permute_status_async: {kind})"))
    timeit(lambda: dcf.transpose2d_async(2, 16384, 16384, w, wo), 4 * w.numel(),
           ("config5 16384x16384 bf16", "transpose (dcf_transpose2d_async: tiled loads, prefetched)"))


def run_profile_kernels(args):
    """One launch per round (two rounds) of the kernels profiled with ncu:
    truncf f32->bf16, fptosi f32->i32, addi / divsi / shli / remsi i8 (the
    last three lane-wise with a refusal mask), remsi i64 (32M elements), the
    batched addf of 1024 256x256 functions, and the 16384x16384 bf16
    transpose (bulk-tensor and plain-load kernels).  Operands are device-resident and larger than L2;
    nothing is timed here (the numbers come from the profiler)."""
    import torch
    import mlirpass_b200 as dcf
    torch.cuda.set_device(0)
    os.environ["DCF_DEVICES"] = "0"
    dcf.init(1)
    dev = torch.device("cuda", 0)
    n = 64 << 20
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    x = torch.randn(n, device=dev, generator=g) * 1e3
    xr = (x.view(torch.int32) & ~0xFFFF).view(torch.float32)          # bf16-representable
    xi = x.clamp(-2e9, 2e9)
    a8 = torch.randint(-128, 127, (n,), dtype=torch.int8, device=dev, generator=g)
    b8 = torch.randint(-128, 127, (n,), dtype=torch.int8, device=dev, generator=g)
    d8 = torch.where(b8 == 0, torch.ones_like(b8), b8)                  # nonzero divisors
    s8 = b8 & 7                                                          # in-range shift amounts
    w = torch.randint(-30000, 30000, (16384, 16384), dtype=torch.int16, device=dev, generator=g)
    o16 = torch.empty(n, dtype=torch.int16, device=dev)
    o32 = torch.empty(n, dtype=torch.int32, device=dev)
    o8 = torch.empty(n, dtype=torch.int8, device=dev)
    wo = torch.empty_like(w)
    st = torch.empty(2, dtype=torch.int64, device=dev)
    r64a = torch.randint(-2**62, 2**62, (n // 2,), dtype=torch.int64, device=dev, generator=g)
    r64b = torch.randint(1, 2**62, (n // 2,), dtype=torch.int64, device=dev, generator=g)
    o64 = torch.empty_like(r64a)
    A = [torch.rand(65536, device=dev, generator=g) for _ in range(1024)]
    B = [torch.rand(65536, device=dev, generator=g) for _ in range(1024)]
    O = [torch.empty(65536, device=dev) for _ in range(1024)]
    tab = dcf.device_jobs([{"op": "addf", "dtype": "f32", "lhs": A[i], "rhs": B[i], "out": O[i]} for i in range(1024)])
    for _ in range(2):
        dcf.run_device_jobs(tab)
        dcf.status_reset(st)
        dcf.convert_async("truncf", "f32", "bf16", xr, o16, st)
        dcf.status_reset(st)
        dcf.convert_async("fptosi", "f32", "i32", xi, o32, st)
        dcf.status_reset(st)
        dcf.binary_async("addi", "i8", a8, b8, o8, st)
        dcf.status_reset(st)
        dcf.binary_async("divsi", "i8", a8, d8, o8, st)
        dcf.status_reset(st)
        dcf.binary_async("shli", "i8", a8, s8, o8, st)
        dcf.status_reset(st)
        dcf.binary_async("remsi", "i8", a8, d8, o8, st)
        dcf.status_reset(st)
        dcf.binary_async("remsi", "i64", r64a, r64b, o64, st)
        dcf.status_reset(st)
        dcf.permute_async(2, (16384, 16384), (1, 0), w, wo, st)
        dcf.transpose2d_async(2, 16384, 16384, w, wo)
    torch.cuda.synchronize()
    print(json.dumps({"workload": "profile-kernels", "launch_rounds": 2}))


def gpu_local_cpus(dev: int) -> list[int]:
    """Host CPUs on the GPU's NUMA node (from sysfs), or every CPU."""
    try:
        import torch
        bus = torch.cuda.get_device_properties(dev).pci_bus_id.lower()
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as fh:
            cpus = []
            for part in fh.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus += list(range(int(lo), int(hi or lo) + 1))
        allowed = os.sched_getaffinity(0)
        return [c for c in cpus if c in allowed] or sorted(allowed)
    except (OSError, ValueError, AttributeError, RuntimeError):
        return sorted(os.sched_getaffinity(0))


def run_h2d(args):
    """The box's host<->device copy ceiling: every GPU of --gpus copies
    1 GiB blocks from page-locked host memory at once, (a) each from its
    own buffer, allocated by a thread bound to the GPU's NUMA node, and
    (b) all from one shared buffer; then the same device->host.  One line
    per mode with the aggregate and each GPU's GB/s (CUDA events per copy,
    the aggregate over the wall time of all copies)."""
    import torch
    n = args.gpus
    nbytes = 1 << 30
    reps = max(3, args.steps)
    shared = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    own, dev_bufs = [None] * n, [None] * n

    def setup(g):
        os.sched_setaffinity(0, gpu_local_cpus(g))
        own[g] = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        own[g].fill_(g)
        dev_bufs[g] = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{g}")

    ts = [threading.Thread(target=setup, args=(g,)) for g in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for mode in ("own", "shared"):
        for direction in ("h2d", "d2h"):
            per = [0.0] * n
            barrier_ = threading.Barrier(n)

            def work(g):
                torch.cuda.set_device(g)
                s = torch.cuda.Stream(g)
                host = own[g] if mode == "own" else shared
                ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(reps)]
                with torch.cuda.stream(s):
                    dev_bufs[g].copy_(host, non_blocking=True) if direction == "h2d" else \
                        host.copy_(dev_bufs[g], non_blocking=True)
                s.synchronize()
                barrier_.wait()
                with torch.cuda.stream(s):
                    for r in range(reps):
                        ev[r][0].record(s)
                        if direction == "h2d":
                            dev_bufs[g].copy_(host, non_blocking=True)
                        else:
                            host.copy_(dev_bufs[g], non_blocking=True)
                        ev[r][1].record(s)
                s.synchronize()
                per[g] = nbytes * reps / (sum(e0.elapsed_time(e1) for e0, e1 in ev) * 1e-3) / 1e9

            t0 = time.perf_counter()
            ts = [threading.Thread(target=work, args=(g,)) for g in range(n)]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            wall = time.perf_counter() - t0
            print(json.dumps({"workload": "h2d-ceiling", "mode": mode, "direction": direction, "n_gpus": n,
                              "bytes_per_copy": nbytes, "copies_per_gpu": reps,
                              "aggregate_GBs_wall": round(n * nbytes * reps / wall / 1e9, 1),
                              "per_gpu_GBs": [round(x, 1) for x in per],
                              "numa_local_cpus": [len(gpu_local_cpus(g)) for g in range(n)] if mode == "own" else None}),
                  flush=True)


def run_pass(args):
    """A whole pipeline through the pass driver on MLIR text: parse / run /
    print phases, like the reference's own bench (fuzz/src/bench.rs:55-66);
    the printed module of the last run is checked against the expected
    results before the line is printed."""
    from mlirpass_b200 import mlir_gen as G
    from mlirpass_b200 import opt
    cfg = args.workload.split(":", 1)[1]
    if cfg == "config1":
        mod, pipe = G.config1_module(), "canonicalize"
    elif cfg == "config2":
        mod, pipe = G.config2_module(), "canonicalize"
    elif cfg.startswith("config3"):
        cfg = cfg if "-" in cfg else "config3-i32"
        mod, pipe = G.config3_module(cfg.split("-")[1]), "canonicalize"
    elif cfg == "config4":
        mod, pipe = G.config4_module(), "canonicalize"
    elif cfg == "config4b":
        mod, pipe = G.config4_module(prerounded=True), "canonicalize"
    elif cfg == "config5":
        mod, pipe = G.config5_module(args.funcs), G.LAYERWISE
    else:
        raise SystemExit(f"unknown workload {args.workload}")
    text = mod.tobytes()
    # The module text is read from page-locked host memory (the driver then
    # copies constants straight from it), unless --pageable.
    src = text if args.pageable else opt.pinned_text(text)
    check = cfg if (cfg != "config5" or args.funcs == 4096) else None
    for n_gpus in ([int(x) for x in args.sweep_gpus.split(",")] if args.sweep_gpus else [args.gpus]):
        _pass_line(args, opt, cfg, pipe, text, src, n_gpus, check)


def _pass_line(args, opt, cfg, pipe, text, src, n_gpus, check):
    runs = []
    out = None
    total = max(1, args.warmup) + args.steps
    for r in range(total):
        t0 = time.perf_counter()
        out, st = opt.run(src, pipe, n_gpus=n_gpus, as_array=True)
        st["wall_ms"] = (time.perf_counter() - t0) * 1e3
        if r >= max(1, args.warmup):
            runs.append(st)
        if r + 1 < total:
            del out
    verified = verify_module(out, check) if check else None
    del out
    best = min(runs, key=lambda s: s["run_ms"])
    line = {"workload": f"pass {cfg}", "pipeline": pipe, "n_gpus": n_gpus, "text_bytes": len(text),
            "text_memory": "pageable" if args.pageable else "pinned",
            "parse_ms": round(best["parse_ms"], 2), "run_ms": round(best["run_ms"], 3),
            "run_ms_mean": round(statistics.mean(s["run_ms"] for s in runs), 3),
            "print_ms": round(best["print_ms"], 2), "call_ms": round(best["call_ms"], 1),
            "wall_ms": round(best["wall_ms"], 1),
            "upload_ms": round(best["upload_ms"], 2), "fold_ms": round(best["fold_ms"], 2),
            "download_ms": round(best["download_ms"], 2),
            "folds": best["folds"], "refused": best["refused"],
            "h2d_bytes": best["h2d_bytes"], "d2h_bytes": best["d2h_bytes"], "batches": best["batches"],
            "runs": len(runs), "verified": verified}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true", help="skip the config 5 pass runs of the default line")
    ap.add_argument("--no-graph", action="store_true", help="launch the value steps from the host, not a CUDA graph")
    ap.add_argument("--workload", default="chain4096",
                    help="chain4096 (the headline line), kernels, profile-kernels, h2d (host<->device copy "
                         "ceiling of --gpus GPUs at once), or pass:<config1|config2|config3-i8|...|config5>")
    ap.add_argument("--funcs", type=int, default=4096, help="functions of config 5")
    ap.add_argument("--pageable", action="store_true", help="pass workloads: keep the module text in pageable memory")
    ap.add_argument("--sweep-gpus", default="", help="pass workloads: GPU counts to run in turn, e.g. 1,2,4,8")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "kernels":
        run_kernels(args)
        return
    if args.workload == "profile-kernels":
        run_profile_kernels(args)
        return
    if args.workload.startswith("pass:"):
        run_pass(args)
        return
    if args.workload == "h2d":
        run_h2d(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)
        if env_int("WORLD_SIZE", 1) > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
