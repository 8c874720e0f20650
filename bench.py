"""Throughput benchmark of the batched policy/value evaluation
(InferenceEngine::predict_batch, include/inference_engine.h:25-32) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload b19c128x10_bs512|b19c256x20_bs1024|b9c128x10_bs256|b9c64x6_bs16
                                |selfplay_b19c128x10|selfplay_b19c128x10_fast|selfplay_b19c128x10_grouped]

A step is one forward pass of the network over one batch of seeded random-
playout positions.  Under torchrun each rank drives its own GPU with its own
batch (weights replicated, no collective on the data path); rank 0 prints one
JSON line.  Numbers:
  value      positions/s over all ranks, inputs resident in HBM, L2 flushed
             (256 MB write) before every timed step, CUDA-event timed on the
             engine's stream, max over ranks;
  e2e        the same through the host API with pinned host buffers: H2D of
             the inputs in the bit-packed wire format, forward, D2H of policy
             and value every step, wall-clock timed, max over ranks; through
             mg_submit_packed with two steps in flight, as the batching server
             runs (e2e_sync: one synchronous mg_forward_packed per step;
             e2e_fp32_planes: fp32 planes through mg_forward);
  roofline   the trunk (all 3x3 convolution layers; the dominant kernel,
             one persistent launch) timed alone with CUDA events:
             algorithmic FLOPs per launch / average launch time, against the
             measured dense bf16 peak;
  cpu_baseline  the oracle (C restatement of src/eigen_engine.cpp) on the
             host cores over a bounded sample (rank 0, N = 1 only), and
             torch_cpu: a torch restatement of the reference network
             (scripts/model.py) on all host cores over a bounded sample;
  configs    (N = 1, default workload only) the same value / e2e / roofline
             for the other predict_batch configurations: 19x19 b20c256
             batch 1024 (the configuration the 60% tensor-peak target is
             quoted on), 9x9 b10c128 batch 256 and 9x9 b6c64 batch 16;
  selfplay   (every N, default workload only) end-to-end self-play MCTS
             visits/s over all N GPUs after the per-rank engines are closed:
             rank 0 runs alphazero_b200/lib/selfplay_cuda with FastSearch
             (threaded and grouped) and with the reference's own search (the
             selfplay_b19c128x10* workloads below) for a bounded window each.
--impl reference times that CPU implementation alone as the reference arm.

selfplay_b19c128x10 is end-to-end self-play instead: the reference's own
search (src/mcts.cpp, compiled unmodified) with 64 game workers x 16 search
threads, 800 simulations per move, max batch 512, over one batching server
and engine per GPU (alphazero_b200/lib/selfplay_cuda); selfplay_b19c128x10_fast
is the same with FastSearch (alphazero_b200/host/fast_search.h, the
reference's algorithm at a lower host cost per visit), and
selfplay_b19c128x10_grouped with FastSearch's grouped mode (each worker's 16
concurrent playouts as rounds on its own thread, a round's leaves evaluated
as one group: one sleep and wake-up per round instead of per playout).  One process drives
all N GPUs (under torchrun rank 0 runs it, the other ranks wait).  A step is
one second of the measured window (at least 10), a warm-up step two seconds
(at least 6).  value = MCTS visits/s = searches completed in the window x 800
/ window seconds; nn_positions_per_s = positions the engines evaluated.  The
reference arm runs the same search with the reference's NNEvaluator over the
oracle engine on one core, as the reference's Eigen backend runs; no search
completes in a bounded window there, so its value is leaf evaluations/s
(one per simulation that reaches a non-terminal leaf).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (board, filters, blocks, batch per GPU, max random moves)
    "b19c128x10_bs512": (19, 128, 10, 512, 250),
    "b19c256x20_bs1024": (19, 256, 20, 1024, 250),
    "b9c128x10_bs256": (9, 128, 10, 256, 60),
    "b9c64x6_bs16": (9, 64, 6, 16, 60),
}
SELFPLAY_WORKLOADS = {
    # name: (board, filters, blocks, game workers, search threads per search,
    #        simulations per move, max batch per evaluator)
    "selfplay_b19c128x10": (19, 128, 10, 64, 16, 800, 512),
    "selfplay_b19c128x10_fast": (19, 128, 10, 64, 16, 800, 512),
    "selfplay_b19c128x10_grouped": (19, 128, 10, 64, 16, 800, 512),
}


def selfplay_search(wl):
    for s in ("fast", "grouped"):
        if wl.endswith("_" + s):
            return s
    return "reference"
DEFAULT_WORKLOAD = "b19c128x10_bs512"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def trunk_flops_per_position(board, filters, blocks, inputs=17):
    """Algorithmic FLOPs of the trunk's 3x3 convolutions for one position:
    board pixels only and the 17 real input planes (the frame rows and the
    zero-padded input channels the kernels also multiply are not counted)."""
    hw = board * board
    c = filters
    return 2 * hw * (9 * inputs * c + blocks * 2 * 9 * c * c)


def flops_per_position(board, filters, blocks, inputs=17, hidden=64):
    """Algorithmic FLOPs of one forward pass (2 per multiply-add)."""
    hw = board * board
    a = hw + 1
    c = filters
    heads = 2 * hw * 3 * c + 2 * 2 * hw * a + 2 * hw * hidden + 2 * hidden
    return trunk_flops_per_position(board, filters, blocks, inputs) + heads


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS, bf16_tflops_sustained=FALLBACK_PEAKS["bf16_tflops"]), "fallback"


def profiled_traffic(workload):
    """DRAM bytes per trunk launch from the committed ncu summary, if any."""
    import glob
    for p in sorted(glob.glob(os.path.join(ROOT, "profiles", f"trunk_*_{workload}.md"))):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.rows = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, nm in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


def torch_cpu_baseline(sd, x, target_s=6.0):
    """A torch restatement of the reference network (scripts/model.py,
    oracle/torch_net.py) on all host cores over a bounded sample of the
    workload, at up to the workload's batch per call."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    from torch_net import TorchNet

    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        net = TorchNet(sd)
        probe = min(len(x), 8)
        net.forward(x[:probe])  # first call: thread pool and allocator warm-up
        t0 = time.perf_counter()
        net.forward(x[:probe])
        per_pos = (time.perf_counter() - t0) / probe
        sample = max(probe, min(len(x), int(target_s / max(per_pos, 1e-9))))
        t0 = time.perf_counter()
        net.forward(x[:sample])
        dt = time.perf_counter() - t0
    finally:
        torch.set_num_threads(prev)
    cpu = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((l.split(":", 1)[1].strip() for l in f if l.startswith("model name")), "")
    except OSError:
        pass
    return {"value": sample / dt, "unit": "positions/s", "cores": threads, "kind": "port",
            "cpu": cpu, "torch": torch.__version__,
            "sample": f"{sample} positions of the same workload in one batch; torch fp32 "
                      f"restatement of scripts/model.py (eval mode) on {threads} threads "
                      f"({dt:.1f} s)"}


def cpu_baseline(sd, x, target_s=12.0):
    """The oracle on all host cores over a bounded sample of the workload
    (about target_s seconds of wall time), with the torch-CPU figure beside
    it."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    threads = os.cpu_count() or 1
    orc = oracle.EigenOracle(sd)
    t0 = time.perf_counter()
    orc.predict_batch(x[:1], oracle.CANONICAL, threads=1)
    per_pos = time.perf_counter() - t0
    sample = int(target_s / max(per_pos, 1e-9)) * threads
    sample = max(min(threads, len(x)), min(sample, len(x)))
    t0 = time.perf_counter()
    orc.predict_batch(x[:sample], oracle.CANONICAL, threads=threads)
    dt = time.perf_counter() - t0
    out = {"value": sample / dt, "unit": "positions/s", "cores": threads, "kind": "port",
           "sample": f"{sample} positions of the same workload; oracle C restatement of "
                     f"src/eigen_engine.cpp on {threads} threads ({dt:.1f} s)",
           "one_core_equivalent": sample / dt / threads}
    try:
        out["torch_cpu"] = torch_cpu_baseline(sd, x)
    except Exception as ex:  # reported, never fatal to the GPU line
        out["torch_cpu"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
    return out


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Ranks:
    """Barrier and max-over-ranks for the per-rank replicas (one process per
    GPU launched by torchrun).  No collective touches the data path: NCCL
    (or gloo on CPU) only carries these scalars."""

    def __init__(self, backend="nccl", device=None, timeout_s=120):
        self.world, self.rank, self.local = dist_setup()
        self.pg = None
        self.device = device
        if self.world > 1:
            import datetime
            import torch.distributed as dist

            kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl" and device is not None:
                kw["device_id"] = device
            dist.init_process_group(backend, **kw)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, v):
        if self.pg is None:
            return float(v)
        import torch

        t = torch.tensor([float(v)], dtype=torch.float64,
                         device=self.device if self.device is not None else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.barrier()
            self.pg.destroy_process_group()
            self.pg = None


def aggregate_rate(world, per_rank_units, steps, max_seconds):
    """Whole-job units per second: every rank processes per_rank_units per
    step, the job takes the slowest rank's time."""
    return world * per_rank_units * steps / max_seconds


def run_reference(args, wl):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    board, filters, blocks, batch, max_moves = WORKLOADS[wl]
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from alphazero_b200 import weights  # seeded numpy weights (no native code)

    sd = weights.make_state_dict(board, filters, blocks, seed=0, variant="init")
    # the reference's own src/game.cpp generates the positions (bit-identical
    # to the product's generator; the reference arm maps no product library)
    x = oracle.ref_random_positions(board, batch, 1000, max_moves)
    threads = os.cpu_count() or 1
    orc = oracle.EigenOracle(sd)
    t0 = time.perf_counter()
    orc.predict_batch(x[:1], oracle.CANONICAL, threads=1)
    per_pos = time.perf_counter() - t0
    # each step: a bounded sample (about 0.5 s of work on all threads)
    sample = max(1, min(batch, int(0.5 * threads / max(per_pos, 1e-9))))
    for _ in range(args.warmup):
        orc.predict_batch(x[:sample], oracle.CANONICAL, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.predict_batch(x[:sample], oracle.CANONICAL, threads=threads)
    dt = time.perf_counter() - t0
    v = sample * args.steps / dt
    line = {
        "impl": "reference", "metric": metric_name(wl), "value": v, "unit": "positions/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(wl),
        "cpu_baseline": {"value": v, "unit": "positions/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} positions per step of the same workload; oracle C "
                                   "restatement of src/eigen_engine.cpp (Eigen3 is absent, so the "
                                   "reference engine itself does not compile)"},
        "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def metric_name(wl):
    board, filters, blocks, batch, _ = WORKLOADS[wl]
    return f"positions/sec ({board}x{board} b{blocks}c{filters}, batch {batch} per GPU)"


def workload_config(wl):
    board, filters, blocks, batch, max_moves = WORKLOADS[wl]
    return {"workload": f"predict_batch {board}x{board} b{blocks}c{filters} batch {batch} per GPU",
            "board": board, "filters": filters, "blocks": blocks, "batch_per_gpu": batch,
            "positions": f"seeded random playouts of 0-{max_moves} legal moves",
            "weights": "seeded random init (export_onnx --init distributions)",
            "l2": "flushed by a 256 MB write before each timed step",
            "parallelism": "replicas; positions sharded per GPU, no collective"}


def trunk_kernel_label(filters, n_convs, trunk_launches):
    """Which kernel runs the trunk on this path, and in how many launches."""
    if filters == 128 and trunk_launches < n_convs:
        return (f"trunk: all {n_convs} 3x3 conv layers, conv3x3_pix_kernel, "
                f"{trunk_launches} persistent launch{'es' if trunk_launches > 1 else ''}")
    kern = "conv3x3_pix_kernel" if filters == 128 else "conv3x3_tc_kernel"
    return f"trunk: all {n_convs} 3x3 conv layers, {kern}, one launch per layer"


def measure_predict(wl, args, ranks, world, rank, local, planes_e2e=True):
    """positions/s (device-resident and end to end) and the trunk roofline
    of workload wl on this rank's GPU; every rank takes the same collective
    steps.  Returns the fields of a bench line (rank 0's view)."""
    import torch

    board, filters, blocks, batch, max_moves = WORKLOADS[wl]
    hw = board * board
    actions = hw + 1
    n_convs = 1 + 2 * blocks
    from alphazero_b200 import host_lib, weights
    from alphazero_b200.engine import CudaEngine, pack_states

    sd = weights.make_state_dict(board, filters, blocks, seed=0, variant="init")
    tmp = tempfile.mkdtemp(prefix="mgb_bench_")
    model = weights.write_onnx(os.path.join(tmp, "model.onnx"), sd)
    eng = CudaEngine(local, precision="bf16", max_batch=batch)
    eng.load_model(model)
    os.remove(model)
    os.rmdir(tmp)
    x = host_lib.random_positions(board, batch, 1000 + rank, max_moves)

    stream = torch.cuda.ExternalStream(eng.stream_handle())
    d_x = torch.from_numpy(x).cuda()
    d_p = torch.empty((batch, actions), device="cuda")
    d_v = torch.empty((batch,), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def barrier():
        ranks.barrier()
        torch.cuda.synchronize()

    # ---- value: device-resident inputs, L2 flushed before each step ----
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            flush.zero_()
            eng.forward_device(d_x.data_ptr(), batch, d_p.data_ptr(), d_v.data_ptr(), None)
    eng.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.zero_()
                starts[i].record(stream)
                eng.forward_device(d_x.data_ptr(), batch, d_p.data_ptr(), d_v.data_ptr(), None)
                ends[i].record(stream)
        eng.synchronize()
    barrier()
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    dev_ms = ranks.max(dev_ms)
    value = aggregate_rate(world, batch, args.steps, dev_ms / 1e3)
    per_forward = eng.launches_per_forward(batch)
    launches = per_forward * args.steps

    # ---- e2e: host API, pinned inputs and outputs, H2D + forward + D2H per
    # step, in the bit-packed wire format (and, for comparison, fp32 planes)
    words = eng.words_per_position()
    bits = torch.from_numpy(pack_states(x).view(np.int32)).pin_memory().numpy().view(np.uint32)
    outs = (torch.empty((batch, actions)).pin_memory().numpy(), torch.empty((batch,)).pin_memory().numpy())

    def e2e_loop(step):
        for _ in range(args.warmup):
            step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        dt = time.perf_counter() - t0
        barrier()
        return aggregate_rate(world, batch, args.steps, ranks.max(dt))

    e2e_sync = e2e_loop(lambda: eng.forward_packed(bits, batch, out=outs))

    # The same through the submission API the batching server uses
    # (mg_submit_packed / mg_wait_submitted): each step still copies its
    # bit-packed inputs from pinned host memory and its policy and value back
    # into pinned host memory, but step k+1's copies and launch are queued
    # while step k computes (two steps in flight, two sets of pinned buffers).
    pin_bits = [torch.from_numpy(pack_states(x).view(np.int32)).pin_memory().numpy().view(np.uint32)
                for _ in range(2)]
    pin_out = [(torch.empty((batch, actions)).pin_memory().numpy(),
                torch.empty((batch,)).pin_memory().numpy()) for _ in range(2)]
    pending = []

    def submitted_step():
        k = len(pending)
        b = k & 1
        pending.append(eng.submit_packed(pin_bits[b], batch, pin_out[b][0], pin_out[b][1]))
        if len(pending) >= 2:
            eng.wait_submitted(pending[-2])

    def e2e_submitted():
        pending.clear()
        for _ in range(args.warmup):
            submitted_step()
        eng.wait_submitted(pending[-1])
        barrier()
        pending.clear()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            submitted_step()
        eng.wait_submitted(pending[-1])  # the last step's results are in host memory
        dt = time.perf_counter() - t0
        barrier()
        return aggregate_rate(world, batch, args.steps, ranks.max(dt))

    e2e = e2e_submitted()
    e2e_planes = None
    if planes_e2e:
        xin = torch.from_numpy(x).pin_memory().numpy()
        e2e_planes = e2e_loop(lambda: eng.forward(xin, want_logits=False))

    # ---- roofline: the dominant kernel, the trunk (every 3x3 conv layer),
    # timed alone on the engine's stream ----
    reps = 10
    eng.forward_device(d_x.data_ptr(), batch, d_p.data_ptr(), d_v.data_ptr(), None)
    eng.launch_trunk(batch, 2)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    eng.launch_trunk(batch, reps)
    c1.record(stream)
    eng.synchronize()
    trunk_ms = ranks.max(c0.elapsed_time(c1) / reps)
    eng.close()
    del d_x, d_p, d_v, flush
    torch.cuda.empty_cache()

    trunk_flops = float(batch) * trunk_flops_per_position(board, filters, blocks)
    peaks, peak_src = load_peaks()
    achieved = trunk_flops / (trunk_ms / 1e3) / 1e12
    trunk_launches = per_forward - 3  # staging, FC, softmax/tanh finish
    out = {
        "value": value, "ms_per_step": dev_ms / args.steps,
        "e2e": {"value": e2e, "unit": "positions/s",
                "h2d_bytes_per_step": world * batch * words * 4,
                "d2h_bytes_per_step": world * batch * (actions + 1) * 4,
                "api": "mg_submit_packed / mg_wait_submitted (bit-packed planes, pinned host "
                       "buffers; two steps in flight, as the batching server runs)"},
        "e2e_sync": {"value": e2e_sync, "unit": "positions/s",
                     "h2d_bytes_per_step": world * batch * words * 4,
                     "d2h_bytes_per_step": world * batch * (actions + 1) * 4,
                     "api": "mg_forward_packed (bit-packed planes, pinned host buffers; one "
                            "synchronous call per step)"},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": profiled_traffic(wl),
                     "kernel": trunk_kernel_label(filters, n_convs, trunk_launches),
                     "flops_per_launch": trunk_flops, "launch_ms": trunk_ms,
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json bf16_tflops, burst)",
                     "peak_sustained": peaks["bf16_tflops_sustained"],
                     "frac_sustained": achieved / peaks["bf16_tflops_sustained"],
                     "timed_launches_ms": trunk_ms * reps},
        "tflops_whole_forward": value * flops_per_position(board, filters, blocks) / 1e12,
        "clocks": clocks.summary(),
    }
    if e2e_planes is not None:
        out["e2e_fp32_planes"] = {"value": e2e_planes, "unit": "positions/s",
                                  "h2d_bytes_per_step": world * batch * 17 * hw * 4,
                                  "d2h_bytes_per_step": world * batch * (actions + 1) * 4,
                                  "api": "mg_forward (fp32 planes, pinned input)"}
    return out, sd, x


# The other predict_batch configurations reported beside the default one.
EXTRA_CONFIGS = ("b19c256x20_bs1024", "b9c128x10_bs256", "b9c64x6_bs16")


def selfplay_records(world, args):
    """Self-play visits/s over all `world` GPUs, FastSearch and the
    reference's own search, each for a bounded window (rank 0 only)."""
    from alphazero_b200 import build

    if not os.path.exists(build.SELFPLAY_BIN):
        return {"unavailable": "selfplay_cuda was not built (the reference tree's src/mcts.cpp is "
                               "needed at build time)"}
    recs = {}
    with tempfile.TemporaryDirectory(prefix="mgb_selfplay_") as tmp:
        model = selfplay_model("selfplay_b19c128x10", tmp)
        for search, wl in (("fast", "selfplay_b19c128x10_fast"), ("grouped", "selfplay_b19c128x10_grouped"),
                           ("reference", "selfplay_b19c128x10")):
            with ClockSampler(0) as clocks:
                out = run_selfplay_binary(build.SELFPLAY_BIN, model, wl, args, world, search=search,
                                          window=(args.selfplay_warmup, args.selfplay_seconds))
            out["clocks_gpu0"] = clocks.summary()
            out["metric"] = "MCTS visits/s"
            out["config"] = selfplay_config(wl)
            recs[search] = out
    return recs


def run_b200(args, wl):
    import torch

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    ranks = Ranks("nccl", device=torch.device("cuda", local))
    board, filters, blocks, batch, max_moves = WORKLOADS[wl]

    m, sd, x = measure_predict(wl, args, ranks, world, rank, local)
    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(sd, x)
    configs = None
    if world == 1 and wl == DEFAULT_WORKLOAD and not args.no_extras:
        configs = {}
        for cw in EXTRA_CONFIGS:
            cm, _, _ = measure_predict(cw, args, ranks, world, rank, local, planes_e2e=False)
            cm.update(metric=metric_name(cw), unit="positions/s", config=workload_config(cw))
            configs[cw] = cm
    ranks.close()
    if rank != 0:
        return
    line = {
        "metric": metric_name(wl), "value": m["value"], "unit": "positions/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(wl),
    }
    line.update({k: v for k, v in m.items() if k not in ("value", "ms_per_step")})
    if base is not None:
        line["cpu_baseline"] = base
    if configs is not None:
        line["configs"] = configs
    if wl == DEFAULT_WORKLOAD and not args.no_extras:
        # The metric's second half: MCTS visits/s over all N GPUs (the
        # per-rank engines are closed; the other ranks have exited).
        line["selfplay"] = selfplay_records(world, args)
    print(json.dumps(line), flush=True)


def selfplay_config(wl):
    board, filters, blocks, workers, threads, sims, max_batch = SELFPLAY_WORKLOADS[wl]
    return {"workload": f"self-play {board}x{board} b{blocks}c{filters}: {workers} game workers x "
                        f"{threads} search threads, {sims} simulations per move, max batch {max_batch}",
            "board": board, "filters": filters, "blocks": blocks, "workers": workers,
            "search_threads": threads, "simulations": sims, "max_batch": max_batch,
            "search": {"fast": "FastSearch (the reference's MCTS algorithm, own implementation; "
                               f"{threads} search threads per game worker)",
                       "grouped": "FastSearch, grouped mode (the reference's MCTS algorithm; each "
                                  f"worker's {threads} concurrent playouts as rounds on its own "
                                  "thread, a round's leaves evaluated as one group)",
                       "reference": "reference src/mcts.cpp compiled unmodified"}[selfplay_search(wl)],
            "weights": "seeded random init (export_onnx --init distributions)",
            "parallelism": "one batching server + engine per GPU, search threads round-robin, "
                           "weights replicated, no collective"}


def selfplay_window(args):
    """(warm-up seconds, measured seconds) for --warmup / --steps."""
    return max(6.0, 2.0 * args.warmup), max(10.0, float(args.steps))


def run_selfplay_binary(exe, model, wl, args, gpus, search=None, window=None):
    board, filters, blocks, workers, threads, sims, max_batch = SELFPLAY_WORKLOADS[wl]
    warm, window = selfplay_window(args) if window is None else window
    cmd = [exe, "--model", model, "--gpus", str(gpus), "--workers", str(workers),
           "--search-threads", str(threads), "--sims", str(sims), "--max-batch", str(max_batch),
           "--warmup-seconds", str(warm), "--seconds", str(window)]
    if search is not None:
        cmd += ["--search", search]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=warm + window + 600)
    if r.returncode != 0:
        raise RuntimeError(f"{os.path.basename(exe)} failed ({r.returncode}): {r.stderr[-2000:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def selfplay_model(wl, tmp):
    """Writes the workload's seeded network as ONNX into directory tmp."""
    from alphazero_b200 import weights

    board, filters, blocks = SELFPLAY_WORKLOADS[wl][:3]
    sd = weights.make_state_dict(board, filters, blocks, seed=0, variant="init")
    return weights.write_onnx(os.path.join(tmp, "model.onnx"), sd)


def oracle_selfplay(wl, args):
    """The reference arm / CPU baseline of the self-play workload."""
    exe = os.path.join(ROOT, "oracle", "_ref", "selfplay_oracle")
    if not os.path.exists(exe):
        return None, "oracle/_ref/selfplay_oracle was not built (no reference tree at build time)"
    with tempfile.TemporaryDirectory(prefix="mgb_selfplay_") as tmp:
        out = run_selfplay_binary(exe, selfplay_model(wl, tmp), wl, args, 0)
    return out, None


def run_selfplay(args, wl):
    world, rank, _ = dist_setup()
    ranks = Ranks("gloo", timeout_s=1800)
    board, filters, blocks, workers, threads, sims, max_batch = SELFPLAY_WORKLOADS[wl]
    line = None
    if rank == 0:
        metric = (f"MCTS visits/sec (self-play {board}x{board} b{blocks}c{filters}, {workers} workers x "
                  f"{threads} search threads, {sims} sims"
                  + {"fast": ", FastSearch)", "grouped": ", FastSearch grouped)",
                     "reference": ")"}[selfplay_search(wl)])
        if args.impl == "reference":
            out, why = oracle_selfplay(wl, args)
            if out is None:
                line = {"impl": "reference", "unavailable": why}
            else:
                v = out["nn_positions_per_s"]
                line = {"impl": "reference", "metric": metric, "value": v, "unit": "visits/s",
                        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                        "ms_per_step": 1000.0, "higher_is_better": True, "scaling": "strong",
                        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                        "config": selfplay_config(wl), "selfplay": out,
                        "cpu_baseline": {"value": v, "unit": "visits/s", "cores": 1, "kind": "port",
                                         "sample": f"{out['seconds']:.0f} s window of the same "
                                                   "self-play; NN on one core like the reference's "
                                                   "Eigen backend; leaf evaluations/s"},
                        "e2e": {"value": v, "unit": "visits/s", "h2d_bytes_per_step": 0,
                                "d2h_bytes_per_step": 0}}
        else:
            from alphazero_b200 import build

            if not os.path.exists(build.SELFPLAY_BIN):
                raise SystemExit("selfplay_cuda was not built: the reference tree's src/mcts.cpp "
                                 "is needed at build time")
            gpus = max(args.gpus, world)
            with ClockSampler(0) as clocks:
                with tempfile.TemporaryDirectory(prefix="mgb_selfplay_") as tmp:
                    out = run_selfplay_binary(build.SELFPLAY_BIN, selfplay_model(wl, tmp), wl, args,
                                              gpus, search=selfplay_search(wl))
            base = None
            if gpus == 1 and not args.no_cpu_baseline:
                base_out, _ = oracle_selfplay(wl, args)
                if base_out is not None:
                    base = {"value": base_out["nn_positions_per_s"], "unit": "visits/s", "cores": 1,
                            "kind": "port",
                            "sample": f"{base_out['seconds']:.0f} s window of the same self-play; "
                                      "the reference's NNEvaluator over the oracle engine on one "
                                      "core; leaf evaluations/s"}
            words = (17 * board * board + 31) // 32
            pps = out["nn_positions_per_s"]
            line = {"metric": metric, "value": out["visits_per_s"], "unit": "visits/s",
                    "n_gpus": gpus, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": 1000.0 * out["seconds"] / max(1, args.steps),
                    "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                    "dtype": "bf16", "data": "synthetic", "config": selfplay_config(wl),
                    "selfplay": out,
                    "e2e": {"value": out["visits_per_s"], "unit": "visits/s",
                            "h2d_bytes_per_step": int(pps * words * 4),
                            "d2h_bytes_per_step": int(pps * (board * board + 2) * 4),
                            "api": "reference MCTS -> ShardedEvaluator -> CudaEngine::predict_raw "
                                   "(bit-packed planes); bytes per one-second step"},
                    "gpu_launches": out["gpu_launches"],
                    "clocks": clocks.summary()}
            if base is not None:
                line["cpu_baseline"] = base
    ranks.close()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD,
                    choices=sorted(WORKLOADS) + sorted(SELFPLAY_WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default workload: skip the other configurations and self-play")
    ap.add_argument("--selfplay-warmup", type=float, default=4.0,
                    help="self-play record: warm-up seconds per search")
    ap.add_argument("--selfplay-seconds", type=float, default=8.0,
                    help="self-play record: measured seconds per search")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    if args.workload in SELFPLAY_WORKLOADS:
        run_selfplay(args, args.workload)
    elif args.impl == "reference":
        run_reference(args, args.workload)
    else:
        run_b200(args, args.workload)


if __name__ == "__main__":
    main()
