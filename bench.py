#!/usr/bin/env python
"""Benchmark: Local-AR + sampling frames/s per GPU and per box, p50/p99
per-frame latency.

Workloads (synthetic, seeded; random-init weights ~N(0, 0.02) of the
NeMo-default Local AR shape: in-projection 768->256, 1 layer, d=256, 4 heads,
FFN 1024, 16 heads 256->2024, 16 tables 2024x768):

* ``config4`` (default, the scaling metric): 1024 sessions x CFG pair sharded
  evenly over the ranks (1024/N per GPU, no collective), 500 frames; 5% of the
  sessions are forced to EOS (``finished``) at a frame drawn from U[50, 500]
  and masked out afterwards; until then EOS is forbidden (``unfinished``);
  ``forbid_eos`` holds for the first 2 decoder steps.  A bench *step* is the
  whole 500-frame run of this rank's sessions; ``value`` = all ranks' session
  frames / max-over-ranks time.
* ``config3``: 64 sessions per GPU, EOS forced at U[200, 600], 600 frames.
* ``config2`` latency (rank 0, N=1 only, also reported inside every N=1 line):
  one session, CFG, seed 1234, 1000 frames with new hidden states, each frame
  one CUDA-graph launch of the frame; p50/p99 over frames by CUDA events.

Also at N=1: the alignment gate (the controller step plus the Local AR's
EOS inputs, once per decoder step) for the config-4 sessions of one GPU, with
the reference's own host controller timed beside it; and the Main Decoder
step for config 5's 256 sessions per GPU (``main_decoder_step``), with the
CPU restatement timed beside it; and config 5's full per-frame loop
(``config5_loop``: decoder step -> alignment gate -> Local AR frame for 256
sessions x 1024 frames, all on the device).

A "frame" is one session's 16-position Local AR step (one decoder hidden in,
16 codec tokens = 2 codec frames x 8 codebooks out).

``--impl reference`` times the reference's path as its CPU oracle (the
PyTorch restatement of the NeMo forward + the C restatement of the sampling
plugin, bit-exact with the reference on its golden vectors) on the host cores,
on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from magpie_tts_rt_b200.model import EMBED, SHAPE_BASELINE, SHAPE_SOFIA, make_weights  # noqa: E402

METRIC = "Local-AR+sampling frames/sec per GPU and box (1/2/4/8); p50 per-frame us"
PATH_NAMES = {1: "phase kernels", 2: "fused cluster kernel", 3: "tile kernel", 4: "pair kernel",
              5: "split kernel x1", 6: "split kernel x2", 7: "split kernel x4", 8: "split kernel x8",
              9: "split kernel x2, 32-row tiles", 10: "quad kernel", 11: "octo kernel"}
# DRAM bytes per launch of the frame kernel, measured by ncu (path, sessions per GPU)
TRAFFIC = {("tile kernel", 1024): 27.64e6, ("pair kernel", 1024): 27.71e6, ("split kernel x4", 256): 23.12e6,
           ("split kernel x8", 64): 20.56e6, ("fused cluster kernel", 1): 18.76e6}
WORKLOADS = {
    "config4": dict(total_streams=1024, frames=500, eos_frac=0.05, eos_lo=50, eos_hi=500, weak=False),
    "config3": dict(per_gpu_streams=64, frames=600, eos_frac=1.0, eos_lo=200, eos_hi=600, weak=True),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4", choices=list(WORKLOADS) + ["config5"],
                    help="config5: the full per-frame loop, 256 sessions per GPU on every rank (weak scaling)")
    ap.add_argument("--frames", type=int, default=None, help="override frames per step (profiling)")
    ap.add_argument("--sessions", type=int, default=None,
                    help="override sessions per GPU (profiling a smaller per-GPU batch, e.g. 256 = config 4 at 4 GPUs)")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--path", type=int, default=0, help="frame path for the config-4 workload (0: AUTO)")
    ap.add_argument("--main-decoder-only", action="store_true",
                    help="run only the Main Decoder step measurement and print its object (profiling)")
    ap.add_argument("--md-sessions", type=int, default=256, help="Main Decoder sessions per GPU (config 5: 256)")
    ap.add_argument("--md-steps", type=int, default=20)
    ap.add_argument("--no-loop", action="store_true", help="skip the config-5 loop measurement")
    ap.add_argument("--loop-only", action="store_true", help="run only the config-5 loop and print its object")
    ap.add_argument("--loop-steps", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--latency-only", action="store_true",
                    help="run only the config-2 latency measurement (with its phase breakdown) and print it")
    ap.add_argument("--r-shape-only", action="store_true",
                    help="run only the d=768 / 2-layer Local AR frame measurement and print its object")
    ap.add_argument("--r-sessions", type=int, nargs="*", default=None)
    ap.add_argument("--phase-trace", default=None, metavar="PATH:SESSIONS",
                    help="print the per-position phase breakdown of the pair (4), split (5-9), quad (10) or octo (11) "
                         "kernel and exit")
    ap.add_argument("--eos-only", action="store_true",
                    help="run only the EOS-projection measurement and print its object (profiling)")
    ap.add_argument("--eos-sessions", type=int, nargs="*", default=None,
                    help="EOS-enabled sessions per measured batch (default 64 and 1024)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def rank_streams(cfg, world, rank):
    if cfg["weak"]:
        n = cfg["per_gpu_streams"]
        return n, rank * n, n * world
    total = cfg["total_streams"]
    n = total // world
    return n, rank * n, total


def eos_schedule(cfg, total, frames, seed=2024):
    """eos_frame[s] for every session of the job (same on all ranks)."""
    rng = np.random.default_rng(seed)
    eos = np.full(total, frames + 1, np.int64)  # never within the run
    k = int(round(cfg["eos_frac"] * total))
    chosen = rng.choice(total, k, replace=False) if k < total else np.arange(total)
    eos[chosen] = rng.integers(cfg["eos_lo"], cfg["eos_hi"] + 1, k)
    return eos


def flag_tables(eos, frames):
    f = np.arange(frames)[:, None]
    e = eos[None, :]
    active = f <= e
    unfinished = f < e
    finished = f == e
    forbid = np.broadcast_to(f < 2, active.shape)
    return active, unfinished, finished, forbid


class ClockSampler:
    """nvidia-smi clocks / throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            p = json.load(fh)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------

def run_ours(args, world, rank, local):
    from magpie_tts_rt_b200 import _lib as L
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch

    cfg = dict(WORKLOADS[args.workload])
    if args.sessions:
        cfg.update(weak=True, per_gpu_streams=args.sessions)
    frames = args.frames or cfg["frames"]
    n, first, total = rank_streams(cfg, world, rank)
    dev = torch.device("cuda", local)
    w = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline")
    eng = LocalArEngine(w, max_streams=n, device=dev, path=args.path)
    eos = eos_schedule(cfg, total, cfg["frames"])[first:first + n]
    act, unf, fin, forb = flag_tables(eos, frames)
    frames_per_step_local = int(act.sum())
    T = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(dev)
    d_act, d_unf, d_fin, d_forb = (T(x, torch.bool) for x in (act, unf, fin, forb))
    seeds = T(np.arange(first, first + n), torch.int64)

    # inputs: new N(0,1) hidden states per frame per session (pinned host, seeded)
    g = torch.Generator().manual_seed(1000 + rank)
    host_hidden = torch.empty(frames, n, 2, EMBED, dtype=torch.bfloat16).pin_memory()
    chunk = max(1, frames // 16)
    for f0 in range(0, frames, chunk):
        f1 = min(frames, f0 + chunk)
        host_hidden[f0:f1].copy_(torch.randn(f1 - f0, n, 2, EMBED, generator=g))
    dev_hidden = host_hidden.to(dev)
    # two staging buffers: frame f+1's host->device copy (copy stream) overlaps frame f
    stages = [torch.empty(n, 2, EMBED, dtype=torch.bfloat16, device=dev) for _ in range(2)]

    counters = torch.zeros(n, dtype=torch.int64, device=dev)
    codec = torch.zeros(frames, n, 8, 2, dtype=torch.int64, device=dev)
    invalid = torch.zeros(frames, n, dtype=torch.int32, device=dev)
    end = torch.zeros(frames, n, dtype=torch.int32, device=dev)
    nxt = torch.zeros(n, EMBED, dtype=torch.bfloat16, device=dev)
    host_codec = torch.empty(frames, n, 8, 2, dtype=torch.int64).pin_memory()
    host_end = torch.empty(frames, n, dtype=torch.int32).pin_memory()

    def batches(hidden_of):
        out = []
        for f in range(frames):
            b = StreamBatch(decoder_hidden=hidden_of(f), unfinished=d_unf[f], finished=d_fin[f],
                            forbid_eos=d_forb[f], rng_seed=seeds, rng_counter=counters, codec_tokens=codec[f],
                            invalid_rows=invalid[f], end_frame_index=end[f], next_embedding=nxt, active=d_act[f])
            out.append(b.c_struct())
        return out

    resident = batches(lambda f: dev_hidden[f])
    staged = batches(lambda f: stages[f % 2])
    shape, weights_c, sampling = eng._shape, eng._w, eng._sampling
    ws, ws_bytes = ctypes.c_void_p(eng.workspace.data_ptr()), eng.workspace.numel()
    launch = L.lib.mtt_b200_launch_local_ar_frame

    def frame_call(cb, stream_handle):
        st = launch(ctypes.byref(shape), ctypes.byref(weights_c), ctypes.byref(sampling), ctypes.byref(cb), ws,
                    ws_bytes, stream_handle)
        if st != 0:
            raise RuntimeError(f"frame launch failed: {st}")

    stream = torch.cuda.current_stream(dev)
    sh = ctypes.c_void_p(stream.cuda_stream)

    def step_resident():
        counters.zero_()
        for f in range(frames):
            frame_call(resident[f], sh)

    copy_stream = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def step_e2e():
        # every step copies each frame's hidden states from pinned host memory and reads the
        # codec tokens / end-frame indices back; the copy of frame f+1 overlaps frame f
        counters.zero_()
        copy_stream.wait_stream(stream)  # the copies start inside the timed region

        def stage_copy(f):
            with torch.cuda.stream(copy_stream):
                if f >= 2:
                    copy_stream.wait_event(used[f % 2])  # frame f-2 has read this buffer
                stages[f % 2].copy_(host_hidden[f], non_blocking=True)
                copied[f % 2].record(copy_stream)

        stage_copy(0)
        for f in range(frames):
            if f + 1 < frames:
                stage_copy(f + 1)
            stream.wait_event(copied[f % 2])
            frame_call(staged[f], sh)
            used[f % 2].record(stream)
        host_codec.copy_(codec, non_blocking=True)
        host_end.copy_(end, non_blocking=True)

    def timed(fn, k):
        barrier(world)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        return e0.elapsed_time(e1) / 1000.0

    for _ in range(args.warmup):
        step_resident()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    t_local = timed(step_resident, args.steps)
    clk = clocks.stop()
    t = max_over_ranks(t_local, world)
    frames_total = sum_over_ranks(frames_per_step_local * args.steps, world)
    value = frames_total / t

    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    te_local = timed(step_e2e, args.steps)
    te = max_over_ranks(te_local, world)
    e2e_value = frames_total / te
    h2d = host_hidden[0].numel() * 2 * frames
    d2h = host_codec.numel() * 8 + host_end.numel() * 4

    # sanity: every session's final frame is valid and the forced-EOS sessions ended at frame 0
    bad = int((invalid.cpu().numpy()[act] != 0).sum())
    end_np = end.cpu().numpy()
    forced_ok = all(end_np[eos[s], s] == 0 for s in range(n) if eos[s] < frames)
    launches_per_frame = eng.launch_count(n)
    return dict(value=value, t=t, e2e=e2e_value, h2d=h2d, d2h=d2h, clocks=clk, n_local=n, total=total,
                path=PATH_NAMES.get(eng.path, str(eng.path)),
                frames=frames, frames_per_step=frames_total / args.steps, invalid=bad, forced_ok=forced_ok,
                launches=launches_per_frame * frames * args.steps, eng=eng, w=w)


def config3_measure(args, peaks):
    """Config 3 on one GPU: 64 sessions x CFG pair, per-session EOS forced at a
    frame U[200, 600] and finished sessions masked out of later frames, 600
    frames per step; frames/s resident and end to end, and the frame call's
    HBM and tensor fractions (algorithmic bytes: the 18.6 MB of weights read
    once per frame plus 31 KB per active session)."""
    import argparse
    a3 = argparse.Namespace(**{**vars(args), "workload": "config3", "sessions": None, "frames": None, "path": 0,
                               "steps": 2, "warmup": 3})
    r = run_ours(a3, 1, 0, 0)
    shape = SHAPE_BASELINE
    active_per_frame = r["frames_per_step"] / r["frames"]
    t_frame = r["t"] / a3.steps / r["frames"]
    bytes_ = shape.frame_weight_params() * 2 + active_per_frame * 31_000
    flops = active_per_frame * 2 * 2 * shape.macs_per_row()
    tensor_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    return {"workload": "config 3: 64 sessions x CFG pair, EOS forced at U[200,600], finished sessions masked, "
                        "600 frames", "frame_path": r["path"], "frames_per_s": r["value"], "e2e_frames_per_s": r["e2e"],
            "avg_frame_call_us": t_frame * 1e6, "hbm_frac": bytes_ / t_frame / 1e9 / peaks["hbm_gbs"],
            "tensor_frac": flops / t_frame / 1e12 / tensor_peak, "invalid_rows": r["invalid"],
            "forced_eos_ok": r["forced_ok"]}


def latency_config2(eng_w, dev, frames=1000, warm=20):
    """Config 2: B=1 CFG pair, seed 1234, new hidden each frame; one CUDA-graph
    launch per frame; per-frame device time by CUDA events."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    eng = LocalArEngine(eng_w, max_streams=1, device=dev)
    b = StreamBatch.allocate(1, device=dev)
    b.rng_seed.fill_(1234)
    b.unfinished.fill_(True)
    g = torch.Generator().manual_seed(77)
    hidden = torch.randn(frames + warm, 1, 2, EMBED, generator=g).to(torch.bfloat16).to(dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            eng.frame(b)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        eng.frame(b)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(frames)]
    with torch.cuda.stream(stream):
        for f in range(frames + warm):
            b.decoder_hidden.copy_(hidden[f])
            b.forbid_eos.fill_(f < 2)
            if f >= warm:
                ev[f - warm][0].record(stream)
            graph.replay()
            if f >= warm:
                ev[f - warm][1].record(stream)
    torch.cuda.synchronize(dev)
    us = np.array([a.elapsed_time(z) * 1000.0 for a, z in ev])
    inv = int(b.invalid_rows.item())
    del graph
    return {"workload": "config2: 1 session x CFG pair, seed 1234, 1000 frames, CUDA graph per frame",
            "frame_path": PATH_NAMES.get(eng.path, str(eng.path)),
            "p50_us": float(np.percentile(us, 50)), "p99_us": float(np.percentile(us, 99)),
            "mean_us": float(us.mean()), "frames": frames, "invalid": inv}


PHASE_STAMPS = ["x ready", "qkv + partial scores", "scores round", "attention", "attention round",
                "o-projection", "o round", "LN2 + FFN1", "FFN2 partials", "FFN2 partials round",
                "FFN2 sum round", "head", "logits round", "sampling", "token round"]


def latency_trace(eng_w, dev, frames=20):
    """Per-position phase breakdown of the config-2 frame (library trace hook
    mtt_b200_test_frame_trace): SM-clock stamps of the first CTA at 16 points
    of each position, averaged over `frames` frames, in microseconds at the
    clock measured over the frame (cycles / global-timer ns)."""
    from magpie_tts_rt_b200 import _lib as L
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    eng = LocalArEngine(eng_w, max_streams=1, device=dev)
    if PATH_NAMES.get(eng.path) != "fused cluster kernel":
        return None
    b = StreamBatch.allocate(1, device=dev)
    b.rng_seed.fill_(1234)
    b.unfinished.fill_(True)
    g = torch.Generator().manual_seed(78)
    stamps = torch.zeros(260, dtype=torch.int64, device=dev)
    per = []
    try:
        L.lib.mtt_b200_test_frame_trace(ctypes.c_void_p(stamps.data_ptr()))
        for f in range(frames + 3):
            b.decoder_hidden.copy_(torch.randn(1, 2, EMBED, generator=g).to(torch.bfloat16))
            eng.frame(b)
            torch.cuda.synchronize(dev)
            if f >= 3:
                per.append(stamps.cpu().numpy().copy())
    finally:
        L.lib.mtt_b200_test_frame_trace(None)
    a = np.stack(per).astype(np.float64)
    mhz = (a[:, 258] - a[:, 256]) / (a[:, 259] - a[:, 257]) * 1000.0
    pos = a[:, :256].reshape(frames, 16, 16)
    d = np.diff(pos, axis=2) / mhz[:, None, None]  # us between consecutive stamps
    per_pos = (pos[:, :, 15] - pos[:, :, 0]) / mhz[:, None]
    return {"sm_mhz": float(np.median(mhz)),
            "frame_us_in_kernel": float(np.median((a[:, 258] - a[:, 256]) / mhz)),
            "position_us_mean": float(per_pos[:, 1:].mean()), "position0_us": float(per_pos[:, 0].mean()),
            "phase_us_mean_p1_15": {k: float(d[:, 1:, i].mean()) for i, k in enumerate(PHASE_STAMPS)}}


QUAD_STAMPS = ["input rows", "q|k|v", "attention", "attention round", "o-projection + round", "LN2", "FFN1",
               "FFN2 partials", "FFN2 partials round", "FFN2 sum + x'' round", "head", "values round", "sampling",
               "token round", "next rows + LN1"]


def quad_trace(w, dev, path, n, frames=10):
    """Per-position phase breakdown of the pair (path 4), split (paths 5-9),
    quad (path 10) or octo (path 11) kernel at n sessions (library trace hook
    mtt_b200_test_frame_trace; the kernels stamp the same 16 points, the pair
    kernel's sampling phase including the next position's rows):
    SM-clock stamps of CTA 0 at 16 points of each position, averaged over
    positions 1..15 of `frames` frames, in microseconds at the clock measured
    over the frame."""
    from magpie_tts_rt_b200 import _lib as L
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    eng = LocalArEngine(w, max_streams=n, device=dev, path=path)
    b = StreamBatch.allocate(n, device=dev)
    b.rng_seed.copy_(torch.arange(n))
    b.unfinished.fill_(True)
    g = torch.Generator().manual_seed(78)
    stamps = torch.zeros(260, dtype=torch.int64, device=dev)
    per = []
    try:
        L.lib.mtt_b200_test_frame_trace(ctypes.c_void_p(stamps.data_ptr()))
        for f in range(frames + 3):
            b.decoder_hidden.copy_(torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16))
            eng.frame(b)
            torch.cuda.synchronize(dev)
            if f >= 3:
                per.append(stamps.cpu().numpy().copy())
    finally:
        L.lib.mtt_b200_test_frame_trace(None)
    a = np.stack(per).astype(np.float64)
    mhz = (a[:, 258] - a[:, 256]) / (a[:, 259] - a[:, 257]) * 1000.0
    pos = a[:, :256].reshape(frames, 16, 16)
    d = np.diff(pos, axis=2) / mhz[:, None, None]
    per_pos = (pos[:, :, 15] - pos[:, :, 0]) / mhz[:, None]
    return {"frame_path": PATH_NAMES.get(eng.path, str(eng.path)), "sessions": n, "sm_mhz": float(np.median(mhz)),
            "frame_us_in_kernel": float(np.median((a[:, 258] - a[:, 256]) / mhz)),
            "position_us_mean": float(per_pos[:, 1:].mean()),
            "phase_us_mean_p1_15": {k: float(d[:, 1:, i].mean()) for i, k in enumerate(QUAD_STAMPS)}}


def tensor_probe(dev):
    """The two measurements behind the frame kernels' shape (library hooks
    mtt_b200_test_umma_cycles / _dsmem_cycles): SM cycles of one tcgen05.mma
    (M = 128, K = 16) for each N, issued back to back on every SM, and the
    bytes per cycle an SM pushes into its 7 cluster peers' shared memory."""
    from magpie_tts_rt_b200 import _lib as L
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = {"umma_cycles_per_instruction": {}, "umma_mac_per_cycle_per_sm": {}}
    cyc = torch.zeros(1024, dtype=torch.int64, device=dev)
    n_mma = 2048
    for n in (16, 32, 48, 64, 96, 128, 256):
        if L.lib.mtt_b200_test_umma_cycles(n, 1, n_mma, sms, ctypes.c_void_p(cyc.data_ptr()), st) != 0:
            return None
        torch.cuda.synchronize(dev)
        c = cyc[:sms].cpu().numpy()
        per = float(np.median(c[c > 0])) / n_mma if (c > 0).any() else None
        out["umma_cycles_per_instruction"][n] = per
        out["umma_mac_per_cycle_per_sm"][n] = 128 * n * 16 / per if per else None
    rounds, clusters, bytes_ = 20, 16, 16384
    if L.lib.mtt_b200_test_dsmem_cycles(bytes_, rounds, clusters, ctypes.c_void_p(cyc.data_ptr()), st) != 0:
        return None
    torch.cuda.synchronize(dev)
    c = cyc[:8 * clusters].cpu().numpy()
    per_round = float(np.median(c[c > 0])) / rounds if (c > 0).any() else None
    out["dsmem_bulk_bytes_per_cycle_per_sm"] = 7 * bytes_ / per_round if per_round else None
    out["dsmem_note"] = "7 peers x 16 KB per round, rounds separated by cluster barriers, 8-CTA clusters"
    return out


def eos_measure(w, dev, peaks, sizes=(64, 1024), calls=20):
    """The frame's EOS projection (tcgen05 GEMM over the enabled sessions'
    rows, guided-logit reduction in the epilogue): frame calls with every
    session's EOS enabled minus the same calls with EOS disabled, CUDA events.
    Algorithmic work: 2 rows x 32,384 x 768 MAC per enabled session, and the
    49.7 MB final projection read once."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    out = {}
    stream = torch.cuda.Stream(dev)
    for n in sizes:
        eng = LocalArEngine(w, max_streams=n, device=dev)
        b = StreamBatch.allocate(n, device=dev)
        g = torch.Generator().manual_seed(n)
        b.decoder_hidden.copy_(torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16))
        b.rng_seed.copy_(torch.arange(n))
        times = {}
        for enabled in (False, True):
            b.unfinished.fill_(not enabled)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    eng.frame(b, stream=stream)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(calls):
                    eng.frame(b, stream=stream)
                e1.record(stream)
            torch.cuda.synchronize(dev)
            times[enabled] = e0.elapsed_time(e1) * 1000.0 / calls
        d_us = times[True] - times[False]
        macs = 2 * n * 32384 * 768
        tflops = 2 * macs / (d_us * 1e-6) / 1e12 if d_us > 0 else None
        gbs = (32384 * 768 * 2 + n * 2 * 768 * 2) / (d_us * 1e-6) / 1e9 if d_us > 0 else None
        tensor_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        out[str(n)] = {"frame_call_us_eos_enabled": times[True], "frame_call_us_eos_disabled": times[False],
                       "eos_projection_us": d_us, "tflops": tflops, "tensor_frac": tflops / tensor_peak if tflops else None,
                       "hbm_gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"] if gbs else None,
                       "frame_path": PATH_NAMES.get(eng.path, str(eng.path))}
    return out


def r_shape_measure(dev, peaks, sizes=(64, 1024), calls=10, seed=5):
    """The reference bundle's accepted Local AR shape (d=768, 2 layers, 12
    heads, FFN 3072, identity in-projection) through the frame entry point:
    its AUTO path is the phase kernels, whose layer GEMMs and 16 heads run on
    the tcgen05 GEMM (gemm_tc.cuh).  One frame call per step, CUDA events on
    the launching stream, eager and replayed from a CUDA graph.  Algorithmic
    work: 2 rows x macs_per_row() MAC per session per frame."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    w = make_weights(SHAPE_SOFIA, seed=seed, dtype=torch.bfloat16, profile="baseline")
    tensor_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    out = {"shape": "d=768, 2 layers, 12 heads, FFN 3072, 16 heads 768->2024, CFG pair, EOS enabled"}
    stream = torch.cuda.Stream(dev)
    for n in sizes:
        eng = LocalArEngine(w, max_streams=n, device=dev)
        b = StreamBatch.allocate(n, device=dev)
        g = torch.Generator().manual_seed(n)
        b.decoder_hidden.copy_(torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16))
        b.rng_seed.copy_(torch.arange(n))
        b.unfinished.fill_(True)
        res = {"frame_path": PATH_NAMES.get(eng.path, str(eng.path))}
        with torch.cuda.stream(stream):
            for _ in range(3):
                eng.frame(b, stream=stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(calls):
                eng.frame(b, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        t_eager = e0.elapsed_time(e1) * 1000.0 / calls
        t_graph = None
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                eng.frame(b, stream=stream)
            with torch.cuda.stream(stream):
                graph.replay()
                e0.record(stream)
                for _ in range(calls):
                    graph.replay()
                e1.record(stream)
            torch.cuda.synchronize(dev)
            t_graph = e0.elapsed_time(e1) * 1000.0 / calls
            del graph
        except RuntimeError as exc:  # capture refused: report the eager number alone
            res["graph_error"] = str(exc).splitlines()[0]
        inv = int(b.invalid_rows.count_nonzero().item())
        t = min(x for x in (t_eager, t_graph) if x is not None)
        flops = n * 2 * 2 * SHAPE_SOFIA.macs_per_row()
        tf = flops / (t * 1e-6) / 1e12
        res.update({"frame_call_us_eager": t_eager, "frame_call_us_graph": t_graph,
                    "frames_per_s": n / (t * 1e-6), "tflops": tf, "tensor_frac": tf / tensor_peak,
                    "algorithmic_flops_per_call": flops, "invalid_rows": inv,
                    "roofline": {"bound": "tensor", "kernel": "phase kernels (one frame call, CUDA graph)",
                                 "achieved": tf, "peak": tensor_peak, "unit": "TFLOP/s", "frac": tf / tensor_peak,
                                 "peak_kind": "measured sustained bf16", "traffic": None}})
        out[str(n)] = res
    return out


def frame_paths_measure(w, dev, peaks, sizes=(64, 128, 256, 512, 1024), calls=20,
                        paths=((10, "quad kernel"), (11, "octo kernel"), (0, "AUTO"))):
    """Frame-call time of the benchmark shape (config 4's flags at its first
    frames: every session unfinished, CFG pair) on the quad kernel (4-CTA
    cluster per 16 sessions) and the octo kernel (8-CTA cluster per 16
    sessions), explicit paths, next to the AUTO path, for the sessions per GPU
    that config 4 puts on 8, 4, 2 and 1 GPUs and config 3's 64 (the octo
    kernel up to 256 sessions).  CUDA events on the launching stream."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    tensor_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    stream = torch.cuda.Stream(dev)
    out = {"workload": "benchmark shape, CFG pair, all sessions unfinished, frame call timed alone"}
    for n in sizes:
        b = StreamBatch.allocate(n, device=dev)
        g = torch.Generator().manual_seed(n)
        b.decoder_hidden.copy_(torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16))
        b.rng_seed.copy_(torch.arange(n))
        b.unfinished.fill_(True)
        row = {}
        for path, name in paths:
            if path == 11 and n > 256:
                continue
            eng = LocalArEngine(w, max_streams=n, device=dev, path=path)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    eng.frame(b, stream=stream)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(calls):
                    eng.frame(b, stream=stream)
                e1.record(stream)
            torch.cuda.synchronize(dev)
            t = e0.elapsed_time(e1) * 1000.0 / calls
            tf = n * 2 * 2 * SHAPE_BASELINE.macs_per_row() / (t * 1e-6) / 1e12
            row[name] = {"frame_path": PATH_NAMES.get(eng.path, str(eng.path)), "frame_call_us": t,
                         "frames_per_s": n / (t * 1e-6), "tensor_frac": tf / tensor_peak,
                         "invalid_rows": int(b.invalid_rows.count_nonzero().item())}
        out[str(n)] = row
    return out


def alignment_gate_measure(dev, peaks, n=1024, stride=512, steps=200, seed=11):
    """The alignment gate (mtt_b200_launch_alignment_batch) for the config-4
    sessions of one GPU: text lengths U[64, 512], a fresh score row per step
    (copied in by a kernel of the same graph, as the Main Decoder writes it),
    `steps` gate launches captured in one CUDA graph; per-launch device time
    by CUDA events.  Algorithmic bytes per launch: per session the
    conditional score row read (2T), the counters read (4T), the prior
    written (4T) and ~40 bytes of scalars.  Beside it, the reference's own
    host controller (oracle/_ref, compiled from the reference's
    alignment_controller.cpp) on the same sessions on one host core."""
    from magpie_tts_rt_b200.local_ar import AlignmentBatch
    rng = np.random.default_rng(seed)
    T = rng.integers(64, stride + 1, n)
    ab = AlignmentBatch.allocate(T.tolist(), token_stride=stride, device=dev)
    unf = torch.zeros(n, dtype=torch.bool, device=dev)
    fe = torch.zeros(n, dtype=torch.bool, device=dev)
    fin = torch.zeros(n, dtype=torch.bool, device=dev)
    end = torch.full((n,), -1, dtype=torch.int32, device=dev)
    frames = 8
    g = torch.Generator().manual_seed(seed)
    src = torch.randn(frames, n, 2, stride, generator=g).to(torch.bfloat16).to(dev)
    stream = torch.cuda.Stream(dev)
    outs = dict(unfinished=unf, forbid_eos=fe, finished=fin, end_frame_index=end)
    with torch.cuda.stream(stream):
        for f in range(3):
            ab.alignment_scores.copy_(src[f % frames])
            ab.gate(stream=stream, **outs)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    gate_only = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for f in range(steps):
            ab.alignment_scores.copy_(src[f % frames])
            ab.gate(stream=stream, **outs)
    with torch.cuda.graph(gate_only, stream=stream):
        for f in range(steps):
            ab.gate(stream=stream, **outs)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(stream):
        graph.replay()
        gate_only.replay()
        e[0].record(stream)
        graph.replay()
        e[1].record(stream)
        e[2].record(stream)
        gate_only.replay()
        e[3].record(stream)
    torch.cuda.synchronize(dev)
    with_copy_us = e[0].elapsed_time(e[1]) * 1000.0 / steps
    gate_us = e[2].elapsed_time(e[3]) * 1000.0 / steps
    inv = int((ab.invalid_state != 0).sum().item())
    del graph, gate_only
    bytes_ = int(T.sum()) * (2 + 4 + 4) + n * 40
    gbs = bytes_ / (gate_us * 1e-6) / 1e9
    out = {"workload": f"{n} sessions (config 4 at 1 GPU), text lengths U[64,{stride}], token stride {stride}",
           "kernel": "alignment_gate_kernel<true>", "us_per_launch": gate_us,
           "us_per_step_with_score_copy": with_copy_us, "invalid_sessions": inv,
           "roofline": {"bound": "hbm", "algorithmic_bytes": bytes_, "achieved": gbs, "unit": "GB/s",
                        "peak": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"]}}
    try:
        from oracle import alignment_ref as R
        if os.path.exists(R.LIBRARY):
            ctrl = [R.RefController(int(t)) for t in T]
            rows = src[0, :, 0].float().cpu().numpy()
            t0 = time.perf_counter()
            reps = 0
            while time.perf_counter() - t0 < 2.0:
                for s, c in enumerate(ctrl):
                    c.advance(rows[s, :T[s]])
                reps += 1
            dt = time.perf_counter() - t0
            out["cpu_baseline"] = {"value": dt / reps * 1e6, "unit": "us per step of all sessions", "cores": 1,
                                   "kind": "reference",
                                   "sample": f"the reference's AlignmentControllerReference::advance on "
                                             f"{n} sessions x {reps} steps"}
    except Exception as ex:  # the baseline is optional; the GPU figure stands alone
        out["cpu_baseline"] = {"unavailable": repr(ex)[:200]}
    return out


def main_decoder_measure(dev, peaks, n=256, steps=20, text=128, cap=467, seed=13, with_cpu=True, graph=True):
    """The Main Decoder step (mtt_b200_launch_main_decoder_step) for config
    5's sessions of one GPU: n sessions x CFG pair, the reference's cache of
    467 positions, 128 text tokens, positions starting U[218, 466 - steps]
    and advancing one per step; `steps` steps timed by CUDA events after 3
    warm-up steps.  Algorithmic bytes per step: the layer weights once, and
    per session the keys and values of every layer, head and row up to its
    position, the text keys and values of every layer, and its ~20 KB of
    activations; FLOPs: 2 x 2 rows x 87.3 M MAC of projections per session
    plus the attention."""
    from magpie_tts_rt_b200.main_decoder import (
        CROSS_DIM, HEAD_DIM, HEADS, LAYERS, WIDTH, MainDecoderBatch, MainDecoderEngine,
        make_main_decoder_weights, step_weight_bytes,
    )
    w = make_main_decoder_weights(seed, positions=cap)
    eng = MainDecoderEngine(w, max_sessions=n, token_stride=text, device=dev)
    b = MainDecoderBatch.allocate(n, cap=cap, token_stride=text, device=dev)
    rng = np.random.default_rng(seed)
    pos0 = torch.from_numpy(rng.integers(218, cap - steps - 4, n)).to(dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    b.embedded.normal_(0, 0.05, generator=g)
    b.cross_k.normal_(generator=g)
    b.cross_v.normal_(generator=g)
    b.self_k.normal_(generator=g)
    b.self_v.normal_(generator=g)
    b.text_length.fill_(text)
    b.cond_mask.fill_(True)
    b.cond_mask[:, 1, 1:] = False
    b.prior.fill_(0.1)
    b.prior[:, 0, :16] = 1.0
    idx = torch.arange(cap, device=dev)
    b.self_mask.copy_((idx[None, None, :] < pos0[:, None, None]).expand(n, 2, cap))
    b.position.copy_(pos0)
    def one_step():
        eng.step(b, stream=stream)
        b.position += 1

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            one_step()
    torch.cuda.synchronize(dev)
    cuda_graph = None
    if graph:
        # one step captured once (the tensor maps and kernel attributes exist
        # after the warm-up) and replayed; the positions advance on the device
        cuda_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cuda_graph, stream=stream):
            one_step()
        torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start_pos = b.position.clone()
        e0.record(stream)
        for _ in range(steps):
            if cuda_graph is not None:
                cuda_graph.replay()
            else:
                one_step()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    del cuda_graph
    us = e0.elapsed_time(e1) * 1000.0 / steps
    bad = int((b.status != 0).sum().item())
    active = (start_pos.double() + 1).cpu().numpy()  # keys read per row and head at the first timed step
    kv = float(LAYERS * 2 * HEADS * HEAD_DIM * 2 * 2) * (active.sum() + n * (steps - 1) / 2)
    cross = float(n * LAYERS * 2 * text * CROSS_DIM * 2 * 2)
    act = n * 2 * 20_000.0
    bytes_ = step_weight_bytes() + kv + cross + act
    macs_proj = LAYERS * (3 * WIDTH * WIDTH + WIDTH * WIDTH + 2 * CROSS_DIM * WIDTH + 2 * 3072 * WIDTH)
    flops = 2 * 2 * n * macs_proj + 2 * 2 * n * LAYERS * (HEADS * HEAD_DIM * 2 * active.mean() + CROSS_DIM * 2 * text)
    gbs = bytes_ / (us * 1e-6) / 1e9
    out = {"workload": f"config 5 per GPU: {n} sessions x CFG pair, cache {cap}, {text} text tokens, positions "
                       f"U[218, {cap - steps - 4}) advancing one per step, {steps} steps",
           "us_per_step": us, "decoder_steps_per_s": n * 1e6 / us, "status_nonzero": bad,
           "kernels": "per layer: 6 tcgen05 GEMMs (gemm_tc_kernel; GELU in the FFN1 epilogue, FFN2 split-K 4) + "
                      "self_attn_kernel + cross_attn_kernel + 3 add_ln_kernel",
           "gpu_launches_per_step": 1 + LAYERS * 11,
           "cuda_graph_per_step": graph,
           "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": bytes_, "achieved": gbs, "unit": "GB/s",
                        "peak": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"],
                        "algorithmic_flops_per_step": flops,
                        "tflops": flops / (us * 1e-6) / 1e12}}
    del b, eng
    torch.cuda.empty_cache()
    if with_cpu:
        from oracle import main_decoder as OMD
        torch.set_num_threads(os.cpu_count() or 1)
        k = 0
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < 8.0 or k < 2:
            inp = OMD.make_step_inputs(100 + k, text, 300, cap)
            OMD.step(w, inp)
            k += 1
        dt = (time.perf_counter() - t0) / k
        out["cpu_baseline"] = {"value": n * dt * 1e6, "unit": "us per step of all sessions", "kind": "port",
                               "cores": torch.get_num_threads(),
                               "sample": f"{k} single-session steps of the PyTorch-CPU restatement (bit-exact with "
                                         f"the reference wrapper), position 300, scaled to {n} sessions"}
    return out


def loop_measure(dev, peaks, n=256, steps=1024, text=128, seed=17):
    """Config 5: the full per-frame loop on the device for n sessions x CFG
    pair per GPU, `steps` frames each, driven by the C++ session engine
    (mtt_b200_session_engine_*): one frame = Main Decoder step (cache growing
    from position 0 to steps - 1, capacity = steps; 128 text states ~N(0, 1))
    -> alignment gate -> Local AR frame (16 positions, sampling, EOS) ->
    position + 1, one CUDA graph per frame replayed by the engine on its own
    stream; the decoder's hidden state, the frame's embedding sum, the
    alignment scores and the prior are shared buffers, so nothing crosses to
    the host inside the timed loop.  Random-init weights (decoder ~N(0, 0.02),
    Local AR as config 4).  Timed by CUDA events around the whole loop after a
    3-frame warm-up (every session re-opened afterwards)."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    from magpie_tts_rt_b200.main_decoder import (CROSS_DIM, LAYERS, MainDecoderEngine, make_main_decoder_weights)
    from magpie_tts_rt_b200.session_engine import SessionEngine
    cap = steps
    wd = make_main_decoder_weights(seed, positions=cap)
    dec = MainDecoderEngine(wd, max_sessions=n, token_stride=text, device=dev)
    wl = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline", with_final=True)
    lar = LocalArEngine(wl, max_streams=n, device=dev)
    eng = SessionEngine(lar, n, text, decoder=dec, cache_capacity=cap)
    g = torch.Generator(device=dev).manual_seed(seed)
    cross_k = torch.randn(LAYERS, 2, text, CROSS_DIM, generator=g, device=dev).to(torch.bfloat16)
    cross_v = torch.randn(LAYERS, 2, text, CROSS_DIM, generator=g, device=dev).to(torch.bfloat16)
    cond = torch.ones(2, text, dtype=torch.bool, device=dev)
    cond[1, 1:] = False
    first = (torch.randn(n, EMBED, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    torch.cuda.synchronize(dev)

    def open_all():
        for s in range(n):
            eng.open(s, s, text, cross_k, cross_v, cond, first[s])

    open_all()
    for _ in range(3):  # eager step, then the captured graph
        eng.step()
    open_all()
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        eng.step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    codes, end, inv = eng.collect(n)
    bad = int((inv != 0).sum())
    finished = int(torch.from_numpy(end).ge(0).sum())
    launches = steps * (145 + 1 + lar.launch_count(n) + 1)
    out = {"workload": f"config 5 per GPU: {n} sessions x CFG pair, {steps} frames, decoder cache growing to "
                       f"{steps}, {text} text states; frame = Main Decoder step -> alignment gate -> Local AR "
                       f"frame, all on the device",
           "driver": "C++ session engine (mtt_b200_session_engine_*), one CUDA graph per frame step",
           "frames_per_s": n * steps / (ms * 1e-3), "ms_per_frame_step": ms / steps, "total_s": ms * 1e-3,
           "gpu_launches": launches, "cuda_graph_per_frame": True,
           "local_ar_path": PATH_NAMES.get(lar.path_for(n), str(lar.path_for(n))),
           "sessions_ended_last_frame": finished, "invalid": bad}
    eng.close_engine()
    del eng, dec, lar
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# CPU baseline (oracle restatement of the reference's path)
# ---------------------------------------------------------------------------

def cpu_oracle_sample(streams=64, min_seconds=10.0, max_frames=40, warm=1):
    from oracle import lt_oracle
    from oracle import sampler as S
    torch.set_num_threads(os.cpu_count() or 1)
    w = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline", with_final=False)
    g = torch.Generator().manual_seed(5)
    seeds = np.arange(streams)
    counter = np.zeros(streams, np.int64)
    done = 0
    t0 = None
    for f in range(max_frames + warm):
        if f == warm:
            t0 = time.perf_counter()
        hidden = torch.randn(streams, 2, EMBED, generator=g).to(torch.bfloat16)
        r = lt_oracle.run_frame(w, hidden, True, False, f < 2, seeds, counter, S.SamplingParams(), eos=False)
        counter = r.counter
        if f >= warm:
            done += 1
            if time.perf_counter() - t0 >= min_seconds:
                break
    dt = time.perf_counter() - t0
    return {"value": streams * done / dt, "unit": "frames/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{streams} sessions x CFG pair x {done} frames of the config-4 shape "
                      f"(PyTorch-CPU NeMo-forward restatement + C sampling restatement), {dt:.1f} s"}


def run_reference(args, world, rank):
    """--impl reference: the reference path's CPU implementation on host cores."""
    if rank != 0:
        return None
    cfg = WORKLOADS[args.workload]
    steps = []
    for i in range(args.warmup + args.steps):
        s = cpu_oracle_sample(streams=64, min_seconds=0.0, max_frames=2, warm=0)
        if i >= args.warmup:
            steps.append(s["value"])
    value = float(np.mean(steps))
    s["value"] = value
    s["sample"] = f"each step: 64 sessions x CFG pair x 2 frames of {args.workload} (bounded sample)"
    return dict(value=value, cpu=s)


def main():
    args = parse()
    world, rank, local = dist_init()
    peaks, peaks_kind = load_peaks()
    if args.loop_only:
        out = loop_measure(torch.device("cuda", local), peaks, steps=args.loop_steps)
        if rank == 0:
            print(json.dumps({"config5_loop": out}), flush=True)
        return
    if args.workload == "config5":
        # every rank runs its own 256 sessions (no data-path collective); the
        # box value is all ranks' frames over the slowest rank's loop time
        barrier(world)
        out = loop_measure(torch.device("cuda", local), peaks, steps=args.loop_steps)
        t = max_over_ranks(out["total_s"], world)
        frames = sum_over_ranks(256.0 * args.loop_steps, world)
        bad = sum_over_ranks(float(out["invalid"]), world)
        if rank == 0:
            print(json.dumps({"metric": "config 5 full per-frame loop frames/sec (box)", "value": frames / t,
                              "unit": "frames/s", "n_gpus": world, "higher_is_better": True, "scaling": "weak",
                              "per_gpu_frames_per_s": frames / t / world, "max_rank_s": t,
                              "rank0": out, "invalid": bad, "vs_baseline": None, "dtype": "bf16",
                              "data": "synthetic"}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.phase_trace:
        path, n = (int(v) for v in args.phase_trace.split(":"))
        w = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline")
        out = quad_trace(w, torch.device("cuda", local), path, n)
        if rank == 0:
            print(json.dumps({"phase_trace": out}), flush=True)
        return
    if args.eos_only:
        w = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline")
        out = eos_measure(w, torch.device("cuda", local), peaks, sizes=tuple(args.eos_sessions or (64, 1024)))
        if rank == 0:
            print(json.dumps({"eos_projection": out}), flush=True)
        return
    if args.latency_only:
        w = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline")
        dev = torch.device("cuda", local)
        out = latency_config2(w, dev)
        out["phase_breakdown"] = latency_trace(w, dev)
        if rank == 0:
            print(json.dumps({"latency_config2": out}), flush=True)
        return
    if args.r_shape_only:
        out = r_shape_measure(torch.device("cuda", local), peaks, sizes=tuple(args.r_sessions or (64, 1024)))
        if rank == 0:
            print(json.dumps({"r_shape_frame": out}), flush=True)
        return
    if args.main_decoder_only:
        out = main_decoder_measure(torch.device("cuda", local), peaks, n=args.md_sessions, steps=args.md_steps,
                                   with_cpu=False)
        if rank == 0:
            print(json.dumps({"main_decoder_step": out}), flush=True)
        return
    cfgw = dict(WORKLOADS[args.workload])
    if args.sessions:
        cfgw.update(weak=True)
    config = {"workload": f"{args.workload}: " + (
        "1024 sessions x CFG pair sharded over N GPUs, 500 frames, 5% forced EOS at U[50,500]"
        if args.workload == "config4" else "64 sessions x CFG pair per GPU, forced EOS at U[200,600], 600 frames"),
        "shape": "in-proj 768->256, 1 layer, d=256, 4 heads, FFN 1024, 16 heads 256->2024",
        "sampling": "CFG 2.5, T 0.6, top-k 80, Philox seeds = session index",
        "l2": "inputs larger than L2 (new hidden states every frame, >1 GB per step at N=1); weights stay "
              "L2-resident across frames as in serving",
        "parallelism": f"session-sharded dp{world}, no collective"}
    if args.sessions:
        config["workload"] += f" (profiling override: {args.sessions} sessions per GPU)"
    if args.impl == "reference":
        r = run_reference(args, world, rank)
        if rank == 0:
            line = {"metric": METRIC, "value": r["value"], "unit": "frames/s", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "impl": "reference",
                    "scaling": "weak" if cfgw["weak"] else "strong", "vs_baseline": None, "dtype": "bf16",
                    "data": "synthetic", "config": config, "cpu_baseline": r["cpu"],
                    "e2e": {"value": r["value"], "unit": "frames/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    res = run_ours(args, world, rank, local)
    latency = None
    if world == 1 and not args.no_latency:
        latency = latency_config2(res["w"], torch.device("cuda", local))
        latency["phase_breakdown"] = latency_trace(res["w"], torch.device("cuda", local))
    align = None
    if world == 1 and not args.no_latency:
        align = alignment_gate_measure(torch.device("cuda", local), peaks)
    md = None
    if world == 1 and not args.no_latency:
        md = main_decoder_measure(torch.device("cuda", local), peaks, n=args.md_sessions, steps=args.md_steps,
                                  with_cpu=rank == 0 and not args.no_cpu_baseline)
    loop = None
    if world == 1 and not args.no_latency and not args.no_loop:
        loop = loop_measure(torch.device("cuda", local), peaks, steps=args.loop_steps)
    probe = eos = rshape = paths = None
    if world == 1 and not args.no_latency:
        probe = tensor_probe(torch.device("cuda", local))
        eos = eos_measure(res["w"], torch.device("cuda", local), peaks)
        rshape = r_shape_measure(torch.device("cuda", local), peaks)
        paths = frame_paths_measure(res["w"], torch.device("cuda", local), peaks)
    c3 = None
    if world == 1 and not args.no_latency and args.workload == "config4":
        c3 = config3_measure(args, peaks)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_oracle_sample()
    if rank == 0:
        shape = SHAPE_BASELINE
        frames_per_step = res["frames_per_step"]
        t_step = res["t"] / args.steps
        # roofline over one frame step of this rank (algorithmic units per frame step)
        active_per_frame = frames_per_step / world / res["frames"]
        flops = active_per_frame * 2 * 2 * shape.macs_per_row()
        bytes_ = shape.frame_weight_params() * 2 + active_per_frame * 31_000
        t_frame = t_step / res["frames"]
        tf = flops / t_frame / 1e12
        gbs = bytes_ / t_frame / 1e9
        tensor_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        # dominant kernel: the frame kernel (98.4% of device time in the launch list); one frame
        # call = that kernel + the EOS projection/decision kernels, timed together by CUDA events
        roof = {"bound": "tensor",
                "kernel": {"tile kernel": "tile_frame_kernel", "pair kernel": "pair_frame_kernel",
                           "fused cluster kernel": "fused_frame_kernel", "split kernel x1": "split_frame_kernel<1, 16>",
                           "split kernel x2": "split_frame_kernel<2, 16>",
                           "split kernel x4": "split_frame_kernel<4, 16>",
                           "split kernel x8": "split_frame_kernel<8, 16>",
                           "split kernel x2, 32-row tiles": "split_frame_kernel<2, 32>",
                           "quad kernel": "quad_frame_kernel<4>", "octo kernel": "quad_frame_kernel<8>"}.get(
                              res["path"], res["path"]) +
                          " (per frame call, with the EOS projection/decision kernels: 0.6% of device time)",
                "achieved": tf, "peak": tensor_peak, "unit": "TFLOP/s", "frac": tf / tensor_peak,
                "peak_kind": f"{peaks_kind} sustained bf16",
                # dram__bytes_read.sum + dram__bytes_write.sum of one frame-kernel launch, taken
                # from an ncu capture of the same kernel at the same sessions per GPU (L2 flushed
                # by ncu before the pass); null for a (kernel, batch) with no capture
                "traffic": TRAFFIC.get((res["path"], res["n_local"])),
                "traffic_source": ("ncu capture of this kernel at this batch (not measured in this run)"
                                   if (res["path"], res["n_local"]) in TRAFFIC else None),
                "avg_frame_call_us": t_frame * 1e6,
                "hbm_achieved_gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"],
                "algorithmic_flops_per_frame_step": flops, "algorithmic_bytes_per_frame_step": bytes_}
        line = {"metric": METRIC, "value": res["value"], "unit": "frames/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["t"] / args.steps * 1000.0,
                "higher_is_better": True, "scaling": "weak" if cfgw["weak"] else "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": config,
                "frames_per_step": frames_per_step, "per_gpu_frames_per_s": res["value"] / world,
                "e2e": {"value": res["e2e"], "unit": "frames/s", "h2d_bytes_per_step": res["h2d"],
                        "d2h_bytes_per_step": res["d2h"]},
                "gpu_launches": res["launches"], "frame_path": res["path"], "clocks": res["clocks"],
                "roofline": roof,
                "latency_config2": latency, "alignment_gate": align, "main_decoder_step": md,
                "config5_loop": loop, "eos_projection": eos, "tensor_probe": probe, "r_shape_frame": rshape,
                "frame_paths": paths, "config3": c3,
                "cpu_baseline": cpu,
                "checks": {"invalid_rows": res["invalid"], "forced_eos_ok": res["forced_ok"]}}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
