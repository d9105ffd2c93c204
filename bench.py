"""Benchmark of the int8 decode step: tokens/s at B = 65536 streams per GPU, as a fraction of the HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3] [--impl b200|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

A step is one decode step of every stream (the reference API's `step(tokens, state)` over B streams). Streams are
independent, so N GPUs each run B streams of their own (weak scaling, no collective on the step path); the timed
region is bracketed by a barrier and a device synchronise, and the time is the max over ranks.

  value     kernel-only throughput: tokens and state resident in HBM, K launches of ygg_step on the launch stream,
            timed with CUDA events on that stream; inputs (the 287 MB model) are larger than L2.
  e2e       the same metric through the public API (B200Yggdrasil.step) with host tokens in pinned memory copied in
            every step and the logits read back every step.
  roofline  algorithmic bytes gathered per token (per-stream weights + state/logit traffic) x tokens per launch /
            the average launch time, against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the reference's own int8 kernel (cpu/ygg.cpp, built under oracle/_ref) on the host cores, one
            stream per core as the reference runs it (`ygg time`, which includes a softmax per token). A workload of
            the d_state 96 format extension (c3n96), whose file the reference's ygg refuses, is timed on the C oracle
            (the scalar port, one core) instead.
--impl reference times that CPU path alone, on rank 0, and prints its own line.
--sweep B1,B2,... measures a batch sweep instead (one JSON line per batch size, kernel time only): decode steps, or
whole rows scored with --mode score.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int8 step tokens/s at B=65536, 1/2/4/8 B200 (% HBM roofline); batch-1 us/token"
UNIT = "tokens/s"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def build_model_file(workload, seed, rank, world, dist):
    """The workload's model file, written once (rank 0) into a shared temp dir. The Zipf-calibrated models (c4, c4f;
    c5 scores c4's) take their router thresholds from tests/golden/zipf_thresholds.npz, the same fixture the parity
    tests pin to the reference's int_forward (tests/golden/make_golden.py calibrates them)."""
    from yggdrasil_b200 import synth
    from yggdrasil_b200.ygg1 import write_model
    w = synth.WORKLOADS[workload]
    d = Path(os.environ.get("YGG_BENCH_DIR", tempfile.gettempdir())) / "ygg_bench"
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"{w.model or workload}_s{seed}_v2.bin"
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        layers = synth.workload_layers(w, seed=seed, thresholds=synth.zipf_thresholds_of(w, ROOT))
        write_model(layers, np.linspace(-1, 1, w.shape.vocab), tmp, extended=w.extended)
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()
    return w, path


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        if shutil.which("nvidia-smi"):
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_run(model_path, workload, steps, warmup, seg=1000, cores=None):
    """The reference's ygg.cpp (oracle/_ref/ygg) on every host core, one stream per core, pinned with taskset:
    `ygg time model x.i32 --seg S --warm W*S` over (W + K) * S tokens per core. Returns (tokens/s, cores, median
    ns/token over cores, kind, sample text)."""
    from oracle import oracle as O
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[workload]
    avail = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count()))
    cores = avail if cores is None else avail[:cores]
    if not O.ref_available():
        return None
    tmp = Path(tempfile.mkdtemp(prefix="ygg_ref_"))
    procs = []
    try:
        for i, c in enumerate(cores):
            x = synth.workload_tokens(w, 1, (warmup + steps) * seg, seed=1000 + i)[0]
            xf = tmp / f"x{i}.i32"
            x.astype(np.int32).tofile(xf)
            cmd = [str(O.REF_YGG), "time", str(model_path), str(xf), "--seg", str(seg), "--warm", str(warmup * seg)]
            if shutil.which("taskset"):
                cmd = ["taskset", "-c", str(c)] + cmd
            procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
        med = []
        for p in procs:
            out, err = p.communicate(timeout=1800)
            if p.returncode:
                raise RuntimeError(f"ygg time failed: {err.strip()[:300]}")
            tok = {k: v for k, v in (t.split("=", 1) for t in out.split() if "=" in t)}
            med.append(float(tok["median"]))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    tps = float(sum(1e9 / m for m in med))
    sample = (f"{len(cores)} processes of `ygg time --seg {seg} --warm {warmup * seg}`, {steps * seg} timed tokens "
              f"each (one stream per core, softmax per token included), median {np.median(med):.0f} ns/token")
    return tps, len(cores), float(np.median(med)), "reference", sample


def cpu_port_run(model_path, workload, seconds=10.0):
    """The C oracle (the scalar restatement of cpu/ygg.cpp) on one core and one stream, for a file the reference's
    ygg refuses (the d_state 96 extension): tokens/s over about `seconds` of stepping, no softmax. Returns the tuple
    of cpu_reference_run."""
    from oracle import oracle as O
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[workload]
    om = O.OracleModel(model_path)
    x = synth.workload_tokens(w, 1, 1 << 20, seed=1000)[0]
    st = om.init_state(1)
    for t in range(64):
        om.step(x[t:t + 1], st)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for t in range(256):
            om.step(x[64 + n + t:65 + n + t], st)
        n += 256
    dt = time.perf_counter() - t0
    sample = (f"the C oracle (scalar port of cpu/ygg.cpp), one stream on one core, {n} steps after 64 warm-up "
              f"steps (no softmax); the reference's ygg refuses d_state 96 files (cpu/ygg.cpp:141-146)")
    return n / dt, 1, dt / n * 1e9, "port", sample


def cpu_model_name():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from yggdrasil_b200 import synth
    w, path = build_model_file(args.workload, 7, 0, 1, None)
    if w.extended:
        res = cpu_port_run(path, args.workload)
    else:
        res = cpu_reference_run(path, args.workload, args.steps, args.warmup, seg=args.ref_seg)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference binary oracle/_ref/ygg is not built"}))
        return 0
    tps, cores, med, kind, sample = res
    line = {"metric": METRIC, "value": tps, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": w.name, "streams_per_core": 1, "cpu": cpu_model_name(),
                       "bytes_per_token": synth.gathered_bytes_per_token(w.shape)},
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "ns_per_token_median": med}
    print(json.dumps(line))
    return 0


def run_score(args, w, path, world, rank, local, dist):
    """Whole rows scored on the GPU (bits of tokens[:, 1:], the reference's score): B rows of T tokens per GPU, the
    fused score kernel (state and logits on chip for the whole row) and, with --grouped, the leaf-grouped path whose
    heavy leaves run as int8 tensor-core GEMMs. Tokens scored per second = B (T - 1) / time, summed over the GPUs."""
    import torch

    from yggdrasil_b200 import Yggdrasil, synth
    dev = torch.device("cuda", local)
    model = Yggdrasil.load(path, backend="b200", device=dev)
    stream = torch.cuda.current_stream(dev)
    B = args.streams or w.streams
    T = args.score_steps or w.steps
    K, W = args.steps, args.warmup
    x = torch.as_tensor(synth.workload_tokens(w, B, T, seed=rank)).to(dev)
    bits = torch.empty(B, dtype=torch.float64, device=dev)

    def timed(fn, reps):
        for _ in range(W):
            fn()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    reps = max(1, K)
    ms_fused = timed(lambda: model.score_into(x, None, bits), reps)
    fused_bits = bits.clone()
    ms_grouped = None
    if args.grouped:
        ms_grouped = timed(lambda: model.score_grouped_into(x, None, bits, min_group=args.min_group), reps)
        if not torch.equal(bits, fused_bits):
            raise RuntimeError("grouped and fused scores differ")
    model.status()
    tok = B * (T - 1) * world
    # end to end through the public API: host tokens in, bits (float64 per row) out
    h = synth.workload_tokens(w, B, T, seed=rank)
    a0 = time.perf_counter()
    model.score(h, batch=B, grouped=args.grouped, min_group=args.min_group)
    e2e_s = time.perf_counter() - a0
    ms = ms_grouped if args.grouped else ms_fused
    bpt = synth.gathered_bytes_per_token(w.shape, with_io=False) + 4
    peak, kind = peaks()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    L = model.layers
    line = {"metric": "tokens scored/s (bits of whole rows)", "value": tok / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": reps, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": w.name, "rows_per_gpu": B, "tokens_per_row": T, "mode": "score",
                       "path": f"grouped (min_group {args.min_group})" if args.grouped else "fused",
                       "fused_tokens_per_s": tok / (ms_fused / 1e3),
                       "grouped_tokens_per_s": tok / (ms_grouped / 1e3) if ms_grouped else None,
                       "bytes_per_token": bpt},
            "roofline": {"bound": "hbm", "achieved": bpt * B * (T - 1) / (ms / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": bpt * B * (T - 1) / (ms / 1e3) / 1e9 / peak, "traffic": None,
                         "peak_kind": kind},
            "e2e": {"value": B * (T - 1) / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(B * T * 4),
                    "d2h_bytes_per_step": int(B * 8)},
            "gpu_launches": reps * ((T - 1) * (5 * L + 1) + 2 if args.grouped else 1)}
    print(json.dumps(line))
    return 0


def run_sweep(args, w, path, world, rank, local, dist):
    """Kernel-only throughput over a batch sweep (streams per GPU; weak scaling under torchrun, time = max over
    ranks). step: 16 untimed steps, W warm-up steps, then K steps with K ~ 2^22 / B (64 to 2048), tokens resident in
    HBM, launched as replays of a CUDA graph of 32 steps (so that a small batch measures the device, not the rate at
    which Python launches). score: rows of T tokens with T ~ 2^24 / B (64 to the workload's row length), the fused
    score kernel."""
    import torch

    from yggdrasil_b200 import Yggdrasil, synth
    dev = torch.device("cuda", local)
    model = Yggdrasil.load(path, backend="b200", device=dev)
    stream = torch.cuda.current_stream(dev)
    peak, kind = peaks()

    def max_ms(ms):
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for B in (int(v) for v in args.sweep.split(",")):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.mode == "step":
            G = 32
            K, W, P = min(2048, max(2 * G, (1 << 22) // B)) // G * G, args.warmup, 16
            x = torch.as_tensor(synth.workload_tokens(w, P + W + G, B, seed=rank)).to(dev)
            state = model.init_state(B)
            logits = torch.empty(B, model.vocab, dtype=torch.float32, device=dev)
            for i in range(P + W):
                model.step_into(x[i], state, state, logits)
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):   # one eager pass on the capture stream first
                for i in range(G):
                    model.step_into(x[P + W + i], state, state, logits)
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(G):
                    model.step_into(x[P + W + i], state, state, logits)
            graph.replay()
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            e0.record(stream)
            for _ in range(K // G):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms = max_ms(e0.elapsed_time(e1)) / K
            tokens, bpt = B * world, synth.gathered_bytes_per_token(w.shape)
            rec = {"steps": K, "us_per_step": ms * 1e3, "launch": "CUDA graph of 32 steps"}
            del graph, x, state, logits
        else:
            T = min(w.steps, max(64, (1 << 24) // B))
            x = torch.as_tensor(synth.workload_tokens(w, B, T, seed=rank)).to(dev)
            bits = torch.empty(B, dtype=torch.float64, device=dev)
            for _ in range(max(1, args.warmup // 3)):
                model.score_into(x, None, bits)
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            e0.record(stream)
            model.score_into(x, None, bits)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms = max_ms(e0.elapsed_time(e1))
            tokens, bpt = B * (T - 1) * world, synth.gathered_bytes_per_token(w.shape, with_io=False) + 4
            rec = {"tokens_per_row": T, "ms": ms}
            del x, bits
        torch.cuda.empty_cache()
        model.status()
        if rank == 0:
            tps = tokens / (ms / 1e3)
            print(json.dumps({"sweep": args.mode, "workload": w.name, "n_gpus": world, "streams_per_gpu": B, **rec,
                              "tokens_per_s": tps, "roofline_frac": tps / world * bpt / 1e9 / peak,
                              "peak_kind": kind}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--workload", default="c3")
    ap.add_argument("--streams", type=int, default=0, help="streams per GPU (default: the workload's, capped 65536)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-seg", type=int, default=2000, help="tokens per timed segment of the CPU reference")
    ap.add_argument("--cpu-steps", type=int, default=100, help="timed segments per core of the CPU baseline")
    ap.add_argument("--batch1-steps", type=int, default=512)
    ap.add_argument("--prime", type=int, default=64, help="untimed steps that give every stream a history first")
    ap.add_argument("--mode", default="step", choices=["step", "score", "float"],
                    help="step: the decode step (the headline metric); score: whole rows scored on the GPU; float: "
                    "only the fp32 float step's measurement (one GPU)")
    ap.add_argument("--score-steps", type=int, default=0, help="tokens per row in score mode (default: the workload's)")
    ap.add_argument("--grouped", action="store_true", help="score mode: also time the leaf-grouped tensor-core path")
    ap.add_argument("--min-group", type=int, default=64, help="streams a leaf needs for the tensor-core path")
    ap.add_argument("--sweep", default="", help="comma-separated streams per GPU: a batch sweep, one line per size")
    ap.add_argument("--global-streams", type=int, default=65536,
                    help="strong scaling: also time this many streams split over the N GPUs (0: off)")
    ap.add_argument("--no-float", dest="float", action="store_false",
                    help="skip the fp32 float step measurement (backend b200f, one-GPU runs)")
    ap.add_argument("--extra", default="c4", help="also measure this workload at 65 536 and 262 144 streams per GPU "
                    "(and 262 144 global under torchrun), with its e2e through step(); '' to skip")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    import torch
    if args.mode == "float":
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        print(json.dumps({"mode": "float", **run_float(dev, torch.cuda.current_stream(dev), args.warmup)}))
        return 0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    from yggdrasil_b200 import Yggdrasil, synth
    w, path = build_model_file(args.workload, 7, rank, world, dist)
    if args.sweep:
        return run_sweep(args, w, path, world, rank, local, dist)
    if args.mode == "score":
        return run_score(args, w, path, world, rank, local, dist)
    B = args.streams or min(w.streams, 65536)
    K, W = args.steps, args.warmup
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        gpu_id = str(local)
    peak, kind = peaks()
    traffic_tab = load_traffic()

    # ---- the headline: the workload at B streams per GPU (weak scaling), kernel-only, clocks sampled
    with ClockSampler(gpu_id) as clk:
        head = measure_step(args, w, path, B, K, W, rank, world, dist, dev, stream, keep_model=True)
    model = head.pop("model")

    # ---- end to end through the public API, host-logits serving loop (the headline's e2e)
    e2e, ke = e2e_serving_loop(model, w, head["state"], B, K, W, rank, world, dist, dev, stream)

    # ---- batch 1 (rank 0): a row scored through the layer wavefront, and one step() call per token
    b1 = b1_step = None
    if rank == 0 and args.batch1_steps:
        b1, b1_step = batch1(model, w, args.batch1_steps, W, dev, stream)
    del head["state"], model
    torch.cuda.empty_cache()

    # ---- strong scaling at the configuration's fixed global batch (c3: 65 536 streams over the N GPUs)
    strong = {}
    if world > 1 and args.global_streams:
        r = measure_step(args, w, path, args.global_streams // world, K, W, rank, world, dist, dev, stream)
        strong[args.workload] = strong_entry(r, args.global_streams, world)
    elif args.global_streams:
        strong[args.workload] = strong_entry(head, B * world, world)

    # ---- the north-star model (c4, 730M shape, Zipf-calibrated) at 65 536 and 262 144 streams per GPU, its strong
    # scaling at 262 144 global streams, and its e2e through step(tokens, state) with host or device consumers
    extra = {}
    if args.extra and args.workload != args.extra:
        xw, xpath = build_model_file(args.extra, 7, rank, world, dist)
        xk = min(K, 256)
        for xb in (65536, 262144):
            keep = xb == 65536
            r = measure_step(args, xw, xpath, xb, xk, W, rank, world, dist, dev, stream, keep_model=keep)
            if keep:
                xmodel, xstate = r.pop("model"), r.pop("state")
                r["e2e_step_api"] = e2e_step_api(xmodel, xw, xstate, xb, W, rank, world, dist, dev, stream)
                for consumer in ("host", "device"):
                    v, ks = e2e_serving_loop(xmodel, xw, xstate, xb, xk, W, rank, world, dist, dev, stream, consumer)
                    r.setdefault("e2e_serving", {})[consumer] = {
                        "value": v, "unit": UNIT, "steps": ks, "h2d_bytes_per_step": xb * 4,
                        "d2h_bytes_per_step": xb * (xw.shape.vocab * 4 if consumer == "host" else 4)}
                del xmodel, xstate
                torch.cuda.empty_cache()
            extra[f"B{xb}"] = summarise(r, xw, xb, world, peak, kind, traffic_tab.get(f"{args.extra}_B{xb}"))
        if world > 1:
            r = measure_step(args, xw, xpath, 262144 // world, xk, W, rank, world, dist, dev, stream)
            strong[args.extra] = strong_entry(r, 262144, world)
        else:
            strong[args.extra] = {"global_streams": 262144, "streams_per_gpu": 262144,
                                  "value": extra["B262144"]["value"], "ms_per_step": extra["B262144"]["ms_per_step"]}

    # ---- the fp32 float step (backend "b200f") on the reference's enwik8 large float model, next to the reference's
    # published 80.1 us/token at batch 1 (its Triton backend, README.md:43); rank 0 of a one-GPU run
    flt = None
    if rank == 0 and world == 1 and args.float:
        flt = run_float(dev, stream, W)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            if w.extended:
                res = cpu_port_run(path, args.workload)
            else:
                res = cpu_reference_run(path, args.workload, steps=args.cpu_steps, warmup=2, seg=args.ref_seg)
        except Exception as e:  # noqa: BLE001
            res = None
            print(f"cpu baseline failed: {e}", file=sys.stderr)
        if res is not None:
            tps, cores, med, ck, sample = res
            cpu = {"value": tps, "unit": UNIT, "cores": cores, "kind": ck, "sample": sample,
                   "cpu": cpu_model_name()}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    hs = summarise(head, w, B, world, peak, kind, traffic_tab.get(f"{args.workload}_B{B}"))
    line = {"metric": METRIC, "value": hs["value"], "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": hs["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": w.name, "streams_per_gpu": B, "global_streams": B * world,
                       "model_bytes": path.stat().st_size, "bytes_per_token": synth.gathered_bytes_per_token(w.shape),
                       "tokens": "i.i.d. DNA bases p=(0.295,0.205,0.205,0.295,0.0001)" if w.tokens == "dna"
                       else "uniform bytes", "l2": "inputs larger than L2 (model file > 126 MB)",
                       "parallelism": f"streams sharded, {world} replica(s)", "primed_steps": args.prime,
                       "effective_leaves_per_layer": hs["effective_leaves_per_layer"],
                       "distinct_leaves_per_layer": hs["distinct_leaves_per_layer"],
                       "leaf_usage": leaf_usage_note(w), "note": w.note},
            "roofline": hs["roofline"],
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": int(B * 4),
                    "d2h_bytes_per_step": int(B * w.shape.vocab * 4), "steps": ke,
                    "path": "step_into serving loop: pinned host tokens up, logits down every step, copies "
                            "overlapped on two streams"},
            "gpu_launches": K,
            "batch1_us_per_token": b1,
            "batch1_step_api_us_per_token": b1_step,
            "strong_scaling": strong or None,
            "cpu_baseline": cpu,
            "clocks": clk.summary()}
    if extra:
        line[args.extra] = {"workload": synth.WORKLOADS[args.extra].name, **extra}
    if flt:
        line["float_step"] = flt
    print(json.dumps(line))
    return 0


def run_float(dev, stream, W, n1=512, big=16384):
    """The fp32 step of backend "b200f" on a random float model of the enwik8 large shape (synth.FLOAT_ENWIK8_LARGE):
    (a) batch 1 through step(tokens, state), one call per token with the token already on the device (as generate()
    keeps it), timed on the host clock; (b) the device time of one batch-1 step, from a CUDA graph of 32 steps
    replayed; (c) tokens/s at `big` streams (kernel time, tokens resident)."""
    import torch

    from yggdrasil_b200 import synth
    from yggdrasil_b200.float_backend import B200FloatYggdrasil
    shape = synth.FLOAT_ENWIK8_LARGE
    layers, ob = synth.random_float_layers(shape, seed=0)
    model = B200FloatYggdrasil(layers, ob, device=dev)
    del layers
    rng = np.random.default_rng(5)
    toks = rng.integers(0, shape["vocab"], n1 + W).astype(np.int32)
    d_toks = torch.as_tensor(toks).to(dev)
    st = model.init_state(1)
    for i in range(W):
        _, st = model.step(d_toks[i:i + 1], st)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(n1):
        _, st = model.step(d_toks[W + i:W + i + 1], st)
    torch.cuda.synchronize(dev)
    api_us = (time.perf_counter() - t0) / n1 * 1e6
    # device time per step: a graph of G step_into launches at batch 1
    G = 32
    d_tok = torch.as_tensor(toks[:G]).to(dev)
    s1 = model.init_state(1)
    lg = torch.empty(1, model.classes, device=dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for i in range(G):
            model.step_into(d_tok[i:i + 1], s1, s1, lg)
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(G):
            model.step_into(d_tok[i:i + 1], s1, s1, lg)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    reps = 16
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dev_us = e0.elapsed_time(e1) * 1e3 / (reps * G)
    del graph
    # throughput at `big` streams
    xb = torch.as_tensor(rng.integers(0, shape["vocab"], (16, big)).astype(np.int32)).to(dev)
    sb = model.init_state(big)
    lb = torch.empty(big, model.classes, device=dev)
    for i in range(W):
        model.step_into(xb[i % 16], sb, sb, lb)
    torch.cuda.synchronize(dev)
    K = 32
    e0.record(stream)
    for i in range(K):
        model.step_into(xb[i % 16], sb, sb, lb)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    tps = big * K / (e0.elapsed_time(e1) / 1e3)
    model.status()
    return {"model": "enwik8 large float shape (V256 L5 d256 b16 D10 F16 k64 R32 R2=64), random weights, fp32",
            "batch1_step_api_us_per_token": api_us, "batch1_step_device_us": dev_us,
            "reference_published_us_per_token": 80.1,
            "reference_published_note": "Triton backend, batch 1, one GPU (README.md:43)",
            "streams": big, "tokens_per_s": tps}


def load_traffic():
    """Per-launch DRAM bytes of the step kernel by workload and batch, from the ncu captures summarised in
    profiles/ (profiles/traffic.json: each entry names the capture's command)."""
    tf = ROOT / "profiles" / "traffic.json"
    if not tf.exists():
        return {}
    return {k: v for k, v in json.loads(tf.read_text()).items() if isinstance(v, dict)}


def leaf_usage_note(w):
    from yggdrasil_b200 import synth
    if w.leaves != "zipf":
        return w.leaves
    return (f"Zipf(1.1) over a seeded leaf order (target {synth.effective_leaves(synth.zipf_leaf_probs(8192, 1.1, 0)):.0f}"
            f" effective leaves); thresholds from tests/golden/zipf_thresholds.npz")


def compulsory_bytes(model, shape, tokens, routes):
    """Bytes one step must move at least, whatever the order of the streams: every distinct record it touches once
    (the token layer's record of each distinct token; each routed layer's record of each distinct leaf), each distinct
    table row once (leaf, token), each router row on a visited path once and each (token, node) threshold once, the
    launch's shared weights (layer-input down projection and its scales, unembedding, output bias), and per stream its
    token, its state in and out and its logits."""
    n, b, D, V = shape.d_state, shape.block_size, shape.router_depth, shape.vocab
    R, R2, k, L = shape.readout_rank, shape.layer_input_rank, shape.input_rank, shape.n_layers
    E, VP = 1 << D, (V + 31) // 32 * 32
    x = np.asarray(tokens, np.int64)
    B = len(x)
    total = len(np.unique(x)) * (2 * n * b + R * n + 2 * n)            # token layer: A, P and its own table row
    total += VP * 4 + L * VP * R                                          # output bias, unembeddings
    per_leaf = 2 * n * b + n * R2 + R * n + ((n * k + 2 * n + 4) if k else 0)
    for l in range(1, L):
        r = np.asarray(routes[:, l], np.int64)
        total += len(np.unique(r)) * per_leaf
        if not k:
            total += len(np.unique(r * V + x)) * 2 * n                   # table rows T_r[x]
        node = r + E
        nodes, pairs = [], []
        for _ in range(D):
            node = node >> 1
            nodes.append(node)
            pairs.append(x * E + node)
        total += len(np.unique(np.concatenate(nodes))) * n               # router rows on the visited paths
        total += len(np.unique(np.concatenate(pairs))) * 4               # thresholds thr[x][node]
        total += R2 * n + 4 * R2                                         # down projection and its scales
    total += B * (4 + 2 * L * n + 4 * V)                                  # token, state in and out, logits
    return int(total)


def measure_step(args, w, path, B, K, W, rank, world, dist, dev, stream, keep_model=False):
    """Kernel-only decode steps of B streams per GPU: prime every stream with `prime` untimed steps (from a zero
    state the first steps route on the token alone), record the leaf usage and the compulsory bytes of one step,
    run W warm-up steps, then time K steps on the launch stream with CUDA events (max over ranks). Tokens are
    resident in HBM (a ring of at most K + W steps)."""
    import torch

    from yggdrasil_b200 import Yggdrasil, synth
    model = Yggdrasil.load(path, backend="b200", device=dev)
    ring = min(K + W, max(64, (1 << 28) // (4 * B)))
    d_tok = torch.as_tensor(synth.workload_tokens(w, ring, B, seed=rank)).to(dev)   # (steps, B)
    state = model.init_state(B)
    logits = torch.empty(B, model.vocab, dtype=torch.float32, device=dev)
    xp = torch.as_tensor(synth.workload_tokens(w, max(args.prime, 1), B, seed=10_000 + rank)).to(dev)
    for i in range(args.prime):
        model.step_into(xp[i], state, state, logits)
    del xp
    _, _, routes, _ = model.step_debug(d_tok[0], state)
    r = routes.cpu().numpy()
    eff, distinct = [], []
    for l in range(1, model.layers):
        h = np.bincount(r[:, l], minlength=1 << model.depth).astype(np.float64)
        p = h[h > 0] / h.sum()
        eff.append(round(float(np.exp(-(p * np.log(p)).sum())), 1))
        distinct.append(int((h > 0).sum()))
    comp = compulsory_bytes(model, w.shape, d_tok[0].cpu().numpy(), r)
    for i in range(W):
        model.step_into(d_tok[i % ring], state, state, logits)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        model.step_into(d_tok[(W + i) % ring], state, state, logits)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1), world, dist, dev)
    model.status()
    out = {"ms_per_step": ms / K, "value": B * K * world / (ms / 1e3), "steps": K,
           "effective_leaves_per_layer": eff, "distinct_leaves_per_layer": distinct, "compulsory_bytes": comp}
    if keep_model:
        out["model"], out["state"] = model, state
    else:
        del model, state
    del d_tok, logits
    torch.cuda.empty_cache()
    return out


def max_over_ranks(ms, world, dist, dev):
    if world > 1:
        import torch
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def summarise(r, w, B, world, peak, kind, traffic):
    """The JSON entry of one measurement: tokens/s (whole job), and the roofline of the step kernel on two bases.
    frac: compulsory bytes of one launch (compulsory_bytes) / launch time / the measured HBM copy peak; algorithmic:
    the survey's gathered bytes per token x B (counts every stream's leaf bytes, also those that L2 serves to the
    streams sharing a leaf, so it is not an HBM bound); traffic: the DRAM bytes ncu measured for one launch of this
    workload and batch (profiles/traffic.json), and its ratio to the compulsory bytes."""
    from yggdrasil_b200 import synth
    sec = r["ms_per_step"] / 1e3
    comp = r["compulsory_bytes"]
    bpt = synth.gathered_bytes_per_token(w.shape)
    roof = {"bound": "hbm", "basis": "compulsory bytes per launch", "achieved": comp / sec / 1e9, "peak": peak,
            "unit": "GB/s", "frac": comp / sec / 1e9 / peak, "peak_kind": kind, "compulsory_bytes": comp,
            "traffic": None,
            "algorithmic": {"bytes_per_token": bpt, "bytes_per_launch": bpt * B, "achieved": bpt * B / sec / 1e9,
                            "frac": bpt * B / sec / 1e9 / peak}}
    if traffic:
        t = float(traffic["dram_bytes_per_launch"])
        roof.update(traffic=t, traffic_source=traffic.get("source"), dram_achieved=t / sec / 1e9,
                    dram_frac=t / sec / 1e9 / peak, dram_over_compulsory=t / comp)
    return {"value": r["value"], "ms_per_step": r["ms_per_step"], "streams_per_gpu": B,
            "effective_leaves_per_layer": r["effective_leaves_per_layer"],
            "distinct_leaves_per_layer": r["distinct_leaves_per_layer"], "roofline": roof,
            **{k: r[k] for k in ("e2e_step_api", "e2e_serving") if k in r}}


def strong_entry(r, global_streams, world):
    return {"global_streams": global_streams, "streams_per_gpu": global_streams // world, "value": r["value"],
            "ms_per_step": r["ms_per_step"]}


def e2e_serving_loop(model, w, state, B, K, W, rank, world, dist, dev, stream, consumer="host"):
    """End to end through step_into with pinned host tokens in and a result out every step: a serving loop with two
    buffers each way; while step i runs (in place), the tokens of step i + 1 go up on one copy stream and the result of
    step i - 1 comes down on another; events keep each buffer's writer after its last reader. consumer "host": the
    (B, V) float32 logits come down; "device": the logits stay on the GPU and only each stream's greedy next token
    (argmax on the device, int32) comes down. Returns (tokens/s, steps)."""
    import torch

    from yggdrasil_b200 import synth
    ke = min(K, 256)
    h_tok = torch.as_tensor(synth.workload_tokens(w, ke, B, seed=20_000 + rank)).pin_memory()
    if consumer == "host":
        h_lg = [torch.empty(B, model.vocab, dtype=torch.float32).pin_memory() for _ in range(2)]
    else:
        h_lg = [torch.empty(B, dtype=torch.int32).pin_memory() for _ in range(2)]
        d_next = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(2)]
    d_tokb = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(2)]
    d_lg = [torch.empty(B, model.vocab, dtype=torch.float32, device=dev) for _ in range(2)]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: [torch.cuda.Event() for _ in range(2)]  # noqa: E731
    uploaded, stepped, downloaded = ev(), ev(), ev()

    def upload(i):
        j = i % 2
        up.wait_event(stepped[j])                  # the step that read this buffer (i - 2) is done
        with torch.cuda.stream(up):
            d_tokb[j].copy_(h_tok[i % ke], non_blocking=True)
            uploaded[j].record(up)

    def loop(n, st):
        for e in stepped + downloaded:
            e.record(stream)
        upload(0)
        for i in range(n):
            j = i % 2
            stream.wait_event(uploaded[j])
            stream.wait_event(downloaded[j])       # the logits buffer's previous download is done
            model.step_into(d_tokb[j], st, st, d_lg[j])
            if consumer != "host":
                d_next[j].copy_(d_lg[j].argmax(-1))
            stepped[j].record(stream)
            if i + 1 < n:
                upload(i + 1)
            down.wait_event(stepped[j])
            with torch.cuda.stream(down):
                h_lg[j].copy_(d_lg[j] if consumer == "host" else d_next[j], non_blocking=True)
                downloaded[j].record(down)
        stream.wait_stream(down)

    st = state.clone()
    loop(W, st)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    loop(ke, st)
    a1.record(stream)
    torch.cuda.synchronize(dev)
    ems = max_over_ranks(a0.elapsed_time(a1), world, dist, dev)
    return B * ke * world / (ems / 1e3), ke


def e2e_step_api(model, w, state, B, W, rank, world, dist, dev, stream, steps=64):
    """The reference-shaped call, `logits, state = model.step(tokens, state)` with host (pinned) tokens, one call after
    the other, timed with events on the launch stream around `steps` calls (max over ranks), with two consumers of the
    logits: "host" copies the (B, V) float32 logits to the host every step; "device" keeps them on the GPU and brings
    back only the greedy next token of each stream (argmax on the device, B int32), as generate() and a sampling
    server do."""
    import torch

    from yggdrasil_b200 import synth
    h_tok = torch.as_tensor(synth.workload_tokens(w, steps, B, seed=30_000 + rank)).pin_memory()
    out = {}
    for consumer in ("host", "device"):
        st = state.clone()
        h_out = (torch.empty(B, model.vocab, dtype=torch.float32) if consumer == "host"
                 else torch.empty(B, dtype=torch.int64)).pin_memory()

        def one(i):
            nonlocal st
            lg, st = model.step(h_tok[i % steps], st)
            h_out.copy_(lg if consumer == "host" else lg.argmax(-1), non_blocking=True)

        for i in range(W):
            one(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for i in range(steps):
            one(i)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        ms = max_over_ranks(a0.elapsed_time(a1), world, dist, dev)
        per_step_out = B * model.vocab * 4 if consumer == "host" else B * 8
        out[consumer] = {"value": B * steps * world / (ms / 1e3), "unit": UNIT, "steps": steps,
                         "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": per_step_out}
    return out


def batch1(model, w, n1, W, dev, stream):
    """Batch 1 on rank 0: (a) device time per token of one stream scoring a row (the launch policy runs the layer
    wavefront for n = 128; state on chip, the f64 softmax/NLL of every token included, as `ygg time` includes its
    softmax); (b) one step(tokens, state) call per token through the public API, tokens already on the device (as
generate() keeps them), each call returning new logits and state tensors. The
    warm-up runs other tokens than the timed ones, so the timed tokens find their leaves' records where a new stream
    would (mostly not in L2)."""
    import torch

    from yggdrasil_b200 import synth
    t1 = torch.as_tensor(synth.workload_tokens(w, 1, n1 + 1, seed=99)).to(dev)
    t1w = torch.as_tensor(synth.workload_tokens(w, 1, n1 + 1, seed=98)).to(dev)
    bits1 = torch.empty(1, dtype=torch.float64, device=dev)
    for i in range(W):
        model.score_into(t1w, None, bits1)
    torch.cuda.synchronize(dev)
    b0, b1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    model.score_into(t1, None, bits1)
    b1e.record(stream)
    torch.cuda.synchronize(dev)
    b1 = b0.elapsed_time(b1e) * 1e3 / n1
    s1 = model.init_state(1)
    for i in range(W):
        _, s1 = model.step(t1w[0, i:i + 1], s1)
    torch.cuda.synchronize(dev)
    b0.record(stream)
    for i in range(n1):
        _, s1 = model.step(t1[0, i:i + 1], s1)
    b1e.record(stream)
    torch.cuda.synchronize(dev)
    return b1, b0.elapsed_time(b1e) * 1e3 / n1


if __name__ == "__main__":
    sys.exit(main())
