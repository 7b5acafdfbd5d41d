"""ResNet-50 v1.5 batch-256 fp32 (3xTF32) inference throughput on B200.

One process per GPU (torchrun for N > 1); the batch of 256 images is split
evenly over the ranks (256/world each), weights replicated, no collective on
the data path -- torch.distributed is used only for the barrier and the
max-over-ranks of the timings.

Prints ONE JSON line (rank 0):
  value      images/s of the whole job, inputs resident in HBM, device time
             (CUDA events around each step on the launching stream, max over ranks)
  e2e        the same through the host-buffer API (onnxb200_graph_run_host_pipelined
             over the timed steps): per step the pinned-host -> device copy of the
             input slice and the device -> host copy of the logits are inside the
             timed region; a step's input copy overlaps the previous step's compute
             (e2e.unpipelined_value: onnxb200_graph_run_host one step at a time)
  roofline   the tcgen05 implicit-GEMM kernel (all Conv/Gemm steps of one run):
             algorithmic FLOPs / device time of those steps, against the
             effective 3xTF32 peak = measured dense bf16 / 6 (burst; the
             sustained fraction beside it), plus achieved GB/s of the
             memory-bound steps
  fast_modes the same workload in the 1xTF32 and BF16 fast modes, each with its
             own roofline
  cpu_baseline  the oracle (a C restatement of the reference's CPU operators,
             batch-parallel like the reference's rayon use) on a bounded sample
`--impl reference` times that same CPU path alone (rank 0), as the reference arm.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GLOBAL_BATCH = 256
SEED = 4
METRIC = "ResNet-50 v1.5 images/sec (batch 256, fp32 via 3xTF32)"
METRIC_FAST = {"tf32": "ResNet-50 v1.5 images/sec (batch 256, fast mode: 1xTF32)",
               "bf16": "ResNet-50 v1.5 images/sec (batch 256, fast mode: BF16)",
               "fp32": "ResNet-50 v1.5 images/sec (batch 256, fp32 on CUDA cores)"}
# DRAM bytes of igemm_tc3_kernel per contraction step, mean over the 50 steps
# of one batch-256 3xTF32 run (49 convolution steps and the classifier Gemm; a
# step whose K loop is split runs two or three launches, all counted):
# dram__bytes_read.sum + dram__bytes_write.sum over the run's 59 launches from an
# ncu DRAM capture of this workload (a measured constant, not re-derived here).
TRAFFIC_PER_LAUNCH_3XTF32 = 447.5e6
L2_BYTES = 126 * 1024 * 1024


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
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
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        loaded = [v for v in sm if v > 0] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


class OracleResNet50:
    """The oracle's ResNet-50 v1.5 (a C restatement of the reference's CPU
    operators, batch-parallel like the reference's rayon use) on a bounded
    sample batch: every host thread this process may use (at most 64, so that
    the sample's activations stay a few GB), one image per thread."""

    def __init__(self, images=None):
        import importlib
        from oracle import oracle as orc
        ob = importlib.import_module("onnx-rs_b200")
        orc.build()
        try:
            self.avail = len(os.sched_getaffinity(0))
        except AttributeError:
            self.avail = os.cpu_count() or 1
        self.threads = max(1, min(self.avail, 64))
        self.n = images or self.threads
        self.orc = orc
        self.nodes, self.inits, _, self.outs = ob.workloads.resnet50(batch=self.n, seed=SEED)
        self.x = ob.workloads.resnet_input(SEED, self.n)

    def run(self):
        """One pass over the sample; returns its wall time in seconds."""
        t0 = time.perf_counter()
        self.orc.run_graph(self.nodes, self.inits, {"X": self.x}, self.outs, nthreads=self.threads)
        return time.perf_counter() - t0

    def sample(self, runs, t):
        return (f"ResNet-50 v1.5 batch {self.n} (a sample of the batch-256 workload), seed {SEED}, oracle C "
                f"restatement of the reference's CPU operators (im2col+GEMM / direct conv), batch split over "
                f"{self.threads} of {self.avail} available host threads, median of {runs} run(s), {t:.2f} s each")


def cpu_baseline(steps=1, images=None, min_seconds=0.0, max_steps=8):
    """The oracle on host cores: at least `steps` runs and more (up to
    `max_steps`) until `min_seconds` of work have been timed."""
    o = OracleResNet50(images)
    times = []
    while len(times) < steps or (sum(times) < min_seconds and len(times) < max_steps):
        times.append(o.run())
    t = statistics.median(times)
    return {"value": o.n / t, "unit": "images/s", "cores": o.threads, "kind": "port",
            "sample": o.sample(len(times), t)}


def run_reference(args):
    """The reference arm: the reference's CPU algorithms (the oracle's C
    restatement; the reference itself is Rust and cannot be built here) on the
    host cores.  A step is one pass over the sample batch (one image per host
    thread); the line reports that batch and the measured per-pass time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    o = OracleResNet50()
    for _ in range(args.warmup):
        o.run()
    times = [o.run() for _ in range(args.steps)]
    t = statistics.median(times)
    value = o.n / t
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "images/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * t,
            "ms_per_step_mean": 1000.0 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "resnet50_v1.5_b256", "global_batch": o.n, "per_step_batch": o.n,
                       "sample": f"each step is one pass over a batch-{o.n} sample of the batch-"
                                 f"{GLOBAL_BATCH} workload (same seed, same images 0..{o.n - 1})",
                       "full_workload_batch": GLOBAL_BATCH,
                       "seq_len": None, "parallelism": f"cpu: {o.threads} threads over the batch"},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": o.threads, "kind": "port",
                             "sample": o.sample(len(times), t)},
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def time_on_stream(fn, steps, warmup, stream, flush=None):
    """Mean device ms of fn() over `steps` runs: CUDA events on `stream` around
    each call, an L2-evicting memset before each (outside the events)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / len(evs)


def run_single_workload(args):
    """One of the path's other workloads on one GPU (conv shapes, stem, MatMul, ResNet-18)."""
    import importlib
    import numpy as np
    import torch
    ob = importlib.import_module("onnx-rs_b200")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    h = ob.Handle(0, precision=args.precision)
    ctx = ob.ExecutionContext(h)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    peaks, peak_src = load_peaks()
    tpeak, tpeak_sus = tensor_peaks(peaks, args.precision)
    wl = args.workload
    if wl.startswith("conv:") or wl == "stem":
        if wl == "stem":
            nodes, inits, ins, outs = ob.workloads.stem_conv(0, batch=args.batch if args.batch != GLOBAL_BATCH else 1)
            x = ob.workloads.stem_input(0, ins[0][1][0])
            w, b = inits["W"], inits["B"]
            attrs = {"strides": (2, 2), "pads": (3, 3, 3, 3), "dilations": (1, 1), "group": 1}
        else:
            x, w, b, attrs = ob.workloads.sweep_case(wl[5:], batch=128 if args.batch == GLOBAL_BATCH else args.batch)
        conv = ob.Conv(attrs["strides"], attrs["pads"], attrs["dilations"], attrs["group"], relu=True)
        n, c, hh, ww = x.shape
        cs = c if c % 4 == 0 else (c + 3) // 4 * 4
        xn = np.zeros((n, hh, ww, cs), np.float32)
        xn[..., :c] = x.transpose(0, 2, 3, 1)
        wt = torch.from_numpy(w).cuda()
        bt = torch.from_numpy(b).cuda()
        xt = torch.from_numpy(xn).cuda()
        if cs != c:  # channel-padded NHWC input: pad the weights with zero input channels too
            wp = np.zeros((w.shape[0], cs, w.shape[2], w.shape[3]), np.float32)
            wp[:, :c] = w
            wt = torch.from_numpy(wp).cuda()
        plan = ob.ConvPlan(ctx, conv, (n, hh, ww, cs), wt, bt, layout=1)
        y = torch.empty(plan.out_shape, dtype=torch.float32, device="cuda")
        ms = time_on_stream(lambda: plan.run(xt, y), args.steps, args.warmup, stream, flush)
        _, oh, ow, co = plan.out_shape
        flops = 2.0 * n * oh * ow * co * (c // attrs["group"]) * w.shape[2] * w.shape[3]
        bytes_ = 4.0 * (n * hh * ww * c + w.size + co + n * oh * ow * co)
        name = "stem_conv7x7s2_relu" if wl == "stem" else wl[5:]
        metric, value, unit = "conv TFLOP/s", flops / ms / 1e9, "TFLOP/s"
        plan.close()
    elif wl in ("matmul", "resnet18"):
        if wl == "matmul":
            nodes, inits, ins, outs = ob.workloads.broadcast_matmul_graph(1)
            a, _, _ = ob.workloads.broadcast_matmul(1)
            x = torch.from_numpy(a).cuda()
            flops = 2.0 * 96 * 512 * 3072 * 768
            bytes_ = 4.0 * (a.size + 12 * 768 * 3072 + 3072 + 96 * 512 * 3072)
            name, metric, unit = "broadcast_matmul_add_relu", "MatMul TFLOP/s", "TFLOP/s"
        else:
            bsz = 32 if args.batch == GLOBAL_BATCH else args.batch
            nodes, inits, ins, outs = ob.workloads.resnet18(batch=bsz, seed=2)
            x = torch.from_numpy(ob.workloads.resnet_input(2, bsz)).cuda()
            flops = ob.workloads.resnet18.conv_flops_per_image * bsz
            bytes_ = None
            name, metric, unit = f"resnet18_b{bsz}", "ResNet-18 images/s", "images/s"
        g = ob.Graph(h, nodes, inits, ins, outs)
        yout = g.alloc_outputs(x.device)
        ms = time_on_stream(lambda: g.run([x], yout), args.steps, args.warmup, stream, flush)
        value = flops / ms / 1e9 if unit == "TFLOP/s" else ins[0][1][0] / (ms / 1e3)
        g.close()
    else:
        raise SystemExit(f"unknown workload {wl}")
    tf = flops / ms / 1e9
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "precision": args.precision,
            "data": "synthetic", "config": {"workload": name, "l2": "flushed between timed steps"},
            "roofline": {"tensor": {"achieved": tf, "peak": tpeak, "unit": "TFLOP/s", "frac": tf / tpeak,
                                    "peak_sustained": tpeak_sus, "frac_of_sustained": tf / tpeak_sus},
                         "hbm": None if bytes_ is None else
                         {"achieved": bytes_ / ms / 1e6, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": bytes_ / ms / 1e6 / peaks["hbm_gbs"]},
                         "peak_source": peak_src},
            "gpu_launches": None}
    print(json.dumps(line), flush=True)
    h.close()


def tensor_peaks(peaks, precision):
    """(burst, sustained) dense peaks in TFLOP/s for a precision: tf32 = bf16 / 2;
    the 3xTF32 effective peak = tf32 / 3 (three tf32 MMAs per product)."""
    burst = peaks.get("bf16_tflops")
    sus = peaks.get("bf16_tflops_sustained", burst)
    div = {"3xtf32": 6.0, "tf32": 2.0, "bf16": 1.0, "fp32": 2.0}[precision]
    return burst / div, sus / div


def roofline_of(prof, peaks, peak_src, precision, traffic=None):
    """Roofline of the contraction kernel over one profiled run (per-step CUDA
    events): algorithmic FLOPs / summed device time of the Conv/Gemm steps,
    against the burst peak (the steps last milliseconds, not seconds) with the
    sustained-peak fraction beside it; and achieved GB/s of the memory-bound
    step kinds against the measured HBM copy bandwidth."""
    tc = [p for p in prof if p["kind"] in ("conv_tc", "gemm")]
    tc_ms = sum(p["ms"] for p in tc)
    tc_flops = sum(p["flops"] for p in tc)
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    burst, sus = tensor_peaks(peaks, precision)
    tf32_burst = peaks["bf16_tflops"] / 2.0
    mem = {}
    for kind in ("maxpool", "gap", "convert", "add", "relu", "affine", "conv_direct"):
        ps = [p for p in prof if p["kind"] == kind]
        ms = sum(p["ms"] for p in ps)
        if not ps or ms <= 0:
            continue
        by = sum(p["bytes"] for p in ps)
        mem[kind] = {"launches": len(ps), "ms": round(ms, 4), "bytes": by, "achieved_gbs": by / ms / 1e6,
                     "frac_of_hbm": by / ms / 1e6 / peaks["hbm_gbs"]}
    basis = {"3xtf32": "3xTF32 effective = dense bf16 / 6 (tf32 = bf16 / 2, three tf32 MMAs per product)",
             "tf32": "tf32 dense = dense bf16 / 2", "bf16": "dense bf16",
             "fp32": "fp32 CUDA cores, compared against tf32 dense"}[precision]
    kernel = "igemm_tc3_kernel" if precision != "fp32" else "conv_direct_kernel"
    return {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s",
            "frac": achieved / burst if burst else None,
            "peak_sustained": sus, "frac_of_sustained": achieved / sus if sus else None,
            "traffic": traffic,
            "traffic_note": "DRAM bytes per contraction step (mean over the run's steps, a K-split step's "
                            "launches together) from one ncu DRAM capture of this workload" if traffic else None,
            "kernel": kernel + " (all Conv/Gemm steps of one run)",
            "launches": len(tc), "flops_per_launch": tc_flops / max(1, len(tc)),
            "peak_source": f"{peak_src} ({'MEASURED_PEAKS.json' if peak_src == 'measured' else 'fallback'}): "
                           f"{basis}; `peak` = burst (bf16_tflops), `peak_sustained` = bf16_tflops_sustained",
            "frac_of_raw_tf32": achieved / tf32_burst if precision in ("3xtf32", "tf32") else None,
            "memory_bound": mem}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="resnet50",
                    help="resnet50 (headline) | resnet18 | stem | matmul | conv:<sweep shape name>")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "tf32", "bf16", "fp32"])
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH, help="global batch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fast-modes", action="store_true", help="skip the tf32 / bf16 lines of the headline")
    ap.add_argument("--profile-json", default=None, help="write the per-step profile here")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(args.warmup, 3)
    if args.workload != "resnet50":
        run_single_workload(args)
        return

    import importlib
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ob = importlib.import_module("onnx-rs_b200")
    lo, hi = ob.sharding.shard_range(args.batch, world, rank)
    per_rank = hi - lo
    nodes, inits, ins, outs = ob.workloads.resnet50(batch=per_rank, seed=SEED)
    conv_flops_img = ob.workloads.resnet50.conv_flops_per_image
    xfull = ob.workloads.resnet_input(SEED, args.batch)
    xs = np.ascontiguousarray(xfull[lo:hi])
    del xfull
    peaks, peak_src = load_peaks()

    # one dedicated stream: the library's kernels, the L2 flush and the CUDA
    # events all go on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    xin = torch.from_numpy(xs).cuda()
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def measure(precision, clocks=None):
        """Device time of K graph replays of this rank's slice: CUDA events
        around each step on the launching stream, L2 evicted between steps
        (outside the events), max over ranks.  Also the time from the barrier's
        release to this rank's last completion event (L2 flushes included)."""
        h = ob.Handle(local, precision=precision)
        assert h.stream_ptr == stream.cuda_stream
        g = ob.Graph(h, nodes, inits, ins, outs)
        yout = g.alloc_outputs(xin.device)
        for _ in range(args.warmup):
            g.run([xin], yout)
        h.synchronize()
        prof = g.profile([xin], yout)
        h.synchronize()
        if clocks:
            clocks.start()
            time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        t_rel = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        t_rel.record(stream)
        l0 = h.launches
        for i in range(args.steps):
            flush.zero_()  # evict L2 between timed iterations (outside the events)
            starts[i].record(stream)
            g.run([xin], yout)
            ends[i].record(stream)
        torch.cuda.synchronize()
        launches = h.launches - l0
        clk = clocks.stop() if clocks else None
        step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
        ms = max_over_ranks(sum(step_ms) / len(step_ms))
        from_barrier_ms = max_over_ranks(t_rel.elapsed_time(ends[-1]))
        return {"h": h, "g": g, "yout": yout, "prof": prof, "ms": ms, "launches": launches, "clocks": clk,
                "from_barrier_ms": from_barrier_ms}

    m = measure(args.precision, ClockSampler(local))
    h, g, prof, ms = m["h"], m["g"], m["prof"], m["ms"]
    stats = g.stats()
    value = args.batch / (ms / 1000.0)

    # ---- end to end through the public host-buffer API
    hin = torch.from_numpy(xs).pin_memory()
    hout = torch.empty(g.output_shapes[0], dtype=torch.float32).pin_memory()
    for _ in range(2):
        g.run_host([hin], [hout])
    barrier()
    torch.cuda.synchronize()
    t_e2e = []
    for _ in range(args.steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.run_host([hin], [hout])
        e1.record(stream)
        e1.synchronize()
        t_e2e.append(e0.elapsed_time(e1))
    barrier()
    e2e_single_ms = max_over_ranks(sum(t_e2e) / len(t_e2e))
    # the same K steps as one pipelined sequence of host batches: every step
    # still copies its whole input from pinned host memory and its logits back,
    # but batch b+1's input copy overlaps batch b's compute
    hin2 = [hin, torch.from_numpy(xs.copy()).pin_memory()]
    houts = [[torch.empty(g.output_shapes[0], dtype=torch.float32).pin_memory()] for _ in range(max(2, args.steps))]
    g.run_host_pipelined([[hin2[b % 2]] for b in range(2)], houts[:2])  # warm-up
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.run_host_pipelined([[hin2[b % 2]] for b in range(args.steps)], houts[:args.steps])
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = args.batch / (e2e_ms / 1000.0)

    traffic = TRAFFIC_PER_LAUNCH_3XTF32 if args.precision == "3xtf32" and args.batch == 256 else None
    roofline = roofline_of(prof, peaks, peak_src, args.precision, traffic)
    by_kind = {}
    for p in prof:
        d = by_kind.setdefault(p["kind"], {"n": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        d["n"] += 1
        d["ms"] += p["ms"]
        d["flops"] += p["flops"]
        d["bytes"] += p["bytes"]
    prof_total = sum(p["ms"] for p in prof)
    if args.profile_json and rank == 0:
        with open(args.profile_json, "w") as f:
            json.dump({"steps": prof, "by_kind": by_kind, "stats": stats}, f, indent=1)
    g.close()
    h.close()

    # ---- the fast modes, separately reported: same workload, same timing
    fast = {}
    if args.precision == "3xtf32" and not args.no_fast_modes:
        for prec in ("tf32", "bf16"):
            fm = measure(prec)
            fast[prec] = {"metric": METRIC_FAST[prec], "value": args.batch / (fm["ms"] / 1000.0),
                          "unit": "images/s", "ms_per_step": fm["ms"], "gpu_launches": int(fm["launches"]),
                          "roofline": roofline_of(fm["prof"], peaks, peak_src, prec)}
            fm["g"].close()
            fm["h"].close()

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(steps=1, min_seconds=10.0)
        line = {
            "metric": METRIC if args.precision == "3xtf32" else METRIC_FAST[args.precision],
            "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32" if args.precision in ("3xtf32", "fp32") else args.precision,
            "precision": args.precision, "data": "synthetic",
            "config": {"workload": "resnet50_v1.5_b256", "global_batch": args.batch, "per_gpu_batch": per_rank,
                       "seq_len": None, "parallelism": f"dp{world} (batch split, weights replicated)",
                       "l2": "flushed between timed steps (2x L2 memset outside the events)",
                       "conv_gflop_per_image": conv_flops_img / 1e9},
            "from_barrier": {"value": args.batch * args.steps / (m["from_barrier_ms"] / 1000.0),
                             "unit": "images/s",
                             "note": "all K steps from the host barrier's release to the last rank's last "
                                     "completion event (CUDA events, max over ranks), L2 flushes included"},
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": int(xs.nbytes) * world,
                    "mode": "onnxb200_graph_run_host_pipelined over the timed steps (each step's input "
                            "copy overlaps the previous step's compute)",
                    "unpipelined_value": args.batch / (e2e_single_ms / 1000.0),
                    "d2h_bytes_per_step": int(hout.numel() * 4) * world},
            "gpu_launches": int(m["launches"]),
            "kernels_per_step": stats["kernels_per_run"],
            "roofline": roofline,
            "fast_modes": fast or None,
            "profile_ms_by_kind": {k: round(v["ms"], 3) for k, v in by_kind.items()},
            "profile_total_ms": prof_total,
            "clocks": m["clocks"],
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
