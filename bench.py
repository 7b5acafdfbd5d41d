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
             effective 3xTF32 peak = measured dense bf16 / 6
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
# DRAM bytes per igemm_tc3_kernel launch, mean over the 54 launches of one
# batch-256 3xTF32 run: ncu dram__bytes_read.sum + dram__bytes_write.sum
# (profiles/resnet50_b256_launch_list.md).
TRAFFIC_PER_LAUNCH_3XTF32 = 467.5e6
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


def cpu_baseline(steps=1, images=None, min_seconds=0.0, max_steps=8):
    """Oracle ResNet-50 (3xTF32 path's reference semantics, fp32) on host cores:
    every host thread this process may use (at most 64, so that the sample's
    activations stay a few GB), one image per thread; at least `steps` runs and
    more (up to `max_steps`) until `min_seconds` of work have been timed."""
    import importlib
    from oracle import oracle as orc
    ob = importlib.import_module("onnx-rs_b200")
    orc.build()
    try:
        avail = len(os.sched_getaffinity(0))
    except AttributeError:
        avail = os.cpu_count() or 1
    threads = max(1, min(avail, 64))
    n = images or threads
    nodes, inits, ins, outs = ob.workloads.resnet50(batch=n, seed=SEED)
    x = ob.workloads.resnet_input(SEED, n)
    times = []
    while len(times) < steps or (sum(times) < min_seconds and len(times) < max_steps):
        t0 = time.perf_counter()
        orc.run_graph(nodes, inits, {"X": x}, outs, nthreads=threads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": n / t, "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"ResNet-50 v1.5 batch {n} (of 256), seed {SEED}, oracle C restatement of the reference's "
                      f"CPU operators (im2col+GEMM / direct conv, batch split over {threads} of {avail} "
                      f"available host threads), median of {len(times)} run(s), {t:.2f} s each"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    res = None
    times = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(steps=1)
        if i >= args.warmup:
            times.append(r)
        res = r
    vals = [r["value"] for r in times]
    value = statistics.median(vals)
    ms = 1000.0 * GLOBAL_BATCH / value
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "images/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "resnet50_v1.5_b256", "global_batch": GLOBAL_BATCH,
                                            "seq_len": None, "parallelism": "cpu threads over batch"},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": res["cores"], "kind": res["kind"],
                             "sample": res["sample"]},
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
    bf16 = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    tpeak = {"3xtf32": bf16 / 6.0, "tf32": bf16 / 2.0, "bf16": bf16, "fp32": bf16 / 2.0}[args.precision]
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
            "roofline": {"tensor": {"achieved": tf, "peak": tpeak, "unit": "TFLOP/s", "frac": tf / tpeak},
                         "hbm": None if bytes_ is None else
                         {"achieved": bytes_ / ms / 1e6, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": bytes_ / ms / 1e6 / peaks["hbm_gbs"]},
                         "peak_source": peak_src},
            "gpu_launches": None}
    print(json.dumps(line), flush=True)
    h.close()


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

    # one dedicated stream: the library's kernels, the L2 flush and the CUDA
    # events all go on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    h = ob.Handle(local, precision=args.precision)
    assert h.stream_ptr == stream.cuda_stream
    g = ob.Graph(h, nodes, inits, ins, outs)
    xin = torch.from_numpy(xs).cuda()
    yout = g.alloc_outputs(xin.device)

    for _ in range(args.warmup):
        g.run([xin], yout)
    h.synchronize()
    prof = g.profile([xin], yout)
    h.synchronize()
    stats = g.stats()

    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    l0 = h.launches
    for i in range(args.steps):
        flush.zero_()  # evict L2 between timed iterations (outside the events)
        starts[i].record(stream)
        g.run([xin], yout)
        ends[i].record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = h.launches - l0
    h.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms_local = sum(step_ms) / len(step_ms)
    ms = max_over_ranks(ms_local)
    clk = clocks.stop()
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
    houts = [[torch.empty(g.output_shapes[0], dtype=torch.float32).pin_memory()] for _ in range(args.steps)]
    g.run_host_pipelined([[hin2[b % 2]] for b in range(2)], houts[:2])  # warm-up
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.run_host_pipelined([[hin2[b % 2]] for b in range(args.steps)], houts)
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = args.batch / (e2e_ms / 1000.0)

    # ---- roofline of the tcgen05 kernel over one run (per-step CUDA events)
    peaks, peak_src = load_peaks()
    tc = [p for p in prof if p["kind"] in ("conv_tc", "gemm")]
    tc_ms = sum(p["ms"] for p in tc)
    tc_flops = sum(p["flops"] for p in tc)
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    by_kind = {}
    for p in prof:
        d = by_kind.setdefault(p["kind"], {"n": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        d["n"] += 1
        d["ms"] += p["ms"]
        d["flops"] += p["flops"]
        d["bytes"] += p["bytes"]
    prof_total = sum(p["ms"] for p in prof)
    bf16 = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    if args.precision == "3xtf32":
        peak = bf16 / 6.0
        basis = "3xTF32 effective = sustained dense bf16 / 6 (tf32 = bf16/2, three MMAs per product)"
    elif args.precision == "tf32":
        peak = bf16 / 2.0
        basis = "tf32 dense = sustained dense bf16 / 2"
    elif args.precision == "bf16":
        peak = bf16
        basis = "sustained dense bf16"
    else:
        peak = bf16 / 2.0
        basis = "fp32 CUDA cores compared against tf32 dense"
    n_tc_launch = len(tc)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if peak else None,
                "traffic": TRAFFIC_PER_LAUNCH_3XTF32 if args.precision == "3xtf32" and args.batch == 256 else None,
                "traffic_note": "DRAM bytes per conv launch from one ncu capture of this workload"
                                " (bytes, mean over the run's launches)",
                "kernel": ("igemm_tc_kernel" if args.precision == "bf16" else "igemm_tc3_kernel")
                + " (all Conv/Gemm launches of one run)",
                "launches": n_tc_launch, "flops_per_launch": tc_flops / max(1, n_tc_launch),
                "peak_source": f"{peak_src}: {basis}",
                "frac_of_raw_tf32": (3 * achieved / (bf16 / 2.0)) if args.precision == "3xtf32" else None}
    if args.profile_json and rank == 0:
        with open(args.profile_json, "w") as f:
            json.dump({"steps": prof, "by_kind": by_kind, "stats": stats}, f, indent=1)

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
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": int(xs.nbytes) * world,
                    "mode": "onnxb200_graph_run_host_pipelined over the timed steps (each step's input "
                            "copy overlaps the previous step's compute)",
                    "unpipelined_value": args.batch / (e2e_single_ms / 1000.0),
                    "d2h_bytes_per_step": int(hout.numel() * 4) * world},
            "gpu_launches": int(launches),
            "kernels_per_step": stats["kernels_per_run"],
            "roofline": roofline,
            "profile_ms_by_kind": {k: round(v["ms"], 3) for k, v in by_kind.items()},
            "profile_total_ms": prof_total,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    g.close()
    h.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
