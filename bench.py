#!/usr/bin/env python3
"""Throughput benchmark of the B200 inference backend (one JSON line on rank 0).

Workload (default): ResNet-50 classification forward, batch 512 of 3x224x224 float32 NCHW input
N(0,1) seed 11, inference-mode BatchNorm, 1000-way FC; synthetic random-init weights (no datasets or
checkpoints exist offline). With --gpus N (launched by torchrun, one process per GPU) the 512-image
batch is sharded 512/N per GPU with replicated weights and no collective ("strong" scaling).

  value  device time: inputs resident in HBM, CUDA events around K replays of the captured kernel
         sequence on the launching stream; whole-job images/s = 512 / max-over-ranks time.
  e2e    the same metric through the plugin interface with host buffers: each step wraps the
         pageable host batch (WrapTensor, no copy) and calls B200InferenceSession.Run, which stages
         it through page-locked memory, copies it to the device, computes and copies the logits back.

--impl reference times the oracle (the CPU restatement of the reference's ONNX Runtime CPU path)
on the host cores instead, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (emit config, batch, unit label)
    "resnet50": ("resnet50", 512),
    "resnet18": ("resnet18", 256),
    "mlp": ("mlp", 8192),
    "stacked_linear": ("stacked_linear", 4096),
    "retinanet": ("retinanet", 16),
    "retinanet_gn": ("retinanet_gn", 16),   # adjacent model: GroupNorm heads (RetinaNetResNet50)
    "vit_base": ("vit_base", 1),            # adjacent model: ViT-B/16, batch 1 as its graph allows
}
METRIC = "ResNet-50 images/sec at 1/2/4/8 B200; % tensor-pipe peak; vs ORT CPU"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region (200 ms period)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[2:]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}


def cpu_baseline(case, sample, budget_s=20.0):
    """The oracle (torch-CPU fp32 restatement of the ORT-CPU path) timed on the first `sample`
    images of the workload's batch. Also returns the oracle's outputs for those images, the
    reference the GPU's outputs of the same rows are checked against."""
    import torch
    from oracle.interp import Interpreter
    cores = len(os.sched_getaffinity(0))
    it = Interpreter(case.model, "fp32", threads=cores)
    feed = {n: (a[:sample] if a.ndim and a.shape[0] == case.inputs[0][1].shape[0] else a) for n, a in case.inputs}
    outs = it.run(feed, case.output_names)   # (also the warm-up run)
    n, t0 = 0, time.perf_counter()
    while True:
        it.run(feed)
        n += 1
        if time.perf_counter() - t0 > budget_s / 2 or n >= 3:
            break
    dt = (time.perf_counter() - t0) / n
    return ({"value": sample / dt, "unit": "images/s", "cores": torch.get_num_threads(), "kind": "port",
             "sample": f"{sample} images of the same workload, oracle/interp.py fp32 (torch CPU), "
                       f"mean of {n} runs"}, outs)


def make_case(name, batch):
    from shorokoo_b200.emit import graphs
    cfg, _ = WORKLOADS[name]
    return graphs.build(cfg, batch=batch)


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    name = args.workload
    batch = WORKLOADS[name][1]
    sample = args.ref_sample
    import torch
    from oracle.interp import Interpreter
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    case = make_case(name, sample)
    it = Interpreter(case.model, "fp32", threads=cores)
    feed = dict(case.inputs)
    for _ in range(args.warmup):
        it.run(feed)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        it.run(feed)
    dt = (time.perf_counter() - t0) / args.steps
    val = sample / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{name} bs{batch} (timed on a {sample}-image sample per step)",
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": val, "unit": "images/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{sample} images per step; ONNX Runtime is not installable offline, so the "
                                   f"oracle's torch-CPU fp32 restatement of its CPU path stands in"},
        "e2e": {"value": val, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="resnet50", choices=sorted(WORKLOADS))
    ap.add_argument("--ref-sample", type=int, default=8, help="images per step of the CPU reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--precision", default="bf16", choices=["bf16", "tf32", "tf32x3"],
                    help="tensor-core operand precision (tf32: the accuracy mode)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's global batch (small cases for profiler captures)")
    ap.add_argument("--devices", type=int, default=1,
                    help="one session over this many GPUs of this process (the library's own batch sharding, "
                         "one host thread per device; what SHOROKOO_B200_DEVICES gives a plugin caller)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.devices > 1 and world > 1:
        ap.error("--devices N runs one process over N GPUs; do not combine it with torchrun ranks")

    if world > 1 and "SHOROKOO_B200_HOST_THREADS" not in os.environ:
        # one process per GPU shares the host: each stages its shard with its share of the cores
        os.environ["SHOROKOO_B200_HOST_THREADS"] = str(max(2, len(os.sched_getaffinity(0)) // world))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))   # host barrier / max only
    from shorokoo_b200 import B200InferenceSessionFactory

    name = args.workload
    total = args.batch or WORKLOADS[name][1]
    per = total // world + (1 if rank < total % world else 0)
    begin = rank * (total // world) + min(rank, total % world)
    full = make_case(name, total) if world == 1 else None
    case = full if full is not None else make_case(name, total)
    # this rank's contiguous shard of the batch
    inputs = [(n, a[begin:begin + per] if a.ndim and a.shape[0] == total else a) for n, a in case.inputs]
    f = B200InferenceSessionFactory(num_devices=args.devices, first_device=local, precision=args.precision)
    sess = f.CreateSession(case.model)
    feeds = {n: f.CreateTensor(a) for n, a in inputs}
    st = sess.stats(feeds)
    macs_per_img = case.macs / total
    n_dev = int(st["devices"])   # devices the session's plans run on (1 unless --devices)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    # ---- device-resident throughput (value) ----
    barrier()
    with ClockSampler(local) as clk:
        ms = max(sess.time_device(feeds, warmup=args.warmup, iters=args.steps))   # max over the session's devices
        barrier()
        # ---- end to end through the plugin interface (e2e): every step hands the host batch to the
        # library the way the reference's CreateTensor<T> does (aliasing the caller's array, no
        # copy: WrapTensor), runs it (Run stages the pageable input through page-locked slots, copies
        # to the device, computes, copies the outputs back) and releases the values ----
        def e2e_step(fresh):
            fd = {n: f.WrapTensor(a) for n, a in inputs} if fresh else feeds
            outs = sess.Run(fd, case.output_names)
            for o in outs:
                o.Dispose()
            if fresh:
                for v in fd.values():
                    v.Dispose()

        e2e = {}
        for fresh in (True, False):   # (False: input already in library page-locked memory)
            for _ in range(args.warmup):
                e2e_step(fresh)
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                e2e_step(fresh)
            torch.cuda.synchronize()
            e2e[fresh] = (time.perf_counter() - t0) / args.steps
            barrier()
        e2e_s = e2e[True]
    clocks = clk.summary()
    t_max = ms
    e_max = e2e_s
    if world > 1:
        tt = torch.tensor([ms, e2e_s, e2e[False]], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, e_max = float(tt[0]), float(tt[1])
        e2e[False] = float(tt[2])

    # ---- roofline of the dominant kernel (tensor-core implicit GEMM), timed per launch ----
    prof = sess.profile(feeds, iters=3)
    tc_kinds = ("conv", "gemm", "attention")   # the tcgen05 launches
    tc_ms = sum(v for k, v in prof if k.split()[0] in tc_kinds)
    tc_launches = sum(1 for k, _ in prof if k.split()[0] in tc_kinds)
    all_ms = sum(v for _, v in prof)
    peak_tflops, peak_hbm, peak_kind = measured_peaks()
    peak_note = f"{peak_kind} bf16 dense (burst)"
    if args.precision in ("tf32", "tf32x3"):   # the dense TF32 tensor rate is half the bf16 rate
        peak_tflops /= 2
        peak_note = f"half the {peak_kind} bf16 dense burst (TF32 dense rate)"
        if args.precision == "tf32x3":   # three MMAs per algorithmic one
            peak_tflops /= 3
            peak_note += ", divided by the three MMAs per K slice of TF32x3"
    # (the profile times device 0's plan: its share of the session's MACs)
    achieved = 2.0 * st["macs"] / n_dev / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get(name) if not args.batch and args.precision == "bf16" else None

    wrapped = {n: f.WrapTensor(a) for n, a in inputs}   # the e2e path's inputs
    h2d, d2h = sess.transfer_bytes(wrapped)
    for v in wrapped.values():
        v.Dispose()
    outs = sess.Run(feeds, case.output_names)
    gpu_head = [o.numpy()[:8] for o in outs]   # this rank's first rows, for the parity check
    for o in outs:
        o.Dispose()

    if rank == 0:
        value = total / (t_max / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world * n_dev, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic (seeded inputs, random-init weights)",
            "config": {"workload": f"{name} forward, batch {total} ({-(-per // n_dev)}/GPU), 3x224x224 fp32 NCHW input"
                       if name.startswith("resnet") else f"{name} forward, batch {total}",
                       "global_batch": total,
                       "parallelism": (f"batch-sharded x{world}, replicated weights, no collective" if n_dev == 1 else
                                       f"one session over {n_dev} devices in one process: the library shards the "
                                       f"batch (contiguous rows, replicated weights, no collective), one host thread "
                                       f"and one staging pipeline per device"),
                       "l2": "inputs larger than L2 (the 308 MB input and a multi-GB activation arena per step)",
                       "precision": {"bf16": "bf16 operands", "tf32": "fp32 operands read as TF32",
                                     "tf32x3": "error-compensated TF32 (hi*hi + hi*lo + lo*hi)"}[args.precision]
                                    + ", fp32 accumulate"},
            "e2e": {"value": total / e_max, "unit": "images/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world,
                    "timing": "host wall clock per step around WrapTensor of the pageable host batch (no copy, "
                              "as CreateTensor<T> aliases a managed array) + Run (staging through page-locked "
                              "memory, the float32 input converted to bf16 there as the plan only reads it as "
                              "bf16, H2D, kernels, D2H of the outputs into host memory) + release; byte counts "
                              "are the copies Run makes"},
            "e2e_pinned_input": {"value": total / e2e[False], "unit": "images/s",
                                 "timing": "Run alone on an input already in library page-locked memory "
                                           "(CreateTensor outside the timed region)"},
            "gpu_launches": int(st["launches"]) * args.steps * world,   # (summed over the session's devices)
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                         "frac": achieved / peak_tflops, "traffic": traffic,
                         "traffic_note": "DRAM bytes read + written per step by these launches, one ncu capture of "
                                         "this workload (profiles/resnet50_bs512_dram_launch_list.md); algorithmic "
                                         "minimum ~23.2e9" if traffic else None,
                         "kernel": f"tcgen05 implicit GEMM (conv_gemm_kernel, conv_pair_kernel on CTA pairs, stem and halo "
                                   f"kernels), {tc_launches} launches/step, "
                                   f"{tc_ms:.3f} of {all_ms:.3f} ms per step timed per launch with CUDA events",
                         "peak_kind": peak_note},
            "clocks": clocks,
            "flops_per_image": 2 * macs_per_img,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                sample = 1 if name.startswith("retinanet") else min(8, total)   # (RetinaNet: ~15 s per image on CPU)
                line["cpu_baseline"], ref = cpu_baseline(case, sample=sample)
                gate = 1e-2 if args.precision == "bf16" else 2e-3
                errs = {}
                for nm, g, r in zip(case.output_names, gpu_head, ref):
                    g = np.asarray(g[:sample], np.float64)
                    r = np.asarray(r, np.float64)
                    errs[nm] = float(np.abs(g - r).max() / max(float(np.abs(r).max()), 1e-30))
                line["parity"] = {"rows": f"0..{sample - 1} of the timed batch (outputs of a Run of the timed session)",
                                  "reference": "oracle fp32 (the CPU baseline run)", "normwise": errs,
                                  "gate": gate, "pass": all(e <= gate for e in errs.values())}
            except Exception as e:   # reported, never fatal for the GPU number
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(line), flush=True)
    sess.Dispose()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
