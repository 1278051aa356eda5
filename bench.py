"""Benchmark: recognized lines/sec (48x320 FP16) of the full recognizer.

One step = one forward of BASELINE config 4 on a batch of 512 synthetic line
images per GPU (HGNet-style backbone, SVTR neck, fused CTC vocabulary
projection + argmax, device CTC collapse) through the Model ABI v2 shell and
the head C-ABI. Each GPU runs an independent replica (request-batch data
parallelism, no collective on the hot path; torch.distributed only
synchronises the timing). `value` is the whole-job lines/s with inputs
resident in HBM; `e2e` repeats the measurement with the pinned-host input
copied in and the decoded tokens copied out every step.

`--impl reference` times the CPU restatement of the same forward (the
reference has no CPU implementation of its layer path; the oracle port in
oracle/ is the CPU baseline) on rank 0 only.
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
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "ppocrv6-native-server_b200"))
sys.path.insert(0, str(REPO))

METRIC = "recognized lines/sec (48x320 FP16)"
UNIT = "lines/s"
MODEL = "rec_b512"
LINES = 512
H, W = 48, 320
SEED = 20261201


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def cpu_port_forward(lines_needed: int, budget_s: float = 20.0):
    """Times the oracle's CPU restatement of the recognizer (torch fp32 with
    the same fp16 storage points) on a bounded sample of the batch; returns
    (lines/s, lines timed, threads)."""
    import numpy as np
    import torch

    from ppocr_b200 import models
    from oracle import models as om

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g, out = models.graph("rec_b2")
    x = np.random.default_rng(SEED).uniform(-1, 1, (2, 3, H, W)).astype(np.float32)
    t0 = time.perf_counter()
    om.run_graph(g, x, out)
    one = time.perf_counter() - t0  # 2 lines, includes first-touch costs
    done, elapsed = 2, one
    while elapsed < budget_s and done < lines_needed:
        t0 = time.perf_counter()
        om.run_graph(g, x, out)
        elapsed += time.perf_counter() - t0
        done += 2
    return done / elapsed, done, threads


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    per_step = []
    lines_per_step = 4
    threads = os.cpu_count() or 1
    total = args.warmup + args.steps
    import numpy as np
    import torch

    from ppocr_b200 import models
    from oracle import models as om

    torch.set_num_threads(threads)
    g, out = models.graph("rec_b2")
    x = np.random.default_rng(SEED).uniform(-1, 1, (2, 3, H, W)).astype(np.float32)
    for i in range(total):
        t0 = time.perf_counter()
        for _ in range(lines_per_step // 2):
            om.run_graph(g, x, out)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            per_step.append(dt)
    t = sum(per_step)
    value = lines_per_step * len(per_step) / t
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * t / len(per_step), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded U(-1,1) line images, random-init weights)",
        "config": {"workload": "config 4 recognizer forward (same graph and weights), CPU restatement "
                               "(oracle/ port; the reference has no CPU layer path)",
                   "lines_per_step": lines_per_step},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{lines_per_step} lines per step (a bounded sample of the 512-line batch)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def b200_arm(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from ppocr_b200 import capi, pipeline

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    lib = capi.load()
    rec = pipeline.LineRecognizer(MODEL, dev)
    rng = np.random.default_rng(SEED + rank)
    x_host = torch.from_numpy(rng.uniform(-1, 1, (LINES, H, W, 3)).astype(np.float16)).pin_memory()
    x_dev = x_host.to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    stream = rec.stream
    op_names = rec.model.lib.op_names(rec.model.handle)
    launches_per_step = len(op_names) + 1 + 2 + 1  # graph ops + input staging + head (2) + collapse

    # ---- device-resident timing
    for _ in range(args.warmup):
        rec.enqueue(x_dev)
    stream.synchronize()
    assert lib.ppocr_b200_device_error() == 0, "kernel wait timed out during warm-up"
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.zero_()
                starts[i].record(stream)
            rec.enqueue(x_dev)
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(step_ms))
    value = world * LINES * args.steps / (total_ms / 1e3)

    # ---- end to end: pinned host in, tokens out, every step
    out_ids = torch.empty(LINES, rec.T, dtype=torch.int32).pin_memory()
    out_len = torch.empty(LINES, dtype=torch.int32).pin_memory()
    out_sc = torch.empty(LINES, dtype=torch.float32).pin_memory()
    x_stage = torch.empty_like(x_dev)
    for _ in range(2):
        with torch.cuda.stream(stream):
            x_stage.copy_(x_host, non_blocking=True)
        rec.enqueue(x_stage)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
    for _ in range(args.steps):
        with torch.cuda.stream(stream):
            x_stage.copy_(x_host, non_blocking=True)
        rec.enqueue(x_stage)
        with torch.cuda.stream(stream):
            out_ids.copy_(rec.out_ids, non_blocking=True)
            out_len.copy_(rec.out_len, non_blocking=True)
            out_sc.copy_(rec.out_score, non_blocking=True)
    with torch.cuda.stream(stream):
        e1.record(stream)
    stream.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * LINES * args.steps / (e2e_ms / 1e3)
    h2d = x_host.numel() * x_host.element_size()
    d2h = out_ids.numel() * 4 + out_len.numel() * 4 + out_sc.numel() * 4

    # ---- roofline of the dominant kernel (stage-4 3x3 implicit GEMM)
    prof = [rec.model.lib.profile(rec.model.handle) for _ in range(3)]
    per_op = [min(p[i] for p in prof) for i in range(len(op_names))]
    dom = max(range(len(per_op)), key=lambda i: per_op[i])
    # algorithmic flops of that op, from the graph's layer table
    from ppocr_b200 import models
    g, _ = models.graph(MODEL)
    flops = op_flops(g, dom)
    peak_tf, peak_hbm, peak_kind = peaks()
    achieved = flops / (per_op[dom] / 1e3) / 1e12 if flops else None
    traffic = None
    tf = REPO / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(op_names[dom] + f"#{dom}")

    cpu = None
    if rank == 0:
        cpu_value, cpu_lines, cores = cpu_port_forward(8)
        cpu = {"value": round(cpu_value, 3), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{cpu_lines} lines of the batch through the oracle's CPU restatement "
                         f"(torch fp32, same graph and weights)"}
    gpu_launches = launches_per_step * args.steps
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded U(-1,1) FP16 NHWC line images, seeded random-init weights)",
            "config": {"workload": "BASELINE config 4: full recognizer forward, 512 lines/GPU of 48x320, "
                                   "HGNet-style backbone 48-128-512-1024-2048 + SVTR neck dim 120 x2 + CTC "
                                   "projection V=18385 with fused argmax + device collapse",
                       "lines_per_gpu": LINES, "parallelism": f"replicas x{world} (no collective)",
                       "l2": "flushed between timed steps (256 MB write outside the timed events)"},
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "tensor", "kernel": f"{op_names[dom]}#{dom}",
                         "achieved": round(achieved, 1) if achieved else None, "peak": peak_tf,
                         "unit": "TFLOP/s", "frac": round(achieved / peak_tf, 4) if achieved else None,
                         "peak_source": f"bf16_tflops of {peak_kind} peaks (fp16 dense rate is the same)",
                         "traffic": traffic, "launch_ms": round(per_op[dom], 4), "flops": flops},
            "cpu_baseline": cpu,
            "gpu_launches": gpu_launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    rec.close()
    if world > 1:
        dist.destroy_process_group()


def op_flops(g, index: int) -> float | None:
    """2*M*N*K of a GEMM-like layer in the generated graph (op list order)."""
    layer = g.layers[index] if index < len(g.layers) else None
    if not layer:
        return None
    if layer["op"] == "conv":
        out = g.tensors[layer["out"]].shape  # NHWC
        w = g.tensors[layer["w"]].const.shape
        if layer["groups"] != 1:
            return 2.0 * out[0] * out[1] * out[2] * out[3] * w[1] * w[2]
        return 2.0 * out[0] * out[1] * out[2] * out[3] * w[1] * w[2] * w[3]
    if layer["op"] == "gemm":
        out = g.tensors[layer["out"]].shape
        w = g.tensors[layer["w"]].const.shape
        rows = 1
        for s in out[:-1]:
            rows *= s
        return 2.0 * rows * w[0] * w[1]
    return None


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()
