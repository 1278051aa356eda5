"""Benchmark: recognized lines/sec (48x320 FP16) and page p50 latency @960^2.

One step = one forward of BASELINE config 4 on a batch of 512 synthetic line
images per GPU (HGNet-style backbone, SVTR neck, fused CTC vocabulary
projection + argmax, device CTC collapse) through the Model ABI v2 shell and
the head C-ABI. Each GPU runs an independent replica (request-batch data
parallelism, no collective on the hot path; torch.distributed only
synchronises the timing and gathers per-rank figures). `value` is the
whole-job lines/s with inputs resident in HBM; `e2e` repeats the measurement
with the pinned-host input copied in and the decoded tokens copied out every
step, through the double-buffered LineStream (the copy of step k+1 runs
during step k).

The second half of the BASELINE metric, page p50 latency, follows on every
rank (`page_p50_ms`, the max over ranks of each rank's p50 over
--page-runs runs of config 5: 8 pages of 960^2 through the detector +
binarize and 512 line crops through the recognizer + head + collapse; pages
sharded: each GPU serves its own 8). `--scaling strong` keeps 512 lines in
total (512/N per GPU) instead of 512 per GPU. `per_rank` lists each rank's
step time, median SM clock and page p50, to name a straggler.

The CPU baseline (`cpu_baseline`, the oracle's CPU restatement on the host
cores) is timed on rank 0 before the ranks join the process group.
`--impl reference` times the same CPU restatement (the reference has no CPU
implementation of its layer path; the oracle port in oracle/ is the CPU
baseline) on rank 0 only. `--config c1|c2|c3|c5|pre|post` measures the other
configurations on one GPU.

Side by side on the same B200: the default line's `abi_forward` times this
repository's recognizer (B=512) and detector (8 pages of 960^2) libraries
through ppocr_model_enqueue, the reference-facing Model ABI call, and the
reference arm's `reference_gpu` times the reference's own compiled runtime
(model_library.cu + runtime.cuh on cuDNN / cuBLAS / CUTLASS, built unmodified
under oracle/_ref around the exporter-vocabulary twin of the same graph)
through the same call.
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
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default 20 for c4; 200 for the sub-millisecond c1-c3 steps and the "
                        "c5 latency distribution)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--model", default=MODEL, choices=["rec_b512", "rec_b256", "rec_b64"],
                   help="compiled recognizer shape of the c4 run (rec_b512 = the benchmark; the smaller "
                        "shapes exist for profiling captures and are named in the output's config)")
    p.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                   help="c4: weak = 512 lines per GPU (rec_b512 on every rank); strong = 512 lines in total split "
                        "over the GPUs (rec_b512/256/128/64 at N = 1/2/4/8)")
    p.add_argument("--no-pages", action="store_true",
                   help="c4: skip the page-latency half of the metric (C5 on every rank after the line timing)")
    p.add_argument("--page-runs", type=int, default=100, help="c4: timed C5 runs per rank for page_p50_ms")
    p.add_argument("--config", default="c4", choices=["c1", "c2", "c3", "c4", "c5", "pre", "post"],
                   help="c4 (default) is the headline recognizer benchmark; c1/c2/c3/c5 measure the other "
                        "BASELINE configurations (CTC head, conv block, neck, page pipeline) on one GPU; pre "
                        "measures the page preprocessing (detector resize/normalize, batched ROI warp); post the DB "
                        "post-processing front end (binarize + connected components with box statistics)")
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
            # The sampler takes a moment to start: wait for its first line so
            # the timed region is covered even when it is short.
            t_end = time.monotonic() + 3.0
            while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.n0 = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            # at least one sample taken after the timed work was issued
            t_end = time.monotonic() + 1.0
            while len(self.lines) <= self.n0 and time.monotonic() < t_end and self.proc.poll() is None:
                time.sleep(0.01)
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


class CpuRecognizer:
    """The oracle's CPU restatement of one recognizer step on two lines:
    graph forward (torch fp32 with the same fp16 storage points), vocabulary
    projection with the head's weights, argmax / softmax-max, and the CTC
    collapse (oracle C restatement)."""

    def __init__(self):
        import ctypes

        import numpy as np
        import torch

        from ppocr_b200 import modelgen, models
        from oracle import layers as L

        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.g, self.out = models.graph("rec_b2")
        self.x = np.random.default_rng(SEED).uniform(-1, 1, (2, 3, H, W)).astype(np.float32)
        spec = models.spec("recognizer")
        hidden, vocab = spec["neck"]["dim"], spec["vocab"]
        w, b = models.head_weights(hidden, vocab)  # the device head's weights (pipeline.Classifier)
        self.w = L.rh(torch.from_numpy(w))
        self.b = L.rh(torch.from_numpy(b))
        self.lib = ctypes.CDLL(str(REPO / "oracle" / "_build" / "liboracle.so"))
        Pv = ctypes.c_void_p
        self.lib.oracle_ctc_collapse.argtypes = [Pv, Pv, ctypes.c_long, ctypes.c_int, ctypes.c_int, Pv, Pv, Pv]
        self.T = 40

    def step(self):
        import numpy as np
        import torch

        from oracle import models as om

        hid, _ = om.run_graph(self.g, self.x, self.out)
        logits = hid.reshape(-1, hid.shape[-1]) @ self.w + self.b
        mx, ids = logits.max(dim=1)
        prob = (1.0 / torch.exp(logits - mx[:, None]).sum(dim=1)).float().numpy()
        ids = ids.to(torch.int32).numpy()
        o_ids = np.empty((2, self.T), np.int32)
        o_len = np.empty(2, np.int32)
        o_sc = np.empty(2, np.float32)
        self.lib.oracle_ctc_collapse(ids.ctypes.data, prob.ctypes.data, 2, self.T, 0, o_ids.ctypes.data,
                                     o_len.ctypes.data, o_sc.ctypes.data)
        return 2


def cpu_port_forward(lines_needed: int, budget_s: float = 20.0):
    """Times the oracle's CPU restatement of the recognizer step on a
    bounded sample of the batch; returns (lines/s, lines timed, threads)."""
    cpu = CpuRecognizer()
    t0 = time.perf_counter()
    done = cpu.step()  # includes first-touch costs
    elapsed = time.perf_counter() - t0
    while elapsed < budget_s and done < lines_needed:
        t0 = time.perf_counter()
        done += cpu.step()
        elapsed += time.perf_counter() - t0
    return done / elapsed, done, cpu.threads


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    per_step = []
    lines_per_step = 4
    total = args.warmup + args.steps
    cpu = CpuRecognizer()
    threads = cpu.threads
    for i in range(total):
        t0 = time.perf_counter()
        for _ in range(lines_per_step // 2):
            cpu.step()
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
        "config": {"workload": "config 4 recognizer step (same graph and weights: forward, vocabulary "
                               "projection, argmax/softmax-max, CTC collapse), CPU restatement (oracle/ port; "
                               "the reference has no CPU layer path)",
                   "lines_per_step": lines_per_step},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{lines_per_step} lines per step (a bounded sample of the 512-line batch)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    # The reference's own GPU layer path on this box, for the side-by-side
    # with this repository's libraries (the b200 arm's `abi_forward`).
    try:
        import torch

        if torch.cuda.is_available():
            _, _, local = dist_env()
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            line["reference_gpu"] = abi_comparison("reference", dev)
        else:
            line["reference_gpu"] = {"unavailable": "no CUDA device"}
    except Exception as exc:  # reported, never fatal to the CPU arm
        line["reference_gpu"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    print(json.dumps(line), flush=True)


STRONG_MODELS = {1: "rec_b512", 2: "rec_b256", 4: "rec_b128", 8: "rec_b64"}


def b200_arm(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from ppocr_b200 import capi, pipeline

    rank, world, local = dist_env()
    # The CPU baselines run first, on rank 0, before any rank joins the
    # process group: the other ranks wait in the rendezvous (no GPU work, no
    # busy barrier), so the host cores are not shared with spinning ranks.
    cpu = cpu_pages = None
    if rank == 0:
        cpu_value, cpu_lines, cores = cpu_port_forward(8)
        cpu = {"value": round(cpu_value, 3), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{cpu_lines} lines of the batch through the oracle's CPU restatement "
                         f"(torch fp32, same graph and weights, vocabulary projection, argmax, collapse), "
                         f"timed before the GPU ranks start"}
        if not args.no_pages:
            cpu_pages = _cpu_c5()
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

    def gather(values: list[float]) -> list[list[float]]:
        t = torch.tensor(values, dtype=torch.float64, device=dev)
        if world == 1:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.tolist() for o in out]

    lib = capi.load()
    strong = args.scaling == "strong"
    if strong:
        if world not in STRONG_MODELS:
            raise SystemExit(f"strong scaling splits 512 lines over 1, 2, 4 or 8 GPUs, not {world}")
        model_name = STRONG_MODELS[world]
    else:
        model_name = args.model
    rec = pipeline.LineRecognizer(model_name, dev)
    LINES = rec.batch
    rng = np.random.default_rng(SEED + rank)
    x_host = torch.from_numpy(rng.uniform(-1, 1, (LINES, H, W, 3)).astype(np.float16)).pin_memory()
    x_dev = x_host.to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    stream = rec.stream
    op_names = rec.model.lib.op_names(rec.model.handle)
    # graph ops after the leading NCHW->NHWC transpose (replaced by a staging
    # copy, no kernel) + vocabulary projection (2 kernels) + collapse (1)
    launches_per_step = sum(1 for n in op_names[1:] if n != "fused") + 2 + 1

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
    rank_total_ms = sum(step_ms)
    total_ms = max_over_ranks(rank_total_ms)
    value = world * LINES * args.steps / (total_ms / 1e3)

    # ---- end to end: pinned host in, tokens out, every step, through the
    # double-buffered LineStream (the copy of step k+1 overlaps step k)
    outs = [(torch.empty(LINES, rec.T, dtype=torch.int32).pin_memory(),
             torch.empty(LINES, dtype=torch.int32).pin_memory(),
             torch.empty(LINES, dtype=torch.float32).pin_memory()) for _ in range(2)]
    out_ids = outs[0][0]
    out_len = outs[0][1]
    out_sc = outs[0][2]
    streamer = pipeline.LineStream(rec)
    streamer.enqueue([x_host] * 2, outs)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
    streamer.enqueue([x_host] * args.steps, [outs[i % 2] for i in range(args.steps)])
    with torch.cuda.stream(stream):
        e1.record(stream)
    stream.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * LINES * args.steps / (e2e_ms / 1e3)
    h2d = x_host.numel() * x_host.element_size()
    d2h = out_ids.numel() * 4 + out_len.numel() * 4 + out_sc.numel() * 4

    # ---- replicas decode one common check batch to identical tokens
    from ppocr_b200.replicas import all_equal_over_ranks, tokens_digest

    x_chk = torch.from_numpy(np.random.default_rng(SEED).uniform(-1, 1, (LINES, H, W, 3))
                             .astype(np.float16)).to(dev)
    rec.enqueue(x_chk)
    chk_ids, chk_len, chk_sc = rec.results(LINES)
    digest = tokens_digest(chk_ids, chk_len, chk_sc)
    identical = all_equal_over_ranks(digest)
    distinct = len(np.unique(np.concatenate([chk_ids[k, :chk_len[k]] for k in range(LINES)])))

    # ---- the CTC head alone (vocabulary projection + merge + collapse)
    head_ms = _event_steps(stream, 10, lambda i: rec.enqueue_head(LINES), flush)
    head_ms = min(head_ms)

    # ---- roofline of the dominant kernel (stage-4 3x3 implicit GEMM)
    prof = [rec.model.lib.profile(rec.model.handle) for _ in range(3)]
    per_op = [min(p[i] for p in prof) for i in range(len(op_names))]
    dom = max(range(len(per_op)), key=lambda i: per_op[i])
    # algorithmic flops of that op, from the graph's layer table
    from ppocr_b200 import models
    g, _ = models.graph(model_name)
    flops = op_flops(g, dom)
    peak_tf, peak_hbm, peak_kind = peaks()
    achieved = flops / (per_op[dom] / 1e3) / 1e12 if flops else None
    traffic = None
    tf = REPO / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(op_names[dom] + f"#{dom}")
    rec.close()
    del flush

    # ---- BASELINE metric, second half: page p50 latency (config 5) on every
    # rank, 8 pages + 512 crops per rank (pages sharded across the GPUs)
    page = None
    if not args.no_pages:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        barrier()
        pg = measure_pages(dev, args.page_runs, max(args.warmup, 3), flush, seed_offset=rank)
        barrier()
        page_p50 = max_over_ranks(pg["p50_ms"])
        page_e2e = max_over_ranks(pg["e2e_p50_ms"])
        page = {"metric": "page p50 latency ms @960^2 (C5: 8 pages -> detector + binarize, 512 line crops "
                          "-> recognizer + head + collapse per GPU)",
                "p50_ms": round(page_p50, 4), "unit": "ms", "higher_is_better": False,
                "pages_per_s": round(world * 8 / (page_p50 / 1e3), 1),
                "p90_ms": pg["p90_ms"], "e2e_p50_ms": round(page_e2e, 4), "runs": pg["runs"],
                "e2e": {"value": round(page_e2e, 4), "unit": "ms", "h2d_bytes_per_step": pg["h2d_bytes_per_run"],
                        "d2h_bytes_per_step": pg["d2h_bytes_per_run"]},
                "roofline": pg["roofline"], "binarize": pg["binarize"],
                "detector_top_ops": pg["detector_top_ops"][:5], "clocks": pg["clocks"],
                "gpu_launches": pg["launches_per_run"] * pg["runs"], "cpu_baseline": cpu_pages}
        rank_page = pg["p50_ms"]
        del flush
    else:
        rank_page = float("nan")

    # ---- the same forwards through the reference-facing Model ABI call, for
    # the side-by-side with the reference's own runtime (--impl reference)
    abi = abi_comparison("b200", dev) if not args.no_pages else None

    csum = clocks.summary()
    per_rank = gather([rank_total_ms / args.steps, csum["sm_mhz"] or 0.0, rank_page])
    gpu_launches = launches_per_step * args.steps
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded U(-1,1) FP16 NHWC line images, seeded random-init weights)",
            "config": {"workload": f"BASELINE config 4: full recognizer forward, {LINES} lines/GPU of 48x320, "
                                   "HGNet-style backbone 48-128-512-1024-2048 + SVTR neck dim 120 x2 + CTC "
                                   "projection V=18385 with fused argmax + device collapse",
                       "model": model_name, "lines_per_gpu": LINES, "lines_total": LINES * world,
                       "parallelism": f"replicas x{world} (no collective)",
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
            "clocks": csum,
            "per_rank": [{"rank": k, "ms_per_step": round(v[0], 4), "sm_mhz": v[1],
                          "page_p50_ms": None if v[2] != v[2] else round(v[2], 4)} for k, v in enumerate(per_rank)],
            "replica_tokens": {"sha256": digest[:16], "identical_across_ranks": identical,
                               "mean_length": round(float(np.mean(chk_len)), 2), "distinct_ids": distinct},
            "head_ms": round(head_ms, 4),
            "ops_ms": {f"{op_names[i]}#{i}": round(per_op[i], 4)
                       for i in sorted(range(len(per_op)), key=lambda i: -per_op[i])[:16]},
        }
        if page is not None:
            line["page_p50_ms"] = page["p50_ms"]
            line["page"] = page
        if abi is not None:
            line["abi_forward"] = abi
        print(json.dumps(line), flush=True)
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
    if layer["op"] == "deconv":  # kernel == stride: one tap per output pixel
        out = g.tensors[layer["out"]].shape
        w = g.tensors[layer["w"]].const.shape  # [Ci, KH, KW, Co]
        return 2.0 * out[0] * out[1] * out[2] * out[3] * w[0]
    if layer["op"] == "gemm":
        out = g.tensors[layer["out"]].shape
        w = g.tensors[layer["w"]].const.shape
        rows = 1
        for s in out[:-1]:
            rows *= s
        return 2.0 * rows * w[0] * w[1]
    return None


# --------------------------------------------------------------------------
# The other BASELINE configurations (one GPU, rank 0). Same timing rules as
# the headline: >= 3 warm-up steps, CUDA events on the launching stream, L2
# flushed (256 MB write) outside the timed events, clocks sampled meanwhile.

CONFIGS = {
    "c1": ("CTC-decoded lines/sec (C1: [32,40,18385] FP16 logits, argmax + softmax-max + collapse)",
           "lines/s", True),
    "c2": ("conv-block images/sec (C2: dw5x5 + pw 64->128 hardswish, [16,48,320,64] FP16 NHWC)",
           "images/s", True),
    "c3": ("neck lines/sec (C3: SVTR neck, 2 blocks, [256,40,120] FP16)", "lines/s", True),
    "c5": ("page p50 latency ms @960^2 (C5: 8 pages -> detector + binarize, 512 line crops -> recognizer)",
           "ms", False),
    "pre": ("preprocessed pages/sec (8 decoded 1080x1920 u8 pages -> 960^2 FP16 NHWC detector input, and 64 "
            "48x320 FP16 NHWC line crops per page by perspective ROI warp)", "pages/s", True),
    "post": ("DB post-processed pages/sec (8 FP32 probability maps 960^2 -> binarize 0.3 -> 8-connected components "
             "with box statistics, max 3000 candidates per page)", "pages/s", True),
}


def _event_steps(stream, steps, body, flush):
    """Per-step device time (ms) of body(i) on `stream`, flush outside."""
    import torch

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        with torch.cuda.stream(stream):
            if flush is not None:
                flush.zero_()
            starts[i].record(stream)
        body(i)
        ends[i].record(stream)
    stream.synchronize()
    return [a.elapsed_time(b) for a, b in zip(starts, ends)]


def abi_forward(so_path, weights_path, dev, steps: int, warmup: int, seed: int = SEED):
    """Device time of one full-batch ppocr_model_enqueue of a Model ABI v2
    library (model_abi.h:11-38), bound through the seven reference symbols
    only, as the reference's catalog loader binds them
    (model_engine_compiled.cpp:43-75): f32 NCHW input resident in HBM, L2
    flushed by a 256 MB write outside the timed events, CUDA events on the
    enqueue stream. The same call times this repository's libraries and the
    reference's own compiled runtime, so the two are compared on one
    interface. Returns {"batch", "ms" (median), "ms_min", "output_shape"}."""
    import ctypes
    from ctypes import c_char_p, c_int, c_size_t, c_void_p

    import numpy as np
    import torch

    from ppocr_b200 import capi

    dll = ctypes.CDLL(str(so_path), mode=ctypes.RTLD_LOCAL)
    sig = {"ppocr_model_info": (c_void_p, []), "ppocr_model_load_weights": (c_void_p, [c_char_p]),
           "ppocr_model_create": (c_void_p, [c_void_p, c_void_p, c_size_t, c_void_p]),
           "ppocr_model_enqueue": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
           "ppocr_model_destroy": (None, [c_void_p]), "ppocr_model_error": (c_char_p, []),
           "ppocr_model_release_resources": (None, [c_void_p])}
    for name, (res, args) in sig.items():
        fn = getattr(dll, name)
        fn.restype, fn.argtypes = res, args
    info = capi.PpocrModelInfo.from_address(dll.ppocr_model_info())
    resources = capi.PpocrModelResources()
    weights = dll.ppocr_model_load_weights(str(weights_path).encode())
    if not weights:
        raise RuntimeError(dll.ppocr_model_error().decode())
    scratch = torch.empty(info.scratch_bytes, dtype=torch.uint8, device=dev)
    handle = dll.ppocr_model_create(weights, scratch.data_ptr(), info.scratch_bytes, ctypes.byref(resources))
    if not handle:
        raise RuntimeError(dll.ppocr_model_error().decode())
    in_shape = tuple(info.input_shape)
    out_shape = tuple(info.output_shape[: info.output_rank])
    batch = in_shape[0]
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.uniform(-1, 1, in_shape).astype(np.float32)).to(dev)
    out = torch.empty(out_shape, dtype=torch.float16 if info.output_element_bytes == 2 else torch.float32,
                      device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    s = c_void_p(stream.cuda_stream)

    def body(i):
        if dll.ppocr_model_enqueue(handle, x.data_ptr(), out.data_ptr(), batch, s) != 0:
            raise RuntimeError(dll.ppocr_model_error().decode())

    try:
        for i in range(max(warmup, 3)):
            body(i)
        stream.synchronize()
        ms = _event_steps(stream, steps, body, flush)
    finally:
        stream.synchronize()
        dll.ppocr_model_destroy(handle)
        dll.ppocr_model_release_resources(ctypes.byref(resources))
    ms.sort()
    return {"batch": batch, "ms": round(ms[len(ms) // 2], 4), "ms_min": round(ms[0], 4),
            "output_shape": list(out_shape)}


def abi_comparison(which: str, dev, steps: int = 10, warmup: int = 3) -> dict:
    """Recognizer (B = 512, 256 and 64 lines) and detector (8 and 1 pages of 960^2) forwards
    through ppocr_model_enqueue: which = "b200" times this repository's fused
    libraries, which = "reference" the reference's own compiled runtime
    (model_library.cu + runtime.cuh on cuDNN / cuBLAS / cuBLASLt / CUTLASS,
    built unmodified around the exporter-vocabulary twin of the same graph
    under oracle/_ref/models/). Same seeded weights function, same input."""
    from ppocr_b200 import models

    res = {"call": "ppocr_model_enqueue (Model ABI v2), f32 NCHW input resident in HBM, full batch, "
                   "L2 flushed between steps, median of %d steps" % steps}
    for key, name in (("recognizer_b512", "rec_b512"), ("recognizer_b256", "rec_b256"),
                      ("recognizer_b64", "rec_b64"), ("detector_8x960", "det_b8"),
                      ("detector_1x960", "det_b1")):
        if which == "b200":
            from ppocr_b200 import capi

            capi.load()  # the model shells link libppocr_b200.so
            so, wname = models.library_path(name), name
        else:
            wname = name + "_xv"
            so = REPO / "oracle" / "_ref" / "models" / wname / "model.so"
        if not Path(so).exists():
            res[key] = {"unavailable": f"{Path(so).relative_to(REPO)} is not built"}
            continue
        try:
            r = abi_forward(so, models.ensure_weights(wname), dev, steps, warmup)
        except RuntimeError as exc:  # e.g. the reference's own workspace-capacity check
            res[key] = {"unavailable": f"{exc}"[:200]}
            continue
        if key.startswith("recognizer"):
            r["lines_per_s"] = round(r["batch"] / (r["ms"] / 1e3), 1)
        else:
            r["pages_per_s"] = round(r["batch"] / (r["ms"] / 1e3), 1)
        res[key] = r
    return res


def op_bytes(g, index: int) -> float:
    """Algorithmic HBM bytes of one graph layer: every distinct tensor it
    reads (activations and constants) plus the one it writes, FP16."""
    import math

    layer = g.layers[index]
    ids = set()
    for k, v in layer.items():
        if k in ("in", "w", "b", "scale", "bias", "add", "a") or (k == "res" and v >= 0):
            if isinstance(v, int) and v >= 0:
                ids.add(v)
            elif isinstance(v, list):
                ids.update(i for i in v if isinstance(i, int) and i >= 0)
    ids.add(layer["out"])
    total = 0
    for i in ids:
        t = g.tensors[i]
        shape = t.const.shape if t.const is not None else t.shape
        total += 2 * math.prod(shape)
    return float(total)


def _per_op(model, reps=3):
    prof = [model.lib.profile(model.handle) for _ in range(reps)]
    return [min(p[i] for p in prof) for i in range(len(prof[0]))]


def _dominant(model, name, bound_hint=None):
    """(index, name, ms, bytes, flops) of the slowest op of a compiled graph."""
    from ppocr_b200 import models

    per = _per_op(model)
    names = model.lib.op_names(model.handle)
    dom = max(range(len(per)), key=lambda i: per[i])
    g, _ = models.graph(name)
    return dom, names[dom], per[dom], op_bytes(g, dom), op_flops(g, dom), per, names


def _roofline_for(kind, ms, bytes_, flops, key, peak_tf, peak_hbm, peak_kind):
    if kind == "tensor" and not flops:
        kind = "hbm"  # not a contraction: bounded by its bytes
    traffic = None
    tf = REPO / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(key)
    if kind == "hbm":
        achieved = bytes_ / (ms / 1e3) / 1e9
        return {"bound": "hbm", "kernel": key, "achieved": round(achieved, 1), "peak": peak_hbm, "unit": "GB/s",
                "frac": round(achieved / peak_hbm, 4), "peak_source": f"hbm_gbs of {peak_kind} peaks",
                "traffic": traffic, "launch_ms": round(ms, 5), "bytes": bytes_}
    achieved = flops / (ms / 1e3) / 1e12
    return {"bound": "tensor", "kernel": key, "achieved": round(achieved, 1), "peak": peak_tf, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tf, 4), "peak_source": f"bf16_tflops of {peak_kind} peaks",
            "traffic": traffic, "launch_ms": round(ms, 5), "flops": flops}


def measure_pages(dev, runs, warm, flush, with_cpu=False, seed_offset=0):
    """BASELINE config 5 on this GPU: 8 FP16 NHWC 960^2 pages (detector +
    binarize) and 512 line crops (recognizer + head + collapse) per run,
    `runs` timed runs after `warm` warm-up runs; CUDA events on the
    pipeline's stream, L2 flushed outside the events, clocks sampled.
    Returns step/e2e times, p50/p90, the detector's dominant-op roofline and
    per-op figures, and (with_cpu) the CPU port's bounded-sample latency."""
    import ctypes

    import numpy as np
    import torch

    from ppocr_b200 import capi, models, pipeline, workloads

    lib = capi.load()
    peak_tf, peak_hbm, peak_kind = peaks()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    r = workloads.rng(SEED + seed_offset)
    pp = pipeline.PagePipeline(device=dev)
    pages_np, crops_np = workloads.c5_pages(r)
    pages_h = torch.from_numpy(pages_np).pin_memory()
    crops_h = torch.from_numpy(crops_np).pin_memory()
    pages, crops = pages_h.to(dev), crops_h.to(dev)
    stream = pp.stream
    for _ in range(warm):
        pp.enqueue(pages, crops)
    stream.synchronize()
    assert lib.ppocr_b200_device_error() == 0
    with ClockSampler(dev.index or 0) as clocks:
        step_ms = _event_steps(stream, runs, lambda i: pp.enqueue(pages, crops), flush)
    bm_h = torch.empty_like(pp.bitmap, device="cpu").pin_memory()
    ids_h = torch.empty_like(pp.rec.out_ids, device="cpu").pin_memory()
    len_h = torch.empty_like(pp.rec.out_len, device="cpu").pin_memory()
    sc_h = torch.empty_like(pp.rec.out_score, device="cpu").pin_memory()
    # End to end through PagePipeline.enqueue_host: pinned pages and crops
    # in, binary maps and decoded lines out, every run; the crops' copy in
    # overlaps the detector and the map's copy out the recognizer, and each
    # run's end event follows all of its copies.
    def e2e_body(i):
        pp.enqueue_host(pages_h, crops_h, bm_h, ids_h, len_h, sc_h)

    for i in range(2):
        e2e_body(i)
    stream.synchronize()
    e2e_ms = _event_steps(stream, runs, e2e_body, None)
    out = {"step_ms": step_ms, "e2e_ms": e2e_ms}
    out["h2d_bytes_per_run"] = (pages_h.numel() + crops_h.numel()) * 2
    out["d2h_bytes_per_run"] = bm_h.numel() + ids_h.numel() * 4 + len_h.numel() * 4 + sc_h.numel() * 4
    dom, dname, dms, dbytes, dflops, per, names = _dominant(pp.det, "det_b8")
    out["roofline"] = _roofline_for("tensor", dms, dbytes, dflops, f"c5:det:{dname}#{dom}", peak_tf, peak_hbm,
                                    peak_kind)
    gdet, _ = models.graph("det_b8")
    top = sorted(range(len(per)), key=lambda i: -per[i])[:10]
    out["detector_top_ops"] = []
    for i in top:
        f = op_flops(gdet, i)
        b = op_bytes(gdet, i)
        out["detector_top_ops"].append({
            "op": f"{names[i]}#{i}", "ms": round(per[i], 5),
            "tflops": round(f / (per[i] / 1e3) / 1e12, 1) if f and per[i] > 0 else None,
            "gbs": round(b / (per[i] / 1e3) / 1e9, 1) if per[i] > 0 else None})
    # binarize alone: 5 B/pixel (f32 read + u8 write)
    n = pp.prob.numel()
    s = ctypes.c_void_p(stream.cuda_stream)
    bin_ms = _event_steps(stream, 20, lambda i: capi.check(lib.ppocr_b200_binarize(
        P(pp.prob), P(pp.bitmap), n, pp.thresh, s)), flush)
    out["binarize"] = _roofline_for("hbm", statistics.mean(bin_ms), 5.0 * n, None, "c5:binarize",
                                    peak_tf, peak_hbm, peak_kind)
    out["detector_eager_ms"] = round(sum(_per_op(pp.det)), 4)
    out["p50_ms"] = round(float(np.percentile(step_ms, 50)), 4)
    out["p90_ms"] = round(float(np.percentile(step_ms, 90)), 4)
    out["e2e_p50_ms"] = round(float(np.percentile(e2e_ms, 50)), 4)
    out["runs"] = runs
    # detector ops after the staged transpose, binarize, recognizer ops
    # after its staged transpose, vocabulary projection (2), collapse (1)
    launched = lambda ns: sum(1 for n in ns[1:] if n != "fused")  # noqa: E731
    out["launches_per_run"] = launched(names) + 1 + launched(pp.rec.model.lib.op_names(pp.rec.model.handle)) + 3
    out["clocks_obj"] = clocks
    out["clocks"] = clocks.summary()
    out["cpu_baseline"] = _cpu_c5() if with_cpu else None
    pp.close()
    return out


def config_arm(args):
    import ctypes

    import numpy as np
    import torch

    from ppocr_b200 import capi, models, pipeline, workloads

    rank, world, local = dist_env()
    if rank != 0:
        return  # the secondary configurations run on one GPU
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = capi.load()
    metric, unit, hib = CONFIGS[args.config]
    peak_tf, peak_hbm, peak_kind = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    r = workloads.rng(SEED)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    warm = max(args.warmup, 3)
    extra = {}

    if args.config == "c1":
        lines, T, V = 32, workloads.SEQ, workloads.VOCAB
        rows = lines * T
        logits_h = torch.from_numpy(workloads.c1_logits(r, lines, T, V).reshape(rows, V)).pin_memory()
        logits = logits_h.to(dev)
        ids = torch.empty(rows, dtype=torch.int32, device=dev)
        prob = torch.empty(rows, dtype=torch.float32, device=dev)
        mx = torch.empty(rows, dtype=torch.float32, device=dev)
        oid = torch.empty(lines, T, dtype=torch.int32, device=dev)
        olen = torch.empty(lines, dtype=torch.int32, device=dev)
        osc = torch.empty(lines, dtype=torch.float32, device=dev)
        h_oid, h_olen, h_osc = (torch.empty_like(t, device="cpu").pin_memory() for t in (oid, olen, osc))
        stream = torch.cuda.Stream(dev)
        s = ctypes.c_void_p(stream.cuda_stream)
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]

        def head(i=None, src=logits):
            if i is not None:
                kev[i][0].record(stream)
            capi.check(lib.ppocr_b200_logits_argmax_prob(P(src), rows, V, P(ids), P(prob), P(mx), 1, s))
            if i is not None:
                kev[i][1].record(stream)
            capi.check(lib.ppocr_b200_ctc_collapse(P(ids), P(prob), lines, T, 0, P(oid), P(olen), P(osc), s))

        for _ in range(warm):
            head()
        stream.synchronize()
        with ClockSampler(local) as clocks:
            step_ms = _event_steps(stream, args.steps, head, flush)
        kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
        units = lines
        # e2e: pinned logits in, decoded ids/lengths/scores out, every step
        stage = torch.empty_like(logits)

        def e2e_body(i):
            with torch.cuda.stream(stream):
                stage.copy_(logits_h, non_blocking=True)
            head(src=stage)
            with torch.cuda.stream(stream):
                h_oid.copy_(oid, non_blocking=True)
                h_olen.copy_(olen, non_blocking=True)
                h_osc.copy_(osc, non_blocking=True)

        e2e_ms = _event_steps(stream, args.steps, e2e_body, None)
        h2d = logits_h.numel() * 2
        d2h = h_oid.numel() * 4 + h_olen.numel() * 4 + h_osc.numel() * 4
        roof = _roofline_for("hbm", kernel_ms, rows * V * 2.0 + rows * 12.0, None, "c1:logits_argmax",
                             peak_tf, peak_hbm, peak_kind)
        launches = 2
        cpu = _cpu_c1(logits_h.numpy(), lines, T, V)
        workload = "BASELINE config 1: CTC head on materialised FP16 logits [32,40,18385] (seeded N(0,1), +4 " \
                   "boost, 30% blank, repeats), device argmax/softmax-max + greedy collapse"
    elif args.config in ("c2", "c3"):
        name = "block_b16" if args.config == "c2" else "neck_b256"
        model = pipeline.CompiledModel(name, dev)
        if args.config == "c2":
            x_np = workloads.c2_input(r, 16)
            units = 16
        else:
            x_np = workloads.c3_tokens(r, 256).reshape(256, 1, workloads.SEQ, 120)
            units = 256
        x_h = torch.from_numpy(x_np).pin_memory()
        x = x_h.to(dev)
        out = model.output_tensor()
        out_h = torch.empty_like(out, device="cpu").pin_memory()
        stream = torch.cuda.Stream(dev)
        for _ in range(warm):
            model.enqueue_nhwc(x, out, stream)
        stream.synchronize()
        with ClockSampler(local) as clocks:
            step_ms = _event_steps(stream, args.steps, lambda i: model.enqueue_nhwc(x, out, stream), flush)
        # e2e through ModelStream: every step copies its input in and its
        # output back inside the timed region, the copies of the neighbouring
        # steps overlapping this step's forward (two copy streams).
        mstream = pipeline.ModelStream(model, stream)
        outs_h = [out_h, torch.empty_like(out_h).pin_memory()]
        mstream.enqueue([x_h] * 2, outs_h)
        mstream.join(stream)
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        mstream.enqueue([x_h] * args.steps, [outs_h[i % 2] for i in range(args.steps)])
        mstream.join(stream)
        e1.record(stream)
        stream.synchronize()
        e2e_ms = [e0.elapsed_time(e1) / args.steps] * args.steps
        extra["e2e_pipeline"] = "ModelStream: H2D of step k+1 and D2H of step k-1 overlap step k"
        h2d = x_h.numel() * 2
        d2h = out_h.numel() * 2
        dom, dname, dms, dbytes, dflops, per, names = _dominant(model, name)
        if dname == "dwpw_block":
            # The fused block reads the depthwise input and writes the
            # pointwise output (the graph's layer table describes the two
            # layers separately): the fused minimum, weights included.
            dbytes = (16 * 48 * 320 * 64 + 16 * 48 * 320 * 128 + 64 * 25 + 128 * 64 + 64 + 128) * 2.0
        roof = _roofline_for("hbm", dms, dbytes, dflops, f"{args.config}:{dname}#{dom}", peak_tf, peak_hbm,
                             peak_kind)
        g, _ = models.graph(name)
        extra["ops"] = [{"op": f"{names[i]}#{i}", "ms": round(per[i], 5),
                         "gbs": round(op_bytes(g, i) / (per[i] / 1e3) / 1e9, 1) if per[i] > 0 else None}
                        for i in range(len(per)) if per[i] > 0]
        if args.config == "c2":
            fused_min = (16 * 48 * 320 * 64 + 16 * 48 * 320 * 128) * 2.0
            extra["block_vs_fused_minimum"] = {
                "bytes": fused_min, "gbs": round(fused_min / (statistics.mean(step_ms) / 1e3) / 1e9, 1),
                "frac": round(fused_min / (statistics.mean(step_ms) / 1e3) / 1e9 / peak_hbm, 4)}
        # c2: the leading NCHW->NHWC op is replaced by a copy (no kernel);
        # c3: every op runs, after one input-staging kernel.
        launches = len(names) - 1 if args.config == "c2" else len(names) + 1
        cpu = _cpu_graph(name, units)
        model.close()
        workload = ("BASELINE config 2: depthwise 5x5 s1 p2 (+folded BN, hardswish) -> pointwise 64->128 "
                    "(+folded BN, hardswish) on FP16 NHWC [16,48,320,64] through the Model ABI v2 shell"
                    if args.config == "c2" else
                    "BASELINE config 3: SVTR neck (2 x [LN -> 8-head MHSA dh 15 -> residual -> LN -> MLP "
                    "120-240-120 swish -> residual]) on FP16 [256,40,120] through the Model ABI v2 shell")
    elif args.config == "pre":
        pages = 8
        src_np = workloads.source_pages(r, pages)
        sh, sw = src_np.shape[1:3]
        boxes = [workloads.line_boxes(r, workloads.LINES_PER_PAGE, sh, sw) for _ in range(pages)]
        src_h = torch.from_numpy(src_np).pin_memory()
        src = src_h.to(dev)
        m_invs = torch.from_numpy(np.stack([b[0] for b in boxes])).to(dev)  # [pages, 64, 9]
        widths = torch.from_numpy(np.stack([b[1] for b in boxes])).to(dev)  # [pages, 64]
        # aspect-preserving content rectangle on a 960 x 960 canvas
        S = workloads.PAGE
        ch, cw = (S * sh // sw, S) if sw >= sh else (S, S * sw // sh)
        det_in = torch.empty(pages, S, S, 3, dtype=torch.float16, device=dev)
        crops = torch.empty(pages * workloads.LINES_PER_PAGE, H, W, 3, dtype=torch.float16, device=dev)
        stream = torch.cuda.Stream(dev)
        s = ctypes.c_void_p(stream.cuda_stream)
        page_bytes = sh * sw * 3
        nb = workloads.LINES_PER_PAGE
        crop_elems = nb * H * W * 3
        dev_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
        warp_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]

        def prep(i=None, source=src):
            if i is not None:
                dev_ev[i][0].record(stream)
            capi.check(lib.ppocr_b200_detector_preprocess(P(source), sw * 3, sh, sw, page_bytes, pages, P(det_in),
                                                          S, S, ch, cw, 0, capi.PREP_F16_NHWC, s))
            if i is not None:
                dev_ev[i][1].record(stream)
                warp_ev[i][0].record(stream)
            for p in range(pages):
                capi.check(lib.ppocr_b200_roi_warp(
                    ctypes.c_void_p(source.data_ptr() + p * page_bytes), sw * 3, sh, sw,
                    ctypes.c_void_p(m_invs.data_ptr() + p * nb * 36), ctypes.c_void_p(widths.data_ptr() + p * nb * 4),
                    ctypes.c_void_p(crops.data_ptr() + p * crop_elems * 2), nb, H, W, 0, capi.PREP_F16_NHWC, s))
            if i is not None:
                warp_ev[i][1].record(stream)

        for _ in range(warm):
            prep()
        stream.synchronize()
        with ClockSampler(local) as clocks:
            step_ms = _event_steps(stream, args.steps, prep, flush)
        det_ms = statistics.mean(a.elapsed_time(b) for a, b in dev_ev)
        warp_ms = statistics.mean(a.elapsed_time(b) for a, b in warp_ev)
        stage = torch.empty_like(src)
        det_h = torch.empty_like(det_in, device="cpu").pin_memory()
        crops_h = torch.empty_like(crops, device="cpu").pin_memory()

        def e2e_body(i):
            with torch.cuda.stream(stream):
                stage.copy_(src_h, non_blocking=True)
            prep(source=stage)
            with torch.cuda.stream(stream):
                det_h.copy_(det_in, non_blocking=True)
                crops_h.copy_(crops, non_blocking=True)

        e2e_ms = _event_steps(stream, args.steps, e2e_body, None)
        h2d = src_h.numel()
        d2h = (det_h.numel() + crops_h.numel()) * 2
        det_bytes = pages * page_bytes + det_in.numel() * 2.0
        roof = _roofline_for("hbm", det_ms, det_bytes, None, "pre:detector_preprocess", peak_tf, peak_hbm,
                             peak_kind)
        warp_bytes = crops.numel() * 2.0 + pages * page_bytes
        extra["roi_warp"] = _roofline_for("hbm", warp_ms, warp_bytes, None, "pre:roi_warp x8 (one per page)",
                                          peak_tf, peak_hbm, peak_kind)
        extra["roi_warp"]["algorithmic"] = "FP16 NHWC crops written + each source page read once"
        # Line tensors (server-side lines path): 512 decoded line images of
        # random sizes -> [512, 48, 320, 3] FP16 NHWC in one call.
        lr = workloads.rng(SEED + 5)
        ims, offs, wsz, hsz = [], [], [], []
        pos = 0
        for _ in range(LINES):
            h_ = int(lr.integers(24, 97))
            w_ = int(lr.integers(8, W * h_ // 48 + 1))
            ims.append(lr.integers(0, 256, h_ * w_ * 3, dtype=np.uint8))
            offs.append(pos)
            wsz.append(w_)
            hsz.append(h_)
            pos += h_ * w_ * 3
        line_px = torch.from_numpy(np.concatenate(ims)).to(dev)
        line_out = torch.empty(LINES, H, W, 3, dtype=torch.float16, device=dev)
        Ln, In = ctypes.c_longlong * LINES, ctypes.c_int * LINES
        offs_c, w_c, h_c, st_c = Ln(*offs), In(*wsz), In(*hsz), In(*[3 * x for x in wsz])
        lines_call = lambda i=None: capi.check(lib.ppocr_b200_line_tensors(  # noqa: E731
            P(line_px), offs_c, w_c, h_c, st_c, LINES, W, P(line_out), capi.PREP_F16_NHWC, s))
        for _ in range(warm):
            lines_call()
        line_ms = statistics.mean(_event_steps(stream, 20, lambda i: lines_call(), flush))
        extra["line_tensors"] = _roofline_for("hbm", line_ms, float(pos + line_out.numel() * 2), None,
                                              "pre:line_tensors (512 lines)", peak_tf, peak_hbm, peak_kind)
        extra["line_tensors"]["algorithmic"] = "decoded u8 line images read once + FP16 NHWC tensor written"
        roof["algorithmic"] = "u8 pages read once + FP16 NHWC canvases written"
        launches = 1 + pages
        units = pages
        cpu = _cpu_pre(src_np[0], boxes[0], ch, cw)
        workload = ("page preprocessing (reference full_page_worker.cpp:345-349, 467-471): 8 decoded u8 RGB "
                    "1080x1920 pages -> detector resize + normalize into a 960x960 canvas (content 540x960) as "
                    "FP16 NHWC, and 64 synthetic rotated line boxes per page -> perspective ROI warp to 48x320 "
                    "FP16 NHWC crops (v/127.5 - 1)")
    elif args.config == "post":
        pages, S, max_comp = 8, workloads.PAGE, 3000
        probs_h = torch.from_numpy(workloads.db_like_maps(r, pages, S)).pin_memory()
        probs = probs_h.to(dev)
        n = probs.numel()
        bitmap = torch.empty(pages, S, S, dtype=torch.uint8, device=dev)
        labels = torch.empty(pages, S, S, dtype=torch.int32, device=dev)
        counts = torch.empty(pages, dtype=torch.int32, device=dev)
        stats = torch.empty(pages, max_comp, 5, dtype=torch.int32, device=dev)
        probq = torch.empty(pages, max_comp, dtype=torch.int64, device=dev)
        ws = torch.empty(lib.ppocr_b200_db_components_workspace(pages, S, S, max_comp), dtype=torch.uint8,
                         device=dev)
        stream = torch.cuda.Stream(dev)
        s = ctypes.c_void_p(stream.cuda_stream)
        cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]

        def post(i=None, src=probs):
            capi.check(lib.ppocr_b200_binarize(P(src), P(bitmap), n, 0.3, s))
            if i is not None:
                cev[i][0].record(stream)
            capi.check(lib.ppocr_b200_db_components(P(bitmap), P(src), pages, S, S, max_comp, P(labels), P(counts),
                                                    P(stats), P(probq), P(ws), s))
            if i is not None:
                cev[i][1].record(stream)

        for _ in range(warm):
            post()
        stream.synchronize()
        assert lib.ppocr_b200_device_error() == 0
        with ClockSampler(local) as clocks:
            step_ms = _event_steps(stream, args.steps, post, flush)
        comp_ms = statistics.mean(a.elapsed_time(b) for a, b in cev)
        stage = torch.empty_like(probs)
        counts_h = torch.empty_like(counts, device="cpu").pin_memory()
        stats_h = torch.empty_like(stats, device="cpu").pin_memory()
        probq_h = torch.empty_like(probq, device="cpu").pin_memory()

        def e2e_body(i):
            with torch.cuda.stream(stream):
                stage.copy_(probs_h, non_blocking=True)
            post(src=stage)
            with torch.cuda.stream(stream):
                counts_h.copy_(counts, non_blocking=True)
                stats_h.copy_(stats, non_blocking=True)
                probq_h.copy_(probq, non_blocking=True)

        e2e_ms = _event_steps(stream, args.steps, e2e_body, None)
        h2d = probs_h.numel() * 4
        d2h = counts_h.numel() * 4 + stats_h.numel() * 4 + probq_h.numel() * 8
        comp_bytes = n * (1.0 + 4.0 + 4.0)  # bitmap + probabilities read, labels written
        roof = _roofline_for("hbm", comp_ms, comp_bytes, None, "post:db_components (7 launches)", peak_tf,
                             peak_hbm, peak_kind)
        roof["algorithmic"] = "u8 bitmap + f32 probabilities read once, int32 labels written once"
        extra["components_per_page"] = [int(c) for c in counts.cpu().tolist()]
        launches = 1 + 8
        units = pages
        cpu = _cpu_post(probs_h.numpy()[0])
        workload = ("DB post-processing front end (reference db_postprocess.cpp:183-252: cv::compare, then "
                    "findContours on the host): 8 synthetic DB-like 960x960 FP32 probability maps (64 rotated "
                    "text-line blobs per page over speckle) -> binarize 0.3 -> 8-connected components labelled "
                    "in OpenCV's order with (left, top, width, height, area) and fixed-point probability sums")
    else:  # c5
        pg = measure_pages(dev, args.steps, warm, flush, with_cpu=True)
        step_ms, e2e_ms = pg.pop("step_ms"), pg.pop("e2e_ms")
        roof, cpu, launches = pg.pop("roofline"), pg.pop("cpu_baseline"), pg.pop("launches_per_run")
        h2d, d2h = pg.pop("h2d_bytes_per_run"), pg.pop("d2h_bytes_per_run")
        clocks = pg.pop("clocks_obj")
        extra.update(pg)
        units = None
        workload = ("BASELINE config 5: 8 FP16 NHWC pages 960x960 -> DB detector (backbone strides 2..32, FPN "
                    "256, head 3x3 -> deconv x2 -> sigmoid) -> binarize 0.3, plus 64 synthetic 48x320 crops per "
                    "page (512) -> recognizer + CTC head + collapse; one batch per run, p50 over runs")

    if args.config == "c5":
        value = float(np.percentile(step_ms, 50))
        e2e_value = float(np.percentile(e2e_ms, 50))
        ms_per_step = value
    else:
        value = units * len(step_ms) / (sum(step_ms) / 1e3)
        e2e_value = units * len(e2e_ms) / (sum(e2e_ms) / 1e3)
        ms_per_step = sum(step_ms) / len(step_ms)
    line = {
        "metric": metric, "value": round(value, 4 if args.config == "c5" else 1), "unit": unit, "n_gpus": 1,
        "steps": len(step_ms), "warmup": warm, "ms_per_step": round(ms_per_step, 4), "higher_is_better": hib,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded, BASELINE distributions; seeded random-init weights)",
        "config": {"workload": workload, "l2": "flushed between timed steps (256 MB write outside the events)"},
        "e2e": {"value": round(e2e_value, 4 if args.config == "c5" else 1), "unit": unit,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": roof, "cpu_baseline": cpu, "gpu_launches": launches * len(step_ms),
        "clocks": clocks.summary(),
    }
    line.update(extra)
    print(json.dumps(line), flush=True)


def _cpu_c1(logits_f16: np.ndarray, lines: int, T: int, V: int):
    """Oracle C argmax/softmax-max (OpenMP, all cores) + the reference's own
    ctc_decode.cpp (oracle/_ref, when built) on all 32 lines."""
    import ctypes

    import numpy as np

    rows = lines * T
    lib = ctypes.CDLL(str(REPO / "oracle" / "_build" / "liboracle.so"))
    Pv = ctypes.c_void_p
    lib.oracle_argmax_prob.argtypes = [Pv, ctypes.c_long, ctypes.c_int, Pv, Pv, Pv, ctypes.c_int]
    lib.oracle_ctc_collapse.argtypes = [Pv, Pv, ctypes.c_long, ctypes.c_int, ctypes.c_int, Pv, Pv, Pv]
    ref_path = REPO / "oracle" / "_ref" / "libref_ctc.so"
    ref = ctypes.CDLL(str(ref_path)) if ref_path.exists() else None
    if ref is not None:
        ref.ref_ctc_decode_batch.argtypes = [Pv, Pv, ctypes.c_int, ctypes.c_int, ctypes.c_int, Pv, Pv, Pv]
    threads = os.cpu_count() or 1
    lg = np.ascontiguousarray(logits_f16.view(np.uint16))
    ids = np.empty(rows, np.int32)
    prob = np.empty(rows, np.float32)
    mx = np.empty(rows, np.float32)
    o_ids = np.empty((lines, T), np.int32)
    o_len = np.empty(lines, np.int32)
    o_sc = np.empty(lines, np.float32)
    times = []
    t_end = time.perf_counter() + 10.0
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        lib.oracle_argmax_prob(lg.ctypes.data, rows, V, ids.ctypes.data, prob.ctypes.data, mx.ctypes.data, threads)
        if ref is not None:
            ref.ref_ctc_decode_batch(ids.ctypes.data, prob.ctypes.data, lines, T, 0, o_ids.ctypes.data,
                                     o_len.ctypes.data, o_sc.ctypes.data)
        else:
            lib.oracle_ctc_collapse(ids.ctypes.data, prob.ctypes.data, lines, T, 0, o_ids.ctypes.data,
                                    o_len.ctypes.data, o_sc.ctypes.data)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": round(lines / med, 1), "unit": "lines/s", "cores": threads,
            "kind": "reference" if ref is not None else "port",
            "sample": f"all {lines} lines per call, median of {len(times)} calls: argmax/softmax-max by the "
                      f"oracle's C restatement (OpenMP), collapse by "
                      + ("the reference's own ctc_decode.cpp compiled as-is" if ref is not None else
                         "the oracle's C restatement")}


def _cpu_graph(name: str, units: int):
    """Oracle torch-CPU restatement of a compiled graph on a bounded sample."""
    import numpy as np
    import torch

    from ppocr_b200 import modelgen, models
    from oracle import models as om

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    family = models.SHAPES[name][0]
    spec = models.spec(family)
    sample = 2 if family == "block" else 64
    g, out = (modelgen.build_block(spec, sample, models.SEED) if family == "block"
              else modelgen.build_neck(spec, sample, models.SEED))
    x = np.random.default_rng(SEED).standard_normal(g.tensors[0].shape).astype(np.float32)
    om.run_graph(g, x, out)
    times = []
    t_end = time.perf_counter() + 10.0
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        om.run_graph(g, x, out)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    unit = "images/s" if family == "block" else "lines/s"
    return {"value": round(sample / med, 2), "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{sample} of the {units} {unit.split('/')[0]} per call, median of {len(times)} calls "
                      f"(oracle torch-CPU fp32 restatement of the same graph and weights; the reference has no "
                      f"CPU layer path)"}


def _cpu_pre(page, boxes, ch, cw):
    """The oracle's numpy restatement of one page's preprocessing (detector
    canvas + its 64 crops) on the host, scaled to the 8 pages of a step."""
    import numpy as np

    from oracle import preprocess as OP

    m, widths = boxes
    t0 = time.perf_counter()
    OP.detector_preprocess(page, 960, 960, ch, cw, False)
    OP.roi_warp(page, m, widths, H, W, False)
    dt = time.perf_counter() - t0
    return {"value": round(1.0 / dt, 3), "unit": "pages/s", "cores": 1, "kind": "port",
            "sample": f"1 page + its 64 crops through oracle/preprocess.py (numpy float32, {dt * 1e3:.0f} ms); "
                      "the reference's preprocessing exists only as CUDA kernels"}


def _cpu_post(prob):
    """One page through the oracle (numpy binarize + scipy labelling +
    statistics, the OpenCV-equivalent CPU path) on the host, scaled to 8."""
    from oracle import components as OC
    from oracle import layers as L

    t0 = time.perf_counter()
    bm = L.binarize(prob, 0.3)
    OC.components(bm, prob)
    dt = time.perf_counter() - t0
    return {"value": round(1.0 / dt, 3), "unit": "pages/s", "cores": 1, "kind": "port",
            "sample": f"1 page of 960^2 through oracle/components.py (numpy + scipy.ndimage, {dt * 1e3:.0f} ms)"}


def _cpu_c5():
    """Page latency on the host cores, from a bounded sample: one 960^2 page
    through the oracle's detector + binarize and 8 line crops through its
    recognizer, scaled to the 8-page, 512-line batch of one run."""
    import numpy as np
    import torch

    from ppocr_b200 import modelgen, models
    from oracle import layers as L
    from oracle import models as om

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rg = np.random.default_rng(SEED)
    gd, od = modelgen.build_detector(models.spec("detector"), 1, 960, models.SEED)
    gr, orr = modelgen.build_recognizer(models.spec("recognizer"), 8, models.SEED)
    page = rg.uniform(-1, 1, (1, 3, 960, 960)).astype(np.float32)
    lines8 = rg.uniform(-1, 1, (8, 3, H, W)).astype(np.float32)
    t0 = time.perf_counter()
    prob, _ = om.run_graph(gd, page, od)
    L.binarize(prob.numpy().ravel(), 0.3)
    t_page = time.perf_counter() - t0
    t0 = time.perf_counter()
    om.run_graph(gr, lines8, orr)
    t_line = (time.perf_counter() - t0) / 8
    batch_ms = 8 * (t_page + 64 * t_line) * 1e3
    return {"value": round(batch_ms, 1), "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"1 page (detector + binarize, {t_page * 1e3:.0f} ms) and 8 lines "
                      f"({t_line * 1e3:.1f} ms/line) through the oracle's torch-CPU restatement, scaled to one "
                      f"run's 8 pages + 512 lines (the reference has no CPU layer path)"}


def json_stdout():
    """Under torchrun, native libraries write banners to the process's
    stdout (NCCL prints its version at the first collective). Send file
    descriptor 1 to stderr and keep the original stdout for the JSON line
    alone, so that stdout holds exactly one line."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        sys.stdout.flush()
        keep = os.dup(1)
        os.dup2(2, 1)
        sys.stdout = os.fdopen(keep, "w", buffering=1)


def main():
    json_stdout()
    args = parse()
    if args.steps is None:
        args.steps = 20 if args.config == "c4" or args.impl == "reference" else 200
    if args.impl == "reference":
        reference_arm(args)
    elif args.config != "c4":
        config_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()
