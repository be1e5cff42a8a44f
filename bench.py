#!/usr/bin/env python
"""Benchmark: deform_conv2d forward+backward on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one forward + backward pass of one deformable-convolution layer over
one batch (plus the grad_weight/grad_bias all-reduce over NCCL when N > 1).
The default workload is the large grouped DCNv2 training step
(c5_train_bf16: global batch 64, 512->512 channels, 38x38, 3x3, pad 2,
dilation 2, groups 2, offset groups 4, bf16), strong-scaled: each of N ranks
takes 64/N samples.  Rank 0 prints one JSON line.

--impl reference times the CPU path that the package's parity tests treat as
ground truth (torchvision.ops.deform_conv2d on the host cores, fp32) on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mps-deform-conv_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

from mps_deform_conv.sharding import OverlappedParamAllReduce, allreduce_param_grads, shard_range  # noqa: E402
from mps_deform_conv.workloads import PROBLEMS, make_inputs  # noqa: E402

METRIC = "deform_conv2d fwd+bwd TFLOP/s & % roofline per B200; samples/s at 1/2/4/8 GPUs"
L2_BYTES = 126 * 1024 * 1024


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    Polls NVML (the counters behind nvidia-smi's clocks.sm / clocks.max.sm /
    clocks_event_reasons.*) every ~2 ms from a thread, so even a timed region
    of tens of milliseconds gets samples; falls back to `nvidia-smi -lms 20`."""
    NAMES = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
             "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []   # (sm_mhz, max_mhz, reasons bitmask)
        self.stop = threading.Event()
        self.proc = None
        self.t = None

    def _poll_nvml(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self.stop.is_set():
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                try:
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    rs = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((float(sm), float(mx), int(rs)))
                time.sleep(0.002)
        finally:
            pynvml.nvmlShutdown()

    def _poll_smi(self):
        q = "clocks.sm,clocks.max.sm,clocks_event_reasons.active"
        self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={q}",
                                      "--format=csv,noheader,nounits", "-lms", "20"],
                                     stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            try:
                self.samples.append((float(parts[0]), float(parts[1]), int(parts[2], 16)))
            except Exception:
                pass

    def __enter__(self):
        try:
            import pynvml  # noqa: F401
            target = self._poll_nvml
        except Exception:
            target = self._poll_smi
        self.t = threading.Thread(target=target, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
        if self.t is not None:
            self.t.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set()
        for _, _, rs in self.samples:
            for nm, bit in self.NAMES.items():
                if rs & bit:
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(x[0] for x in self.samples),
                "sm_max_mhz": max(x[1] for x in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU path
def cpu_reference_step(p, inp, threads):
    """torchvision CPU fwd(+bwd) in fp32 on one sample batch; returns seconds."""
    from torchvision.ops import deform_conv2d as tv_dc
    torch.set_num_threads(threads)
    x = inp["input"].float().requires_grad_(p.training)
    off = inp["offset"].float().requires_grad_(p.training)
    w = inp["weight"].float().requires_grad_(p.training)
    b = inp["bias"].float().requires_grad_(p.training) if inp["bias"] is not None else None
    m = inp["mask"].float().requires_grad_(p.training) if inp["mask"] is not None else None
    t0 = time.perf_counter()
    out = tv_dc(x, off, w, b, stride=(p.stride,) * 2, padding=(p.padding,) * 2,
                dilation=(p.dilation,) * 2, mask=m)
    if p.training:
        out.backward(inp["grad_output"].float())
    return time.perf_counter() - t0


def cpu_sample_batch(p):
    """Samples per CPU step: about 1-3 s of host work per step."""
    est = {"c1_dcnv1_fp32": 1, "c2_dcnv2_fp32": 2, "c3a_backbone_bf16": 2,
           "c3b_backbone_s2_bf16": 2, "c4_video_fp16": 1, "c5_train_bf16": 1}
    return est.get(p.name, 1)


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    p = PROBLEMS[args.workload]
    threads = os.cpu_count() or 1
    nb = cpu_sample_batch(p)
    inp = make_inputs(p, "cpu", batch=nb, dtype=torch.float32)
    for _ in range(args.warmup):
        cpu_reference_step(p, inp, threads)
    ts = [cpu_reference_step(p, inp, threads) for _ in range(args.steps)]
    total = sum(ts)
    samples_s = nb * args.steps / total
    tflops = p.flops(nb) * args.steps / total / 1e12
    cpu_model = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu_model = next((l.split(":", 1)[1].strip() for l in f if l.startswith("model name")), "")
    except Exception:
        pass
    sample = (f"{nb} sample(s) of {p.name} per step, torchvision.ops.deform_conv2d CPU fp32 "
              f"fwd{'+bwd' if p.training else ''}, {threads} threads, {cpu_model}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tflops, 6), "unit": "TFLOP/s",
        "samples_per_s": round(samples_s, 4), "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, workload distributions)",
        "config": {"workload": p.name, "description": p.description, "global_batch": p.batch,
                   "sample_batch": nb},
        "cpu_baseline": {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(tflops, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU path
def run_ours(args):
    import mps_deform_conv as mdc
    from mps_deform_conv import _abi

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    p = PROBLEMS[args.workload]
    if args.batch:  # a reduced case of the same layer (ncu captures); the JSON line names its batch
        p = dataclasses.replace(p, batch=args.batch)
    first, nb = shard_range(p.batch, world, rank)
    peaks = load_peaks()
    inp = make_inputs(p, dev, batch=nb, batch_offset=first)
    stride, pad, dil = (p.stride,) * 2, (p.padding,) * 2, (p.dilation,) * 2
    x, off, w, b, m, go = (inp[k] for k in ("input", "offset", "weight", "bias", "mask", "grad_output"))
    leaves = [t for t in (x, off, w, b, m) if t is not None]
    if p.training:
        for t in leaves:
            t.requires_grad_(True)
    param_grads_idx = [2] + ([3] if b is not None else [])

    # grad_weight and grad_bias sum over the global batch: one flat-bucket
    # all-reduce per step after the backward, or with --overlap started from
    # the backward's parameter-gradient hook on a side stream (it then runs
    # beside the backward's final layout passes; measured equal at 2 GPUs and
    # about 1% slower at 8 on this step, whose all-reduce is 2.4 MB)
    overlap = world > 1 and p.training and args.overlap
    ar = OverlappedParamAllReduce() if overlap else None
    mdc.set_param_grad_hook(ar)

    def reduce_grads(grads):
        if ar is not None:
            ar.wait()
        elif world > 1:
            allreduce_param_grads([grads[i] for i in range(len(grads)) if leaves[i] is w or leaves[i] is b])

    fwd_ev = []

    def step(record=None):
        out = mdc.deform_conv2d(x, off, w, b, stride, pad, dil, m)
        if record is not None:
            record.record()
        if p.training:
            grads = torch.autograd.grad(out, leaves, go)
            reduce_grads(grads)
            return grads
        return out

    in_bytes = sum(t.numel() * t.element_size() for t in (x, off, m, go) if t is not None)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev) if in_bytes < 2 * L2_BYTES else None

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()

    # ---- profiled pass: K eager steps with per-kernel CUDA events recorded by
    # the library on the launching stream (kernel shares, roofline, launches)
    launches0 = _abi.launch_count()
    _abi.profile_enable(True)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
            torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
        evs[i][0].record()
        step(record=evs[i][1])
        evs[i][2].record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    _abi.profile_enable(False)
    launches_per_step = (_abi.launch_count() - launches0) / args.steps
    prof = _abi.profile_summary()
    eager_ms = max_over_ranks(sum(a.elapsed_time(c) for a, _, c in evs), world)
    fwd_ms = [a.elapsed_time(f) for a, f, _ in evs]

    # ---- timed region: the whole step (forward, backward, NCCL all-reduce)
    # captured once in a CUDA graph and replayed K times; per-step events,
    # L2 flushed between steps when the inputs are smaller than L2
    graph = None
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            ok = 1
        except Exception as exc:  # keep every rank on the same path
            graph, ok = None, 0
            print(f"[bench] graph capture failed, timing eager steps: {exc}", file=sys.stderr)
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([ok], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            if int(t.item()) == 0:
                graph = None
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    gevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            if flush is not None:
                flush.zero_()
            gevs[i][0].record()
            if graph is not None:
                graph.replay()
            else:
                step()
            gevs[i][1].record()
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in gevs), world)
    launches = int(round(launches_per_step * args.steps))
    clocks = clk.summary()
    timed_with_graph = graph is not None
    if graph is not None:
        del graph
        torch.cuda.synchronize()

    flops_step_job = p.flops(p.batch)          # all ranks together
    tflops = flops_step_job * args.steps / (total_ms / 1e3) / 1e12
    samples_s = p.batch * args.steps / (total_ms / 1e3)

    # ---- dominant kernel roofline (per-kernel CUDA events recorded by the library)
    kern = sorted(prof, key=lambda r: -r[2])
    roof = None
    if kern:
        name, nl, kms = kern[0]
        avg_s = kms / nl / 1e3
        rf = kernel_roofline(p, nb, name)
        if rf["bound"] == "tensor":
            achieved = rf["per_launch"] / avg_s / 1e12
            peak = peaks["bf16_tflops_sustained"]
            unit = "TFLOP/s"
        else:
            achieved = rf["per_launch"] / avg_s / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        roof = {"kernel": name, "bound": rf["bound"], "achieved": round(achieved, 2),
                "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
                "traffic": args.traffic_per_launch or measured_traffic(p.name, name, nb),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch (profiles/dram_traffic.txt)",
                "avg_launch_ms": round(kms / nl, 4),
                "launches": nl, "peak_source": peaks["source"] + (" (sustained bf16)" if unit == "TFLOP/s" else ""),
                "algorithmic_per_launch": rf["per_launch"], "note": rf["note"]}
        if name == "dcn_dgrad_tc":
            # the same launch against the bound it actually meets: the fp32
            # grad_input accumulation (4 corners x C x T per output pixel,
            # red.global.add on 128-byte lines) runs on the L2's reduction units
            red = 4.0 * p.kernel * p.kernel * p.in_channels * nb * p.out_hw[0] * p.out_hw[1] * 4
            roof["l2_reduction"] = {
                "bytes_per_launch": red, "achieved_TBps": round(red / avg_s / 1e12, 3),
                "ceiling_TBps": 6.2,
                "ceiling_source": "single-kernel measurement on this GPU type: red.global.add.v4.f32, 8 lanes per "
                                  "128-byte line, random lines of an L2-resident 64 MB target, every SM busy"}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(p, inp, args, dev, world)

    # ---- CPU baseline on rank 0 at N=1
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(p)

    suite = None
    if world == 1 and not args.no_suite:
        suite = run_suite(dev, skip=p.name)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tflops, 3), "unit": "TFLOP/s",
            "samples_per_s": round(samples_s, 2), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[p.dtype],
            "data": "synthetic (seeded; workload distributions)",
            "config": {"workload": p.name, "description": p.description, "global_batch": p.batch,
                       "per_gpu_batch": nb, "parallelism": f"batch-sharded dp{world}" + (
                           (", grad_weight/grad_bias NCCL all-reduce on a side stream, overlapping the "
                            "backward's final layout passes" if overlap else
                            ", grad_weight/grad_bias NCCL all-reduce after the backward")
                           if world > 1 and p.training else ""),
                       "l2": "flushed between steps (256 MB write)" if flush is not None
                       else f"inputs {in_bytes / 2**20:.0f} MB per rank > L2",
                       "fwd_ms_per_step": round(sum(fwd_ms) / args.steps, 4)},
            "roofline": roof,
            "kernels": [{"name": n, "launches": l, "ms": round(t, 4)} for n, l, t in kern],
            "timing": ("CUDA-graph replay of the captured step" if timed_with_graph else "eager steps")
                      + f"; eager profiled pass {round(eager_ms / args.steps, 4)} ms/step",
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
            "other_workloads": suite,
            "tensor_cores": bool(mdc._get_lib().uses_tensor_cores(
                x, w, p.stride, p.stride, p.padding, p.padding, p.dilation, p.dilation,
                p.groups, p.offset_groups, p.use_mask)),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_suite(dev, skip, steps=5, warmup=3):
    """Short device-timed fwd(+bwd) runs of the other workloads (N=1): one
    entry per problem with ms/step (CUDA-graph replay of the step, as the
    main timed region; the eager time beside it), TFLOP/s, samples/s, which
    kernel family ran it and its top kernels (from the eager pass).  Inputs
    stay resident; the L2 is flushed between steps.  Forward-only problems on the tensor cores get a second
    entry, "<name>/frozen_cl": the same call as a channels_last network in
    inference makes it (input already channels_last, weights frozen, so the
    forward weight image is built once: set_weight_image_cache)."""
    import mps_deform_conv as mdc
    from mps_deform_conv import _abi
    res = {}
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def measure(p, inp, channels_last=False):
        st, pd, dl = (p.stride,) * 2, (p.padding,) * 2, (p.dilation,) * 2
        x = inp["input"].contiguous(memory_format=torch.channels_last) if channels_last else inp["input"]
        leaves = [t.requires_grad_(p.training) if t is not None else None
                  for t in (x, inp["offset"], inp["weight"], inp["bias"], inp["mask"])]
        lv = [t for t in leaves if t is not None]

        def step():
            out = mdc.deform_conv2d(leaves[0], leaves[1], leaves[2], leaves[3], st, pd, dl, leaves[4])
            if p.training:
                torch.autograd.grad(out, lv, inp["grad_output"])
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        _abi.profile_enable(True)
        ms = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            ms += a.elapsed_time(b)
        _abi.profile_enable(False)
        prof = sorted(_abi.profile_summary(), key=lambda r: -r[2])
        ms /= steps
        eager_ms = ms
        # the step's device time without host launch gaps: captured once in a
        # CUDA graph and replayed, as the main timed region does
        timing = "eager steps"
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            torch.cuda.synchronize()
            tot = 0.0
            for _ in range(steps):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                graph.replay()
                b.record()
                torch.cuda.synchronize()
                tot += a.elapsed_time(b)
            ms = tot / steps
            timing = "CUDA-graph replay"
            del graph
            torch.cuda.synchronize()
        except Exception as exc:  # keep the eager time
            print(f"[bench] {p.name}: graph capture failed, eager time kept: {exc}", file=sys.stderr)
        tc = bool(mdc._get_lib().uses_tensor_cores(inp["input"], inp["weight"], p.stride, p.stride, p.padding,
                                                   p.padding, p.dilation, p.dilation, p.groups,
                                                   p.offset_groups, p.use_mask))
        return tc, {"description": p.description, "pass": "fwd+bwd" if p.training else "fwd",
                    "ms_per_step": round(ms, 4), "timing": timing, "eager_ms_per_step": round(eager_ms, 4),
                    "tflops": round(p.flops() / (ms / 1e3) / 1e12, 3),
                    "samples_per_s": round(p.batch / (ms / 1e3), 1),
                    "min_hbm_bytes": p.min_hbm_bytes(),
                    "hbm_frac_of_measured": round(p.min_hbm_bytes() / (ms / 1e3) / 1e9 / load_peaks()["hbm_gbs"], 4),
                    "kernels": "tcgen05 fused" if tc else "tcgen05 tf32 GEMMs, CUDA-core gather and scatter",
                    "top": [{"name": n, "ms_per_step": round(t / steps, 4)} for n, l, t in prof[:3]]}

    for name, p in PROBLEMS.items():
        if name == skip:
            continue
        inp = make_inputs(p, dev)
        tc, res[name] = measure(p, inp)
        if tc and not p.training:
            mdc.set_weight_image_cache(True)
            try:
                _, r = measure(p, inp, channels_last=True)
            finally:
                mdc.set_weight_image_cache(False)
            r["description"] += "; channels_last input, frozen weights (cached weight image)"
            res[name + "/frozen_cl"] = r
        del inp
        torch.cuda.empty_cache()
    return res


def measured_traffic(workload: str, kernel: str, batch: int):
    """DRAM bytes per launch of `kernel` from the committed ncu summaries
    (profiles/dram_traffic.txt: workload, kernel, batch, bytes per launch);
    scaled by batch when measured on a different batch; None if absent."""
    path = os.path.join(REPO, "profiles", "dram_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 4 and not line.startswith("#") and parts[0] == workload and parts[1] == kernel:
                    return float(parts[3]) * batch / float(parts[2])
    except OSError:
        pass
    return None


def kernel_roofline(p, nb, name):
    """Algorithmic work per launch of a named kernel, for nb samples per launch."""
    ho, wo = p.out_hw
    f = p.flops_forward(nb)
    es = torch.tensor([], dtype=p.dtype).element_size()
    t = p.kernel * p.kernel
    if "fwd" in name:
        return {"bound": "tensor", "per_launch": f, "note": "2*Co*K_red*P forward FLOPs"}
    if "dgrad" in name or "wgrad" in name:
        return {"bound": "tensor", "per_launch": f, "note": "2*Co*K_red*P FLOPs (one backward GEMM)"}
    # gather / scatter kernels: HBM-bound, unique bytes
    x = nb * p.in_channels * p.height * p.width * es
    off = nb * 2 * p.offset_groups * t * ho * wo * es
    msk = nb * p.offset_groups * t * ho * wo * es if p.use_mask else 0
    return {"bound": "hbm", "per_launch": x + off + msk, "note": "input+offset+mask bytes"}


def run_e2e(p, inp, args, dev, world):
    """Same step through the public API with host buffers: every step copies
    its inputs (input, offset, mask, grad_output) from pinned host memory and
    reads its result back (grad_weight and grad_bias when training, the output
    otherwise).  The copies of step i+1 run on a copy stream while step i
    computes (two device buffer sets), as a training input pipeline would."""
    import mps_deform_conv as mdc
    host = {k: (v.detach().cpu().pin_memory() if v is not None else None) for k, v in inp.items()}
    keys = [k for k in ("input", "offset", "mask", "grad_output") if host[k] is not None]
    if not p.training:
        keys.remove("grad_output")
    stride, pad, dil = (p.stride,) * 2, (p.padding,) * 2, (p.dilation,) * 2
    dev_w = inp["weight"].detach().clone().requires_grad_(p.training)
    dev_b = inp["bias"].detach().clone().requires_grad_(p.training) if inp["bias"] is not None else None
    h2d = sum(host[k].numel() * host[k].element_size() for k in keys)
    bufs = [{k: torch.empty_like(inp[k]) for k in keys} for _ in range(2)]
    if p.training:
        res_host = [torch.empty(dev_w.shape, dtype=dev_w.dtype).pin_memory()] + \
            ([torch.empty(dev_b.shape, dtype=dev_b.dtype).pin_memory()] if dev_b is not None else [])
    else:
        res_host = [torch.empty((inp["input"].shape[0], p.out_channels) + p.out_hw, dtype=p.dtype).pin_memory()]
    d2h = sum(t.numel() * t.element_size() for t in res_host)
    main = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        b = bufs[i % 2]
        with torch.cuda.stream(cs):
            if i >= 2:
                cs.wait_event(freed[i % 2])
            for k in keys:
                b[k].copy_(host[k], non_blocking=True)
            copied[i % 2].record(cs)

    def compute(i):
        b = bufs[i % 2]
        main.wait_event(copied[i % 2])
        x = b["input"].detach().requires_grad_(p.training)
        off = b["offset"].detach().requires_grad_(p.training)
        m = b["mask"].detach().requires_grad_(p.training) if "mask" in b else None
        out = mdc.deform_conv2d(x, off, dev_w, dev_b, stride, pad, dil, m)
        if p.training:
            lv = [t for t in (x, off, dev_w, dev_b, m) if t is not None]
            grads = torch.autograd.grad(out, lv, b["grad_output"])
            res = [grads[2]] + ([grads[3]] if dev_b is not None else [])
            if isinstance(mdc._param_grad_hook, OverlappedParamAllReduce):
                mdc._param_grad_hook.wait()
            elif world > 1:
                allreduce_param_grads(res)
        else:
            res = [out]
        for h, r in zip(res_host, res):
            h.copy_(r, non_blocking=True)
        freed[i % 2].record(main)

    def run(n, start=None):
        if start is not None:
            cs.wait_event(start)
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            compute(i)

    run(max(args.warmup, 3))
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(main)
    run(args.steps, start=s)
    e.record(main)
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e), world)
    tflops = p.flops(p.batch) * args.steps / (ms / 1e3) / 1e12
    return {"value": round(tflops, 3), "unit": "TFLOP/s",
            "samples_per_s": round(p.batch * args.steps / (ms / 1e3), 2),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "pipeline": "inputs of step i+1 copied on a second stream during step i"}


def cpu_baseline(p):
    threads = os.cpu_count() or 1
    nb = cpu_sample_batch(p)
    inp = make_inputs(p, "cpu", batch=nb, dtype=torch.float32)
    cpu_reference_step(p, inp, threads)  # warm-up
    reps = 3
    total = sum(cpu_reference_step(p, inp, threads) for _ in range(reps))
    tflops = p.flops(nb) * reps / total / 1e12
    return {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "samples_per_s": round(nb * reps / total, 4),
            "sample": f"{reps} x {nb} sample(s) of {p.name}, torchvision.ops.deform_conv2d CPU fp32 "
                      f"fwd{'+bwd' if p.training else ''}, {threads} threads"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c5_train_bf16", choices=sorted(PROBLEMS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-suite", action="store_true", help="skip the short runs of the other workloads")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps instead of a CUDA graph")
    ap.add_argument("--overlap", action="store_true",
                    help="start the parameter-gradient all-reduce from the backward's hook on a side stream")
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch override: a reduced case of the workload for ncu captures")
    ap.add_argument("--traffic-per-launch", type=float, default=None,
                    help="ncu dram bytes per launch of the dominant kernel, if captured")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
