"""Benchmark: ResNet-50 bf16 inference, batch 256 per GPU, 224x224 (the headline workload).

One process per GPU (torchrun for N > 1). Each rank builds the fused NHWC bf16 inference
plan (BatchNorm folded into tcgen05 implicit-GEMM convs, captured in one CUDA graph) and
processes its own 256 images: inference needs no collective, so scaling is weak and the
only cross-rank traffic is the host-side barrier and the max-over-ranks of the timings.

Printed JSON line (rank 0):
  value   images/s of the whole job, device-resident inputs, graph replay, max over ranks
  e2e     images/s through InferencePlan.serve with host buffers: per step the pinned
          host->device copy of the step's NCHW input (a bf16 image; e2e.fp32_input is the same
          loop with the fp32 image), on the transfer stream overlapping the previous step's
          forward, the forward, and the device->host copy of the logits, all inside the timed
          region
  roofline  the dominant kernels (the tensor-core convs): algorithmic conv+FC FLOPs of one
          step divided by their time per step, measured by the kernels' own per-CTA
          %globaltimer stamps in a graph replay of the same forward
  configs   (N = 1) short runs of the other configs: the conv sweep, ResNet-18 training and
          the MobileNet-style stack
  cpu_baseline  the reference engine's own CPU ResNet-50 forward (oracle/_ref/libomref.so,
          AVX2 + OpenMP on every host core) on a bounded sample, rank 0 at N=1 only

--impl reference times that reference CPU implementation on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ResNet-50 bf16 images/s at 1/2/4/8 B200; conv implicit-GEMM % of TC peak"
BATCH = 256
# DRAM read+write bytes of the 54 conv_tc_kernel launches of one batch-64 forward, from one ncu
# capture (profiles/conv_tc_kernel_traffic_resnet50_b64.md); traffic grows with the batch.
CONV_TRAFFIC_B64 = 2.311e9


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["bf16_tflops_sustained"], d["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=300))
        return world, rank, local, dist
    return world, rank, local, None


def _barrier(dist):
    """Host-side barrier over gloo (a CPU-tensor all-reduce), independent of NCCL."""
    if dist is not None:
        import torch
        dist.all_reduce(torch.zeros(1))


def _max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _wait_gil_free(event) -> None:
    """Wait for the compute stream through the backend (a ctypes call, which releases the GIL,
    so the clock sampler thread keeps sampling during the wait), then for `event`."""
    from omnimatchdeeplearningtool_b200._lib import call
    call("omCudaSynchronize")
    event.synchronize()


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed region: through NVML
    in a background thread every 5 ms (so a timed region of a few tens of ms still gets
    samples), else through `nvidia-smi -lms 200`. Only reads GPU state; changes nothing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.file = None
        self.thread = None
        self.samples = []
        self.mask = 0
        self.max_mhz = None
        self._stop = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            prop = torch.cuda.get_device_properties(self.device)
            bus = "%08x:%02x:%02x.0" % (prop.pci_domain_id, prop.pci_bus_id, prop.pci_device_id)
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            self._start_smi()
            return
        self._stop = threading.Event()

        def loop():
            while True:
                try:
                    self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                    self.mask |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                except Exception:
                    pass
                if self._stop.wait(0.005):
                    break

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def _start_smi(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            reasons = sorted(n for n, bit in self.REASONS.items() if self.mask & bit)
            return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                    "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, 5 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def _host_threads() -> int:
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _reference_cpu(batch: int, iters_min: int, seconds: float):
    """The reference engine's CPU ResNet-50 forward on `batch` images (or the oracle port
    when the reference library was not built). Returns (images/s, kind, cores, sample)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    net = synth.resnet_spec(50)
    w = synth.make_weights(net)
    x = synth.normal_input(batch)
    cores = _host_threads()
    orc.set_threads(cores)
    h = orc.ref_model(1, 1000, w, net)
    out = np.empty((batch, 1000), np.float32)
    if h is not None:
        kind = "reference"
        run = lambda: orc.ref().omref_model_forward(h, x.ctypes.data, batch, 224, 224, out.ctypes.data)
    else:
        kind = "port"
        run = lambda: orc.forward(net, w, x)
    run()  # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < iters_min or time.perf_counter() - t0 < seconds:
        run()
        n += 1
    dt = time.perf_counter() - t0
    sample = (f"ResNet-50 fp32 forward, batch {batch} at 224x224, {n} iterations "
              f"({dt:.1f} s), OMP threads={cores}")
    return n * batch / dt, kind, cores, sample


def run_train(args, world, rank, local, dist):
    """Config 3: ResNet-18 fp32 training step (forward with batch-statistics BN, softmax CE,
    backward with the gradient buckets' NCCL all-reduces overlapping it, SGD momentum 0.9,
    lr 0.01 on the mean gradient), batch 128 per GPU, weak scaling. The all-reduces go through
    the backend's C ABI (distributed.NcclCommunicator); torch only times and barriers."""
    import torch
    from omnimatchdeeplearningtool_b200 import backend, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.distributed import (DataParallel, DistributedConfig,
                                                            NcclCommunicator)
    from omnimatchdeeplearningtool_b200.plan import Fp32Net

    backend.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(backend.stream_handle(), device=local)
    batch = args.batch if args.batch != BATCH else 128
    net = synth.resnet_spec(18, 1000)
    weights = synth.make_weights(net)
    # BatchNorm statistics from the conv epilogue (omCudaConv2dBatchNorm2dAct) and the stem in
    # its space-to-depth form (omCudaStemConv2dBatchNorm2dAct); the training parity test runs
    # this form at config 3
    fnet = Fp32Net(net, weights, batch, 224, 224, fused_bn_stats=True, stem_s2d=True)
    comm = NcclCommunicator(rank, world, timeout_ms=120000) if world > 1 else None
    dp = DataParallel(fnet, DistributedConfig(world, rank), comm)
    x = DeviceBuffer.from_numpy(synth.normal_input(batch, seed=rank))
    y = DeviceBuffer.from_numpy(synth.onehot_labels(batch, 1000, seed=100 + rank))
    loss = DeviceBuffer.zeros(4)

    def one_step():
        fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
        dp.step(0.01, 0.9)

    for _ in range(args.warmup):
        one_step()
    dp.check()
    call("omCudaSynchronize")
    # one rank: the whole step (forward, backward, SGD) is captured once and replayed as a CUDA
    # graph; with several ranks the steps stay eager (the bucket all-reduces start from the
    # backward's gradient hook)
    graph = world == 1
    if graph:
        c0 = backend.launch_count()
        fnet.capture_step(x.ptr, y.ptr, loss.ptr, 0.01, 0.9)
        launches_per_step = backend.launch_count() - c0
        for _ in range(2):
            fnet.replay_step()
        call("omCudaSynchronize")
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    _barrier(dist)
    l0 = backend.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
    for _ in range(args.steps):
        if graph:
            fnet.replay_step()
        else:
            one_step()
    with torch.cuda.stream(stream):
        e1.record()
    _wait_gil_free(e1)
    dp.check()
    torch.cuda.synchronize()
    launches = (launches_per_step * args.steps if graph
                else backend.launch_count() - l0)
    _barrier(dist)
    clk = clocks.stop()
    t = _max_over_ranks(dist, e0.elapsed_time(e1) / 1e3)
    lv = float(loss.to_numpy((1,))[0])
    if rank == 0:
        flops_per_img = 3 * synth.conv_flops(net)  # forward + input and weight gradients
        tf = args.steps * batch * flops_per_img / t / 1e12
        line = {
            "metric": "ResNet-18 fp32 training images/s (config 3)", "value": args.steps * batch * world / t,
            "unit": "images/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) inputs, uniform labels, He-normal weights)",
            "config": {"workload": "resnet18 fp32 training step, SGD momentum 0.9 lr 0.01",
                       "batch_per_gpu": batch, "global_batch": batch * world,
                       "parallelism": f"dp{world}, NCCL all-reduce of gradient buckets "
                                      "overlapping the backward (backend C ABI)",
                       "launch": "CUDA graph of the whole step" if graph else "eager"},
            "tflops_per_gpu": tf, "gpu_launches": launches,
            "loss_last_step": lv, "clocks": clk, "kernel_error": backend.kernel_error(),
        }
    else:
        line = None
    if comm is not None:
        comm.close()
    fnet.close()
    return line


def run_sweep(args, world, rank, local, dist):
    """Config 2: one conv2d + BatchNorm2d (eval) + ReLU layer per shape -- 3x3 s1 p1 and 1x1 s1,
    C = K in {64,128,256,512}, H = W in {56,28,14,7}, N = 32 -- in fp32, bf16 and fp16. Each
    timed run is preceded by a 256 MB write that flushes L2; CUDA events bracket the layer
    alone. Parity of the same layers is checked in tests/test_gpu_conv_sweep.py."""
    import torch
    from omnimatchdeeplearningtool_b200 import backend, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.layers import ConvBnReluLayer

    backend.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(backend.stream_handle(), device=local)
    flush = DeviceBuffer(256 << 20)
    peak_burst, _, _, peak_src = _peaks()
    n = 32
    rows = []
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = backend.launch_count()
    for ks in (3, 1):
        for c in (64, 128, 256, 512):
            for h in (56, 28, 14, 7):
                data = synth.conv_layer_data(c, h, ks, n, seed=900 + c + h + ks)
                for dt in ("fp32", "bf16", "fp16"):
                    layer = ConvBnReluLayer(*data, 1, ks // 2, dt)
                    for _ in range(args.warmup):
                        layer.run()
                    total = 0.0
                    with torch.cuda.stream(stream):
                        for _ in range(args.steps):
                            call("omCudaMemset", flush.ptr, 1, flush.nbytes)
                            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            e0.record()
                            layer.run()
                            e1.record()
                            e1.synchronize()
                            total += e0.elapsed_time(e1) / 1e3
                    t = total / args.steps
                    tf = layer.flops / t / 1e12
                    rows.append({"k": ks, "c": c, "h": h, "dtype": dt, "us": round(t * 1e6, 2),
                                 "tflops": round(tf, 1),
                                 "frac_of_peak": round(tf / peak_burst, 3) if dt != "fp32" else None})
                    layer.close()
    clk = clocks.stop()
    launches = backend.launch_count() - launches0
    flush.free()
    if rank == 0:
        def agg(dt):
            sel = [r for r in rows if r["dtype"] == dt]
            fl = sum(2 * n * r["h"] * r["h"] * r["c"] * r["c"] * r["k"] * r["k"] for r in sel)
            return fl / sum(r["us"] * 1e-6 for r in sel) / 1e12
        line = {
            "metric": "conv2d+BN+ReLU layer sweep TFLOP/s (config 2)", "value": agg("bf16"),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs, He-normal weights)",
            "config": {"workload": "32 layer shapes x {fp32, bf16, fp16}, N=32, L2 flushed "
                                   "before every timed run", "batch": n},
            "aggregate_tflops": {dt: round(agg(dt), 1) for dt in ("fp32", "bf16", "fp16")},
            "peak": peak_burst, "peak_kind": f"bf16_tflops burst ({peak_src})",
            "sweep": rows, "clocks": clk, "gpu_launches": launches,
            "kernel_error": backend.kernel_error(),
        }
        return line
    return None


def run_mobilenet(args, world, rank, local, dist):
    """Config 5: MobileNet-style stack fp16 inference, batch 256 per GPU (graph replay).

    The depthwise kernels' HBM rate comes from a graph of the forward's depthwise launches
    alone, replayed back to back (each reads its own input buffer and writes its own output,
    over 1 GB in all, larger than L2); algorithmic bytes = input read once + output written
    once. The pointwise convs' rate comes from launch-duration stamps (conv_stamp_profile)."""
    import ctypes

    import torch
    from omnimatchdeeplearningtool_b200 import _lib, backend, synth
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    backend.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(backend.stream_handle(), device=local)
    batch = args.batch
    net = synth.mobilenet_spec()
    plan = InferencePlan(net, synth.make_weights(net), batch=batch, dtype=_lib.DTYPE_F16)
    plan.set_input(synth.normal_input(batch, seed=rank))
    plan.launch()
    call("omCudaSynchronize")
    plan.capture()
    for _ in range(args.warmup):
        plan.launch()
    call("omCudaSynchronize")
    clocks = ClockSampler(local)
    clocks.start()
    _barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(args.steps):
            plan.launch()
        e1.record()
    _wait_gil_free(e1)
    _barrier(dist)
    clk = clocks.stop()
    t = _max_over_ranks(dist, e0.elapsed_time(e1) / 1e3)
    # depthwise launches alone, as one graph
    dw = [i for i, m in enumerate(plan.meta) if m.get("kind") == "depthwise"]
    dw_bytes = sum(batch * plan.meta[i]["cs"] * 2 * (plan.meta[i]["h"] * plan.meta[i]["wd"] +
                                                     plan.meta[i]["p"] * plan.meta[i]["q"])
                   for i in dw)
    call("omCudaGraphBeginCapture")
    try:
        for i in dw:
            plan.ops[i]()
    finally:
        g = ctypes.c_void_p()
        st = lib.omCudaGraphEndCapture(ctypes.byref(g))
    _lib.check(st, "omCudaGraphEndCapture")
    for _ in range(3):
        call("omCudaGraphLaunch", g.value)
    reps = max(3, args.steps)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record()
        for _ in range(reps):
            call("omCudaGraphLaunch", g.value)
        e3.record()
    e3.synchronize()
    dw_s = e2.elapsed_time(e3) / 1e3 / reps
    lib.omCudaGraphDestroy(g.value)
    durs, _ = conv_stamp_profile(plan, 5)
    tc_s = float(sum(durs))
    peak_burst, _, hbm, peak_src = _peaks()
    dw_gbs = dw_bytes / dw_s / 1e9
    tc_tf = plan.conv_flops / tc_s / 1e12
    line = None
    if rank == 0:
        line = {
            "metric": "MobileNet-style stack fp16 images/s (config 5)",
            "value": args.steps * batch * world / t, "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": {"workload": "mobilenet-style stack fp16 inference",
                                            "batch_per_gpu": batch},
            "roofline": {"bound": "hbm", "kernel": "depthwise_nhwc (3x3, BN + ReLU6 fused)",
                         "achieved": dw_gbs, "peak": hbm, "unit": "GB/s", "frac": dw_gbs / hbm,
                         "peak_kind": f"hbm_gbs ({peak_src})",
                         "method": "graph of the depthwise launches alone, replayed",
                         "depthwise_us_per_step": dw_s * 1e6,
                         "pointwise_tc_us_per_step": tc_s * 1e6,
                         "pointwise_tc_tflops": tc_tf,
                         "pointwise_frac_of_burst": tc_tf / peak_burst},
            "clocks": clk, "kernel_error": backend.kernel_error(),
        }
    plan.close()
    return line


def extra_configs(args, world, rank, local, dist):
    """Short runs of configs 2, 3 and 5 for the default N=1 line (each with its own clocks)."""
    import copy
    out = {}
    a = copy.copy(args)
    a.steps, a.warmup = 2, 1
    sw = run_sweep(a, world, rank, local, dist)
    if sw:
        out["conv_sweep"] = {k: sw[k] for k in ("value", "unit", "aggregate_tflops", "peak",
                                                 "peak_kind", "clocks", "gpu_launches")}
        out["conv_sweep"]["config"] = sw["config"]
        best = max((r for r in sw["sweep"] if r["dtype"] == "bf16"), key=lambda r: r["tflops"])
        out["conv_sweep"]["best_bf16_layer"] = best
    a = copy.copy(args)
    a.steps, a.warmup, a.batch = 5, 3, 128
    tr = run_train(a, world, rank, local, dist)
    if tr:
        _, _, _, src = _peaks()
        out["r18_train"] = {k: tr[k] for k in ("value", "unit", "ms_per_step", "tflops_per_gpu",
                                                "config", "clocks", "loss_last_step")}
        out["r18_train"]["tf32_dense_nominal_tflops"] = 1100.0
        out["r18_train"]["frac_of_tf32_nominal"] = tr["tflops_per_gpu"] / 1100.0
    a = copy.copy(args)
    a.steps, a.warmup, a.batch = 10, 3, 256
    mb = run_mobilenet(a, world, rank, local, dist)
    if mb:
        out["mobilenet"] = {k: mb[k] for k in ("value", "unit", "ms_per_step", "roofline",
                                                "config", "clocks")}
    return out


def run_reference(args, world, rank, dist):
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    net = synth.resnet_spec(50)
    w = synth.make_weights(net)
    batch = args.ref_batch
    x = synth.normal_input(batch)
    cores = _host_threads()
    orc.set_threads(cores)
    h = orc.ref_model(1, 1000, w, net)
    out = np.empty((batch, 1000), np.float32)
    if h is not None:
        kind = "reference"
        run = lambda: orc.ref().omref_model_forward(h, x.ctypes.data, batch, 224, 224, out.ctypes.data)
    else:
        kind = "port"
        run = lambda: orc.forward(net, w, x)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    v = args.steps * batch / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs, He-normal weights)",
        "config": {"workload": f"resnet50 inference (reference CPUBackend, fp32), batch {batch} "
                               "per step at 224x224", "batch": batch},
        "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": kind,
                         "sample": f"ResNet-50 fp32 forward, batch {batch} per step, "
                                   f"OMP threads={cores}"},
        "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def conv_stamp_profile(plan, reps: int):
    """Per-launch durations of the plan's tensor-core conv kernels inside a CUDA-graph replay.

    A second graph of the same forward is captured with launch-duration stamps on
    (omCudaConvStamps: every conv_tc_kernel CTA writes %globaltimer at its start and its end);
    it is replayed `reps` times, and after each replay a launch's duration is its last CTA end
    minus its first CTA start. Returns (median seconds per tensor-core op in plan order, median
    seconds of one stamped replay from CUDA events around it)."""
    import ctypes

    import numpy as np
    import torch
    from omnimatchdeeplearningtool_b200 import _lib, backend
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    n_tc = len(plan.tc_op_index)
    cap = n_tc * 4 * 148
    stamps = DeviceBuffer(cap * 16)
    call("omCudaSynchronize")
    call("omCudaConvStamps", stamps.ptr, cap)
    call("omCudaGraphBeginCapture")
    try:
        for fn in plan.ops:
            fn()
    finally:
        g = ctypes.c_void_p()
        st = lib.omCudaGraphEndCapture(ctypes.byref(g))
    _lib.check(st, "omCudaGraphEndCapture")
    first = (ctypes.c_int * n_tc)()
    ctas = (ctypes.c_int * n_tc)()
    count = ctypes.c_int()
    call("omCudaConvStampLaunches", first, ctas, n_tc, ctypes.byref(count))
    call("omCudaConvStamps", None, 0)
    if count.value != n_tc:
        raise RuntimeError(f"stamped {count.value} conv launches, expected {n_tc}")
    stream = torch.cuda.ExternalStream(backend.stream_handle())
    per_rep, replay = [], []
    for r in range(reps + 2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record()
            call("omCudaGraphLaunch", g.value)
            e1.record()
        e1.synchronize()
        raw = stamps.to_numpy((cap, 2), np.uint64).astype(np.int64)
        if r < 2:
            continue  # warm-up replays
        d = [(raw[f:f + c, 1].max() - raw[f:f + c, 0].min()) * 1e-9 for f, c in zip(first, ctas)]
        per_rep.append(d)
        replay.append(e0.elapsed_time(e1) / 1e3)
    lib.omCudaGraphDestroy(g.value)
    stamps.free()
    return list(np.median(np.array(per_rep), axis=0)), float(np.median(replay))


def conv_groups(plan):
    """Label of each tensor-core op: stem, fc, a fused 3x3 + 1x1 pair, 256-wide (long reductions
    on 256-wide tiles), 3x3 or 1x1 (the rest, by filter size)."""
    import ctypes
    from omnimatchdeeplearningtool_b200._lib import call
    labels = []
    for i in plan.tc_op_index:
        m = plan.meta[i]
        if m.get("kind") == "stem":
            labels.append("stem + max pool" if m.get("pool") else "stem")
            continue
        if m.get("kind") == "pair":
            labels.append("3x3+1x1 pair")
            continue
        if m.get("out_dtype") == 0:  # fp32 logits: the classifier
            labels.append("fc")
            continue
        tp = (ctypes.c_int * 4)()
        call("omCudaConvTilePlan", plan.batch, m["h"], m["wd"], m["cs"], m["k"], m["ks"], m["ks"],
             m["stride"], m["pad"], int(m["res"] is not None), tp)
        labels.append("256-wide" if tp[0] == 256 else ("3x3" if m["ks"] == 3 else "1x1"))
    return labels


def conv_op_flops(plan):
    out = []
    for i in plan.tc_op_index:
        m = plan.meta[i]
        out.append(m["flops"] if "flops" in m else
                   2 * plan.batch * m["p"] * m["q"] * m["k"] * m["c"] * m["ks"] * m["ks"])
    return out


def _serve_e2e(plan, x, args, world, dist, stream):
    """Images/s through InferencePlan.serve with pinned host buffers (max over ranks)."""
    import ctypes

    import numpy as np
    import torch
    from omnimatchdeeplearningtool_b200._lib import call
    in_bytes = plan.in_bytes
    out_bytes = plan.batch * plan.net.classes * 4
    hin = [ctypes.c_void_p() for _ in range(2)]
    hout = [ctypes.c_void_p() for _ in range(2)]
    src = plan.host_input(x)
    for b in hin:
        call("omCudaMallocHost", ctypes.byref(b), in_bytes)
        ctypes.memmove(b.value, src.ctypes.data, in_bytes)
    for b in hout:
        call("omCudaMallocHost", ctypes.byref(b), out_bytes)
    ins = [hin[i % 2].value for i in range(args.steps)]
    outs = [hout[i % 2].value for i in range(args.steps)]
    plan.serve(ins[:max(3, args.warmup)], outs[:max(3, args.warmup)])
    call("omCudaSynchronize")
    _barrier(dist)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record()
        plan.serve(ins, outs)
        e3.record()
    e3.synchronize()
    call("omCudaSynchronize")
    _barrier(dist)
    t = _max_over_ranks(dist, e2.elapsed_time(e3) / 1e3)
    logits = np.frombuffer(ctypes.string_at(outs[-1], out_bytes), np.float32).copy()
    # copy-only: the same per-step host->device copies alone on the transfer stream
    call("omCudaSynchronize")
    _barrier(dist)
    t0 = time.perf_counter()
    for i in range(args.steps):
        call("omCudaTransferH2D", plan.inputs[i % 2].ptr, ins[i], in_bytes)
    call("omCudaSyncTransferStream")
    t_copy = _max_over_ranks(dist, time.perf_counter() - t0)
    for b in hin + hout:
        call("omCudaFreeHost", b.value)
    return (args.steps * plan.batch * world / t, in_bytes, out_bytes, logits,
            in_bytes * args.steps / t_copy / 1e9)


def run_ours(args, world, rank, local, dist):
    global BATCH
    BATCH = args.batch
    import numpy as np
    import torch
    from omnimatchdeeplearningtool_b200 import _lib, backend, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.plan import InferencePlan

    backend.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(backend.stream_handle(), device=local)
    net = synth.resnet_spec(50)
    weights = synth.make_weights(net)
    plan = InferencePlan(net, weights, batch=BATCH, dtype=_lib.DTYPE_BF16)
    x = synth.normal_input(BATCH, seed=rank)
    plan.set_input(x)
    plan.launch()
    call("omCudaSynchronize")
    plan.capture()
    kernels_per_step = plan.n_launches

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # ---------------------------------------------------------------- device-resident value
    for _ in range(args.warmup):
        plan.launch()
    call("omCudaSynchronize")
    clocks = ClockSampler(local)
    clocks.start()
    _barrier(dist)
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(args.steps):
            plan.launch()
        e1.record()
    _wait_gil_free(e1)
    torch.cuda.synchronize()
    _barrier(dist)
    clk = clocks.stop()
    t_dev = e0.elapsed_time(e1) / 1e3
    t_dev_max = _max_over_ranks(dist, t_dev)
    value = args.steps * BATCH * world / t_dev_max

    # ---------------------------------------------------------------- end to end, host buffers
    # InferencePlan.serve: per step, the step's NCHW batch goes host->device on the transfer
    # stream (pinned source) and its logits come back device->host; the copy of step i+1
    # overlaps the forward of step i. The headline takes the image in bf16 (the plan's
    # input_dtype: half the bytes of fp32, logits bit-identical); the fp32-image figure and a
    # copy-only timing of each stand beside it.
    plan16 = InferencePlan(net, weights, batch=BATCH, dtype=_lib.DTYPE_BF16,
                           input_dtype=_lib.DTYPE_BF16)
    plan16.set_input(x)
    plan16.launch()
    call("omCudaSynchronize")
    plan16.capture()
    e2e16, in16, out_bytes, logits16, copy16 = _serve_e2e(plan16, x, args, world, dist, stream)
    plan16.close()
    e2e32, in32, _, logits32, copy32 = _serve_e2e(plan, x, args, world, dist, stream)
    finite = bool(np.isfinite(logits32).all() and np.array_equal(logits16, logits32))
    # 8-bit images as a camera or decoder delivers them, normalised on the GPU inside the stem's
    # pre-pass (the reference's ImageNet normalisation of inferBatch): a quarter of the fp32
    # bytes. Checked against the fp32 image sample / 255 normalised on the host.
    from omnimatchdeeplearningtool_b200.plan import IMAGENET_NORM
    x8 = np.random.Generator(np.random.PCG64(1000 + rank)).integers(
        0, 256, (BATCH, 3, 224, 224), dtype=np.uint8)
    plan8 = InferencePlan(net, weights, batch=BATCH, dtype=_lib.DTYPE_BF16,
                          input_dtype=_lib.DTYPE_U8, input_norm=IMAGENET_NORM)
    plan8.set_input(x8)
    plan8.launch()
    call("omCudaSynchronize")
    plan8.capture()
    e2e8, in8, _, logits8, copy8 = _serve_e2e(plan8, x8, args, world, dist, stream)
    plan8.close()
    mean = np.asarray(IMAGENET_NORM[0], np.float32).reshape(1, 3, 1, 1)
    inv = (np.float32(1.0) / np.asarray(IMAGENET_NORM[1], np.float32)).reshape(1, 3, 1, 1)
    x8f = ((x8.astype(np.float32) / np.float32(255.0) - mean) * inv).astype(np.float32)
    plan.set_input(x8f)
    plan.launch()
    ref8 = plan.logits.to_numpy((BATCH, net.classes)).reshape(-1)
    u8_identical = bool(np.array_equal(logits8, ref8))

    # ---------------------------------------------------------------- conv kernel roofline
    durs, replay_s = conv_stamp_profile(plan, max(3, min(args.steps, 10)))
    conv_s = float(sum(durs))
    flops = conv_op_flops(plan)
    labels = conv_groups(plan)
    groups = {}
    for lab, d, f in zip(labels, durs, flops):
        gsum = groups.setdefault(lab, {"launches": 0, "us": 0.0, "gflop": 0.0})
        gsum["launches"] += 1
        gsum["us"] += d * 1e6
        gsum["gflop"] += f / 1e9
    for gsum in groups.values():
        gsum["share_of_conv_time"] = round(gsum["us"] / (conv_s * 1e6), 4)
        gsum["tflops"] = round(gsum["gflop"] / 1e3 / (gsum["us"] * 1e-6), 1)
        gsum["us"] = round(gsum["us"], 1)
        gsum["gflop"] = round(gsum["gflop"], 1)
    achieved = plan.conv_flops / conv_s / 1e12
    peak_burst, peak_sust, _, peak_src = _peaks()
    err = backend.kernel_error()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_dev_max / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs, He-normal weights, BN running stats seeded)",
            "config": {"workload": "resnet50 (ImageNet stem) bf16 inference, NHWC fused plan, "
                                   "CUDA-graph replay", "batch_per_gpu": BATCH,
                       "global_batch": BATCH * world, "image": "3x224x224",
                       "parallelism": f"batch-sharded x{world}, no collective",
                       "l2": "inputs larger than L2 (154 MB fp32 input, >1 GB activations "
                             "per step)"},
            "e2e": {"value": e2e16, "unit": "images/s", "h2d_bytes_per_step": in16,
                    "d2h_bytes_per_step": out_bytes,
                    "input": "bf16 NCHW image (InferencePlan input_dtype; logits bit-identical "
                             "to the fp32-image plan)",
                    "fp32_input": {"value": e2e32, "h2d_bytes_per_step": in32},
                    "u8_input": {"value": e2e8, "h2d_bytes_per_step": in8,
                                 "input": "uint8 NCHW image, / 255 and ImageNet-normalised on "
                                          "the GPU in the stem's pre-pass",
                                 "logits_identical_to_host_normalised_fp32": u8_identical},
                    "h2d_copy_only_gbs": {"bf16_input": copy16, "fp32_input": copy32,
                                          "u8_input": copy8}},
            "roofline": {"bound": "tensor", "kernel": "conv_tc_kernel (tcgen05 implicit GEMM)",
                         "achieved": achieved, "peak": peak_burst, "unit": "TFLOP/s",
                         "frac": achieved / peak_burst,
                         "peak_kind": f"bf16_tflops burst ({peak_src}): the timed region is a "
                                      "short graph replay",
                         "frac_of_sustained": achieved / peak_sust,
                         "conv_us_per_step": conv_s * 1e6,
                         "stamped_replay_us": replay_s * 1e6,
                         "conv_share_of_step": conv_s / (t_dev_max / args.steps),
                         "method": "per-CTA %globaltimer stamps in a graph replay of the same "
                                   "forward: each launch = last CTA end - first CTA start",
                         "groups": groups,
                         "traffic": CONV_TRAFFIC_B64 * BATCH / 64,
                         "traffic_unit": "bytes per step, conv launches (ncu at batch 64, "
                                         "scaled by batch)",
                         "flops_per_step": plan.conv_flops,
                         "launches_per_step": len(plan.tc_op_index)},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clk,
            "kernel_error": err,
            "logits_finite_and_bf16_input_identical": finite,
        }
        if world == 1 and not args.no_extra_configs:
            line["configs"] = extra_configs(args, world, rank, local, dist)
        if world == 1 and not args.no_cpu_baseline:
            v, kind, cores, sample = _reference_cpu(8, 2, 10.0)
            line["cpu_baseline"] = {"value": v, "unit": "images/s", "cores": cores,
                                    "kind": kind, "sample": sample}
        print(json.dumps(line), flush=True)
    plan.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="r50-infer",
                    choices=["r50-infer", "r18-train", "mobilenet-infer", "conv-sweep"],
                    help="r50-infer is the headline metric; the others are configs 3, 5 and 2")
    ap.add_argument("--ref-batch", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the short config 2/3/5 runs the default N=1 line carries")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="images per GPU (the metric is quoted at 256; smaller sizes are for "
                         "profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local, dist = _dist()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, dist)
        elif args.workload in ("r18-train", "mobilenet-infer", "conv-sweep"):
            fn = {"r18-train": run_train, "mobilenet-infer": run_mobilenet,
                  "conv-sweep": run_sweep}[args.workload]
            line = fn(args, world, rank, local, dist)
            if line is not None:
                print(json.dumps(line), flush=True)
        else:
            run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
