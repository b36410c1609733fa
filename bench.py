#!/usr/bin/env python
"""YOLO26n FP32 640x640 inference throughput on B200 (images/s).

Workload: the YOLO26n forward (backbone, neck, Detect head, top-300 decode)
on seeded U[0,1) 640x640 images with seeded random-init weights in the
converter's .bin layout, 64 images per GPU per step.  64 is the batch of the
8-GPU benchmark configuration; each GPU runs its own 64-image shard
(image-parallel, no collective), so scaling is weak.

  value    images/s of the whole job with the inputs already in HBM:
           K graph launches of yb_cuda_forward_device, timed with CUDA events
           on the launching stream, max over ranks.
  e2e      the same through the host API yb_cuda_forward: pinned host input
           copied to HBM every step, detections copied back every step.
  roofline the tcgen05 convolution family (every conv launch of a forward),
           algorithmic bytes / measured time against the measured HBM copy
           bandwidth, plus conv TFLOP/s against the measured bf16 peak.
  cpu_baseline  the reference's own C forward (compiled from its sources under
           oracle/_ref) on the host cores, one process per core.

Further legs in the same JSON line:
  strong   the batch-64 benchmark as a fixed global batch (64/N images per
           GPU), device-resident and end to end with the detections gathered
           into rank 0's host memory;
  int8     the INT8 forward on the same images (device calibration over 32
           seeded images), with its own roofline object;
  config5  the s-width INT8 forward at 1280x1280, global batch 16 (16/N per
           GPU);
  int8_conv_sweep / fp32_conv_sweep  the five isolated convolution shapes of
           the benchmark's sweep, device-resident, TOPS / TFLOP/s and GB/s.

`--impl reference` times that CPU reference alone, on the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "yolo-baremetal_b200")
sys.path.insert(0, PKG)

METRIC = "images/sec YOLO26n 640² FP32 & INT8 at 1/2/4/8 B200; conv TFLOPS/TOPS vs peak"
UNIT = "images/s"
DATA = ("synthetic: seeded U[0,1) 640x640 images (numpy PCG64), seeded random-init YOLO26n weights "
        "(Kaiming conv, BN gamma 1+-0.1, beta/mean N(0,0.1), var U(0.5,1.5)) in the converter .bin layout")
# DRAM bytes (read + write) per algorithmic byte of the convolution launches:
# ncu (dram__bytes_read.sum + dram__bytes_write.sum, one kernel, three
# launches) of the three longest conv_tc_kernel launches of a 16-image
# 640x640 forward (model.1, model.2.cv2, model.3): 372.4 MB of DRAM traffic
# for 472.1 MB of algorithmic bytes (inputs and weights read once, outputs
# written once).  Below 1: no operand is re-read from DRAM; part of each
# output is still in L2 when the launch ends.
CONV_DRAM_PER_ALGO = 372.4 / 472.1
CONV_DRAM_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the three longest conv_tc_kernel "
                    "launches of a 16-image forward (model.1, model.2.cv2, model.3; one kernel, 1 + 2 launches): "
                    "0.79 DRAM bytes per algorithmic byte, applied to this line's algorithmic bytes per launch")


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons while the timed region runs.

    Reads NVML in a background thread every 10 ms (read-only queries), so
    even a timed region of a few hundred milliseconds gets dozens of samples;
    falls back to `nvidia-smi -lms 100` when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits.
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, bus_id: str | None):
        self.bus_id = bus_id
        self.proc = None
        self.out = None
        self.thread = None
        self.stop = None
        self.rows = []  # (sm_mhz, max_mhz, reason bits)

    def _nvml_loop(self, nv, h):
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.rows.append((float(sm), float(mx), int(fn(h))))
            except Exception:
                pass
            self.stop.wait(0.01)

    def __enter__(self):
        if not self.bus_id:
            return self
        try:
            import threading

            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByPciBusId(self.bus_id.encode())
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                   "-i", self.bus_id]
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the first sample land before the timed region starts
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        if self.thread:
            for s, m, bits in self.rows:
                sm.append(s)
                mx = max(mx, m)
                for n, b in self.REASON_BITS.items():
                    if bits & b:
                        reasons.add(n)
            source = "nvml"
        else:
            if not self.out:
                return None
            try:
                rows = [r.split(",") for r in open(self.out.name).read().strip().splitlines() if r.strip()]
                os.unlink(self.out.name)
            except Exception:
                return None
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in rows:
                try:
                    sm.append(float(r[1]))
                    mx = max(mx, float(r[2]))
                    for i, n in enumerate(names):
                        if r[5 + i].strip().lower().startswith("active"):
                            reasons.add(n)
                except Exception:
                    continue
            source = "nvidia-smi"
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": source}


def bus_id_of(dev: int):
    try:
        import torch

        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return None


# ---------------------------------------------------------------- CPU reference
def _ref_worker(conn, weights, H, W, seed, use_ref):
    """One host core: loads the CPU implementation once, then runs one forward
    per 'go' message and replies with the elapsed seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np  # noqa: F401
    import yb_weights as yw

    img = yw.make_input(seed, H, W).reshape(-1)
    if use_ref:
        import oracle as orc

        lib = orc.Reference.lib()
        lib.ref_open.restype = C.c_void_p
        lib.ref_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int]
        lib.ref_run.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        h = lib.ref_open(weights.encode(), H, W, 1)
        run = lambda: lib.ref_run(h, img.ctypes.data, None)  # noqa: E731
    else:
        import oracle as orc

        o = orc.Oracle(weights)
        run = lambda: o.forward(img.reshape(1, 3, H, W))  # noqa: E731
    conn.send("ready")
    while True:
        msg = conn.recv()
        if msg == "stop":
            break
        t0 = time.perf_counter()
        st = run()
        conn.send((time.perf_counter() - t0, st if isinstance(st, int) else 0))


class CpuPool:
    def __init__(self, procs, weights, H, W, use_ref):
        ctx = mp.get_context("spawn")
        self.conns, self.ps = [], []
        for i in range(procs):
            a, b = ctx.Pipe()
            p = ctx.Process(target=_ref_worker, args=(b, weights, H, W, 1000 + i, use_ref), daemon=True)
            p.start()
            self.conns.append(a)
            self.ps.append(p)
        for c in self.conns:
            assert c.recv() == "ready"

    def step(self):
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        res = [c.recv() for c in self.conns]
        if any(r[1] != 0 for r in res):
            raise RuntimeError("CPU reference forward failed")
        return time.perf_counter() - t0

    def close(self):
        for c in self.conns:
            c.send("stop")
        for p in self.ps:
            p.join(timeout=10)


def cpu_kind():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    return ("reference", True) if orc.Reference.available() else ("port", False)


def cpu_baseline(weights, H, W, procs, steps):
    kind, use_ref = cpu_kind()
    pool = CpuPool(procs, weights, H, W, use_ref)
    try:
        total = sum(pool.step() for _ in range(steps))
    finally:
        pool.close()
    return {"value": procs * steps / total, "unit": UNIT, "cores": procs, "kind": kind,
            "sample": f"{procs} processes x {steps} single-image {W}x{H} forwards (one per core), wall time"}


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# --------------------------------------------------------------------- main
def make_weights(tmpdir):
    import yb_weights as yw

    path = os.path.join(tmpdir, "yolo26n_seed0.bin")
    yw.write_bin(path, yw.random_state("n", 0))
    return path


def config(n, batch, hw):
    return {"workload": f"YOLO26n FP32 forward + top-300 decode, {hw}x{hw}, {batch} images per GPU "
                        f"(the batch-64 benchmark shard), image-parallel",
            "images_per_gpu": batch, "global_batch": batch * n, "input_hw": [hw, hw],
            "parallelism": f"dp{n} (image sharding, no collective)",
            "l2_policy": "inputs larger than L2 (315 MB of input and >3 GB of activations per GPU per step)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    with tempfile.TemporaryDirectory() as td:
        weights = make_weights(td)
        procs = os.cpu_count() or 1
        kind, use_ref = cpu_kind()
        pool = CpuPool(procs, weights, args.hw, args.hw, use_ref)
        try:
            for _ in range(args.warmup):
                pool.step()
            total = sum(pool.step() for _ in range(args.steps))
        finally:
            pool.close()
    value = procs * args.steps / total
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA,
            "config": config(args.gpus, args.batch, args.hw), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": kind,
                             "sample": f"each step: {procs} processes run one {args.hw}x{args.hw} forward each "
                                       f"({cpu_model()})"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def parse_cpulist(text):
    """CPU ids of a sysfs cpulist such as "0-55,112-167"."""
    cpus = set()
    for part in text.strip().split(","):
        if part:
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def bind_to_gpu_numa_node(dev):
    """Restricts this process to the CPUs of the NUMA node that hosts GPU
    `dev`'s PCIe link, before any pinned host buffer is allocated: the pages
    are then placed on that node (first touch) and the host<->device copies
    do not cross the socket interconnect.  Returns the node, or None where
    sysfs does not tell it (the process is then left unbound)."""
    import torch

    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = parse_cpulist(f.read()) & os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def run_ours(args):
    import numpy as np
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    numa_node = bind_to_gpu_numa_node(local)
    dist = None
    gather_group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        # Host-memory group for gathering detections into rank 0's host memory.
        gather_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
    B, H = args.batch, args.hw
    tmpdir = tempfile.mkdtemp(prefix=f"yb_bench_{rank}_")
    weights = make_weights(tmpdir)
    model = yb.Model(weights, device=local)
    imgs = yw.make_batch(range(rank * B + 1, rank * B + B + 1), H, H)
    host_in = torch.from_numpy(imgs).pin_memory()
    host_out = torch.empty((B, 300, 6), dtype=torch.float32).pin_memory()
    L = yb.lib()

    def e2e_step():
        yb.check(L.yb_cuda_forward(model.ctx, host_in.data_ptr(), B, H, H, host_out.data_ptr(), 300, None, None, None),
                 "yb_cuda_forward")

    e2e_step()  # builds the pipelined plans (16-image sub-batches)
    # Device-resident leg: the whole batch as one plan; its input buffer is
    # filled once with this rank's images, outside the timed region.
    d_in, d_out = model.plan_io(B, H, H)
    dev_imgs = host_in.to(f"cuda:{local}")
    # A dedicated stream: the library launches on exactly this stream, so the
    # CUDA events below bracket the forward's kernels.
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    model.forward_device(dev_imgs.data_ptr(), d_out, B, H, H, 300, stream.cuda_stream)
    torch.cuda.synchronize()
    del dev_imgs

    def dev_step():
        model.forward_device(d_in, d_out, B, H, H, 300, stream.cuda_stream)

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        dev_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(bus_id_of(local) if rank == 0 else None) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            dev_step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = clk.summary() if rank == 0 else None

    # End to end through the host API: H2D of the pinned batch, forward, D2H.
    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    # End to end from 8-bit frames (the reference's camera path: 640x640 RGB,
    # resize_rgb_bilinear + preprocess on the device): a quarter of the bytes.
    rgb8 = rgb8_frames(rank, B, H)
    e2e8_s = timed_rgb8(L, model, rgb8, host_out, B, H, args, barrier, max_over_ranks)
    es_s = timed_stream(model, host_in, B, H, args, barrier, max_over_ranks)
    es8_s = timed_stream(model, rgb8, B, H, args, barrier, max_over_ranks, rgb8=True)

    n_ops = C.c_int()
    yb.check(L.yb_cuda_profile_ops(model.ctx, B, H, H, 300, 0, None, 0, C.byref(n_ops)), "yb_cuda_profile_ops")
    line = None
    if rank == 0:
        stats = (OpStat * n_ops.value)()
        yb.check(L.yb_cuda_profile_ops(model.ctx, B, H, H, 300, 3, stats, n_ops.value, C.byref(n_ops)),
                 "yb_cuda_profile_ops")
        conv = [s for s in stats if s.kind == 0]
        conv_ms = sum(s.ms for s in conv)
        conv_bytes = sum(s.bytes for s in conv)
        conv_flops = sum(s.flops for s in conv)
        all_ms = sum(s.ms for s in stats)
        hbm, bf16, src = peaks()
        achieved = conv_bytes / (conv_ms * 1e-3) / 1e9
        per_kind = {}
        for s in stats:
            k = ["conv_tc", "stem", "dwconv", "maxpool", "attention", "decode", "topk"][s.kind]
            d = per_kind.setdefault(k, {"launches": 0, "ms": 0.0})
            d["launches"] += 1
            d["ms"] += s.ms
        for d in per_kind.values():
            d["share"] = d["ms"] / all_ms
        value = world * B * args.steps / (dev_ms * 1e-3)
        traffic = CONV_DRAM_PER_ALGO * conv_bytes / len(conv)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "precision": "fp32 activations in HBM; conv products as bf16 hi/lo pairs (3 tcgen05 UMMAs) "
                             "with fp32 accumulation in TMEM",
                "data": DATA, "config": config(world, B, H),
                "e2e": {"value": world * B * args.steps / es_s, "unit": UNIT,
                        "h2d_bytes_per_step": world * host_in.numel() * 4,
                        "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": STREAM_NOTE,
                        "pinned_buffers_numa_node_rank0": numa_node},
                "e2e_sync": {"value": world * B * args.steps / e2e_s, "unit": UNIT,
                             "h2d_bytes_per_step": world * host_in.numel() * 4,
                             "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": SYNC_NOTE},
                "e2e_rgb8": {"value": world * B * args.steps / es8_s, "unit": UNIT,
                             "h2d_bytes_per_step": world * rgb8.numel(),
                             "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": STREAM_NOTE,
                             "sync_value": world * B * args.steps / e2e8_s,
                             "source": f"{B} seeded uint8 RGB frames {H}x{H} per GPU per step through "
                                       "yb_cuda_forward_rgb8_submit (device resize_rgb_bilinear + /255, then the "
                                       "forward); same metric, 8-bit inputs instead of the fp32 tensor; "
                                       "sync_value: one blocking yb_cuda_forward_rgb8 per step"},
                "gpu_launches": n_ops.value * args.steps,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "traffic": traffic,
                             "traffic_source": CONV_DRAM_SOURCE,
                             "kernel": "all tcgen05 convolution launches of one forward (conv_tc_kernel and the fused "
                                       "bottleneck_tc_kernel)",
                             "launches": len(conv), "bytes_per_launch": conv_bytes / len(conv),
                             "ms_per_launch": conv_ms / len(conv), "peak_source": src},
                "conv_tflops": {"achieved": conv_flops / (conv_ms * 1e-3) / 1e12, "peak": bf16,
                                "frac": conv_flops / (conv_ms * 1e-3) / 1e12 / bf16, "peak_source": src,
                                "note": "algorithmic FP32 FLOPs; the tensor pipe executes 3x (split-bf16)"},
                "forward_breakdown_ms": {k: round(v["ms"], 4) for k, v in per_kind.items()},
                "forward_share": {k: round(v["share"], 4) for k, v in per_kind.items()},
                "clocks": clocks}
    if not args.no_strong and args.global_batch % world == 0:
        st = strong_leg(model, args, world, rank, local, barrier, max_over_ranks, gather_group)
        if rank == 0:
            line["strong"] = st
    if not args.no_int8:
        i8 = int8_leg(model, args, world, rank, stream, host_in, host_out, barrier, max_over_ranks)
        if rank == 0:
            line["int8"] = i8
    model.close()
    if not args.no_config5 and CONFIG5_GLOBAL % world == 0:
        c5 = config5_leg(args, world, rank, local, tmpdir, barrier, max_over_ranks)
        if rank == 0:
            line["config5"] = c5
    if rank == 0 and not args.no_int8_sweep:
        line["int8_conv_sweep"] = int8_conv_sweep(peaks()[0])
    if rank == 0 and not args.no_fp32_sweep:
        hbm, bf16, src = peaks()
        line["fp32_conv_sweep"] = fp32_conv_sweep(hbm, bf16, src)
    if dist:
        dist.barrier()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        procs = min(os.cpu_count() or 1, 64)
        line["cpu_baseline"] = cpu_baseline(weights, H, H, procs, 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def rgb8_frames(rank, B, H):
    import numpy as np
    import torch

    rng = np.random.default_rng(20000 + rank)
    return torch.from_numpy(rng.integers(0, 256, size=(B, H, H, 3), dtype=np.uint8)).pin_memory()


def timed_rgb8(L, model, rgb8, host_out, B, H, args, barrier, max_over_ranks):
    """Wall time of K yb_cuda_forward_rgb8 calls (pinned 8-bit frames in,
    detections out), max over ranks."""
    import torch

    import yolo_b200 as yb

    def step():
        yb.check(L.yb_cuda_forward_rgb8(model.ctx, rgb8.data_ptr(), B, H, H, 0, H, H, host_out.data_ptr(), 300),
                 "yb_cuda_forward_rgb8")

    for _ in range(max(1, args.warmup // 2)):
        step()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    e = max_over_ranks(time.perf_counter() - t0)
    barrier()
    return e


def timed_stream(model, src, B, H, args, barrier, max_over_ranks, rgb8=False):
    """Wall time of K streamed steps (yb_cuda_forward_submit or
    yb_cuda_forward_rgb8_submit, then yb_cuda_forward_wait): two batches in
    flight, each step copying its own pinned input to the device and its
    detections back into one of two pinned output buffers; max over ranks."""
    import torch

    outs = [torch.empty((B, 300, 6), dtype=torch.float32).pin_memory() for _ in range(2)]

    def run(k):
        pending = []
        for i in range(k):
            if len(pending) == 2:
                model.wait(pending.pop(0))
            o = outs[i % 2]
            if rgb8:
                pending.append(model.submit_rgb8(src.data_ptr(), B, H, H, o.data_ptr(), H, H))
            else:
                pending.append(model.submit(src.data_ptr(), B, H, H, o.data_ptr()))
        for t in pending:
            model.wait(t)

    run(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    run(args.steps)
    torch.cuda.synchronize()
    e = max_over_ranks(time.perf_counter() - t0)
    barrier()
    return e


STREAM_NOTE = ("streaming: yb_cuda_forward_submit / yb_cuda_forward_wait with two batches in flight; every step "
               "copies its own pinned input to the device and its detections back inside the timed region")
SYNC_NOTE = "one blocking yb_cuda_forward call per step (pipelined 16-image sub-batches inside the call)"


INT8_KINDS = ["conv_i8", "stem_i8", "dw3x3_i8", "maxpool_concat_i8", "attention_i8", "decode", "topk"]
INT8_CALIB_IMAGES = 32  # seeded U[0,1) calibration images (the benchmark's INT8 recipe)


def int8_leg(model, args, world, rank, stream, host_in, host_out, barrier, max_over_ranks):
    """INT8 YOLO26n on the same images: device calibration (FP32 forwards
    with statistics over 32 seeded U[0,1) images), then the batch of this
    rank timed device-resident (CUDA events) and end to end through
    yb_cuda_forward (pinned host buffers, wall clock), and batch-1 latency.
    Every rank runs the same steps; times are the max over ranks."""
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    L = yb.lib()
    B, H = args.batch, args.hw
    calib = yw.make_batch(range(10000, 10000 + INT8_CALIB_IMAGES), H, H)
    t0 = time.perf_counter()
    scales = model.calibrate_int8(calib, apply=True)
    calib_s = time.perf_counter() - t0
    del calib
    d_in, d_out = model.plan_io(B, H, H)
    torch.cuda.synchronize()
    yb.check(L.yb_cuda_forward(model.ctx, host_in.data_ptr(), B, H, H, host_out.data_ptr(), 300, None, None, None),
             "yb_cuda_forward")
    torch.cuda.synchronize()
    # Fill the device-resident plan's input once (outside the timed region).
    dev_imgs = host_in.to("cuda")
    model.forward_device(dev_imgs.data_ptr(), d_out, B, H, H, 300, stream.cuda_stream)
    torch.cuda.synchronize()
    del dev_imgs
    for _ in range(args.warmup):
        model.forward_device(d_in, d_out, B, H, H, 300, stream.cuda_stream)
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(bus_id_of(torch.cuda.current_device()) if rank == 0 else None) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            model.forward_device(d_in, d_out, B, H, H, 300, stream.cuda_stream)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = clk.summary() if rank == 0 else None
    # End to end (pipelined 16-image sub-batches, pinned host buffers).
    for _ in range(max(1, args.warmup // 2)):
        yb.check(L.yb_cuda_forward(model.ctx, host_in.data_ptr(), B, H, H, host_out.data_ptr(), 300, None, None,
                                   None), "yb_cuda_forward")
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        yb.check(L.yb_cuda_forward(model.ctx, host_in.data_ptr(), B, H, H, host_out.data_ptr(), 300, None, None,
                                   None), "yb_cuda_forward")
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    rgb8 = rgb8_frames(rank, B, H)
    e2e8_s = timed_rgb8(L, model, rgb8, host_out, B, H, args, barrier, max_over_ranks)
    es_s = timed_stream(model, host_in, B, H, args, barrier, max_over_ranks)
    es8_s = timed_stream(model, rgb8, B, H, args, barrier, max_over_ranks, rgb8=True)
    # Batch 1 (the single-image INT8 configuration): device-resident latency.
    d1_in, d1_out = model.plan_io(1, H, H)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        model.forward_device(d1_in, d1_out, 1, H, H, 300, stream.cuda_stream)
    ev0.record(stream)
    reps1 = max(args.steps, 20)
    for _ in range(reps1):
        model.forward_device(d1_in, d1_out, 1, H, H, 300, stream.cuda_stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    b1_ms = max_over_ranks(ev0.elapsed_time(ev1)) / reps1
    n_ops = C.c_int()
    yb.check(L.yb_cuda_profile_ops(model.ctx, B, H, H, 300, 0, None, 0, C.byref(n_ops)), "yb_cuda_profile_ops")
    out = None
    if rank == 0:
        stats = (OpStat * n_ops.value)()
        yb.check(L.yb_cuda_profile_ops(model.ctx, B, H, H, 300, 3, stats, n_ops.value, C.byref(n_ops)),
                 "yb_cuda_profile_ops")
        conv = [s for s in stats if s.kind == 0]
        conv_ms = sum(s.ms for s in conv)
        conv_ops = sum(s.flops for s in conv)
        all_ms = sum(s.ms for s in stats)
        per_kind = {}
        for s in stats:
            d = per_kind.setdefault(INT8_KINDS[s.kind], {"launches": 0, "ms": 0.0})
            d["launches"] += 1
            d["ms"] += s.ms
        tops = conv_ops / (conv_ms * 1e-3) / 1e12
        conv_bytes = sum(s.bytes for s in conv)
        hbm = peaks()[0]
        i8_achieved = conv_bytes / (conv_ms * 1e-3) / 1e9
        i8_bytes_img = sum(s.bytes for s in stats) / B
        out = {"metric": "images/sec YOLO26n 640x640 INT8", "value": world * B * args.steps / (dev_ms * 1e-3),
               "unit": UNIT, "ms_per_step": dev_ms / args.steps, "dtype": "int8 (int32 accumulation)",
               "config": {"workload": f"YOLO26n INT8 forward + top-300 decode, {H}x{H}, {B} images per GPU, "
                                      "image-parallel", "images_per_gpu": B, "global_batch": B * world},
               "calibration": {"images": INT8_CALIB_IMAGES, "source": "device (FP32 forwards with statistics), "
                               "seeded U[0,1) images", "scales": len(scales), "seconds": round(calib_s, 3)},
               "e2e": {"value": world * B * args.steps / es_s, "unit": UNIT,
                       "h2d_bytes_per_step": world * host_in.numel() * 4,
                       "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": STREAM_NOTE},
               "e2e_sync": {"value": world * B * args.steps / e2e_s, "unit": UNIT,
                            "h2d_bytes_per_step": world * host_in.numel() * 4,
                            "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": SYNC_NOTE},
               "e2e_rgb8": {"value": world * B * args.steps / es8_s, "unit": UNIT,
                            "h2d_bytes_per_step": world * rgb8.numel(),
                            "d2h_bytes_per_step": world * host_out.numel() * 4, "mode": STREAM_NOTE,
                            "sync_value": world * B * args.steps / e2e8_s},
               "batch1": {"ms_per_image": b1_ms, "images_per_s": world / (b1_ms * 1e-3),
                          "note": "device-resident single-image forward, one per GPU"},
               "clocks": clocks,
               "gpu_launches": n_ops.value * args.steps,
               "roofline": {"bound": "hbm", "achieved": i8_achieved, "peak": hbm, "unit": "GB/s",
                            "frac": i8_achieved / hbm, "traffic": None, "peak_source": peaks()[2],
                            "kernel": "conv_i8_kernel (all tcgen05 kind::i8 convolution launches of one forward)",
                            "launches": len(conv), "bytes_per_launch": conv_bytes / len(conv),
                            "ms_per_launch": conv_ms / len(conv),
                            "note": "algorithmic int8 bytes (input, output and weights once per launch) over "
                                    "CUDA-event launch times"},
               "forward_roofline": {"bytes_per_image": i8_bytes_img,
                                    "achieved_gbs": world * B * args.steps / (dev_ms * 1e-3) * i8_bytes_img / 1e9,
                                    "frac": world * B * args.steps / (dev_ms * 1e-3) * i8_bytes_img / 1e9 / hbm,
                                    "note": "whole INT8 forward: algorithmic bytes of every launch per image x "
                                            "images/s, against the measured HBM copy bandwidth"},
               "conv_tops": {"achieved": tops, "peak_nominal": INT8_PEAK_TOPS_NOMINAL,
                             "frac_of_nominal": tops / INT8_PEAK_TOPS_NOMINAL,
                             "note": "algorithmic int8 ops (2 x MACs) of the conv_i8 launches"},
               "forward_breakdown_ms": {k: round(v["ms"], 4) for k, v in per_kind.items()},
               "forward_share": {k: round(v["ms"] / all_ms, 4) for k, v in per_kind.items()}}
    model.set_int8(None)
    return out


# The isolated conv shapes of the benchmark's conv-GEMM sweep: (ci, co, k, stride, H = W).
INT8_SWEEP = [(3, 16, 3, 2, 640), (16, 32, 3, 2, 320), (64, 64, 1, 1, 160), (128, 128, 3, 1, 40), (256, 256, 3, 1, 20)]
INT8_PEAK_TOPS_NOMINAL = 4500.0  # dense int8 tensor throughput of one B200 (datasheet; not measured on this pool)


def int8_conv_sweep(hbm_gbs, batch=16, reps=30):
    """Device-resident timing of the INT8 convolution (yb_int8_conv_run) on
    the sweep shapes, 16 images per launch, CUDA events on a dedicated stream
    over `reps` launches after 5 warm-up launches.  ops = 2 x MACs of the
    real channels; bytes = int8 input + output + weights once."""
    import numpy as np
    import torch

    import yolo_b200 as yb

    L = yb.lib()
    stream = torch.cuda.Stream()
    rows = []
    tot_ops = tot_ms = 0.0
    for ci, co, k, stride, hw in INT8_SWEEP:
        rng = np.random.default_rng(ci * 1000 + co)
        w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
        b = (rng.standard_normal(co) * 0.1).astype(np.float32)
        wq = np.zeros((co, ci, k, k), np.int8)
        bq, mult, shift = (np.zeros(co, np.int32) for _ in range(3))
        lut = np.zeros(256, np.int8)
        yb.check(L.yb_int8_quantize_conv(w.ctypes.data, b.ctypes.data, co, ci, k, k, 0.02, 0.05, 0.05, 1,
                                         wq.ctypes.data, bq.ctypes.data, mult.ctypes.data, shift.ctypes.data,
                                         lut.ctypes.data), "yb_int8_quantize_conv")
        h = C.c_void_p()
        pad = (k - 1) // 2
        yb.check(L.yb_int8_conv_create(torch.cuda.current_device(), wq.ctypes.data, bq.ctypes.data,
                                       mult.ctypes.data, shift.ctypes.data, lut.ctypes.data, co, ci, k, k, stride,
                                       pad, C.byref(h)), "yb_int8_conv_create")
        cp = L.yb_int8_conv_ci_pad(h)
        x = torch.zeros((batch, hw, hw, cp), dtype=torch.int8, device="cuda")
        x[..., :ci] = torch.randint(-127, 128, (batch, hw, hw, ci), dtype=torch.int8, device="cuda")
        ho = (hw + 2 * pad - k) // stride + 1
        y = torch.empty((batch, ho, ho, co), dtype=torch.int8, device="cuda")
        torch.cuda.synchronize()
        run = lambda: yb.check(L.yb_int8_conv_run(h, x.data_ptr(), batch, hw, hw, y.data_ptr(),  # noqa: E731
                                                  C.c_void_p(stream.cuda_stream)), "yb_int8_conv_run")
        for _ in range(5):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        yb.check(L.yb_int8_conv_check(h), "yb_int8_conv_check")
        L.yb_int8_conv_destroy(h)
        ops = 2.0 * batch * ho * ho * co * ci * k * k
        nbytes = batch * hw * hw * ci + batch * ho * ho * co + co * ci * k * k
        tot_ops += ops
        tot_ms += ms
        rows.append({"shape": f"{ci}->{co} {k}x{k} s{stride} @{hw}x{hw}", "ms": round(ms, 5),
                     "tops": round(ops / (ms * 1e-3) / 1e12, 2), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                     "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm_gbs, 3)})
    tops = tot_ops / (tot_ms * 1e-3) / 1e12
    return {"images_per_launch": batch, "shapes": rows, "tops_all_shapes": round(tops, 2),
            "peak_tops": INT8_PEAK_TOPS_NOMINAL, "frac": round(tops / INT8_PEAK_TOPS_NOMINAL, 4),
            "peak_source": "nominal dense int8 (datasheet), not measured",
            "note": "bit-exact against the CPU INT8 oracle (tests/test_gpu_int8.py); small maps fit in L2"}


FP32_SWEEP = INT8_SWEEP  # the same five shapes, FP32 (split-bf16 tcgen05 products, fp32 accumulation)


def fp32_conv_sweep(hbm_gbs, bf16_tflops, src, batch=16, reps=30):
    """Device-resident timing of the FP32 convolution (yb_conv_run: conv +
    bias + SiLU with the model graph's kernel and operand mode for the shape)
    on the sweep shapes, `batch` images per launch, CUDA events on a dedicated
    stream over `reps` launches after 5 warm-up launches.  FLOPs = 2 x MACs;
    bytes = fp32 input + output + weights once (4 bytes per element)."""
    import numpy as np
    import torch

    import yolo_b200 as yb

    L = yb.lib()
    stream = torch.cuda.Stream()
    rows = []
    tot_flops = tot_bytes = tot_ms = 0.0
    for ci, co, k, stride, hw in FP32_SWEEP:
        rng = np.random.default_rng(ci * 1000 + co)
        w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
        b = (rng.standard_normal(co) * 0.1).astype(np.float32)
        pad = (k - 1) // 2
        h = C.c_void_p()
        yb.check(L.yb_conv_create(torch.cuda.current_device(), w.ctypes.data, b.ctypes.data, co, ci, k, k, stride,
                                  pad, 1, C.byref(h)), "yb_conv_create")
        cp = L.yb_conv_ci_pad(h)
        ho = (hw + 2 * pad - k) // stride + 1
        cop = (co + 7) // 8 * 8
        if cp == 0:
            x = torch.randn((batch, ci, hw, hw), device="cuda")
        else:
            x = torch.zeros((2, batch, hw, hw, cp), dtype=torch.bfloat16, device="cuda")
            v = torch.randn((batch, hw, hw, ci), device="cuda")
            x[0, ..., :ci] = v.to(torch.bfloat16)
            x[1, ..., :ci] = (v - x[0, ..., :ci].float()).to(torch.bfloat16)
        y = torch.empty((2, batch, ho, ho, cop), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        run = lambda: yb.check(L.yb_conv_run(h, x.data_ptr(), batch, hw, hw, y.data_ptr(),  # noqa: E731
                                             C.c_void_p(stream.cuda_stream)), "yb_conv_run")
        for _ in range(5):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        yb.check(L.yb_conv_destroy(h), "yb_conv_destroy")
        flops = 2.0 * batch * ho * ho * co * ci * k * k
        nbytes = 4.0 * (batch * hw * hw * ci + batch * ho * ho * co + co * ci * k * k)
        tot_flops += flops
        tot_bytes += nbytes
        tot_ms += ms
        gbs = nbytes / (ms * 1e-3) / 1e9
        tf = flops / (ms * 1e-3) / 1e12
        rows.append({"shape": f"{ci}->{co} {k}x{k} s{stride} @{hw}x{hw}", "ms": round(ms, 5),
                     "tflops": round(tf, 2), "tflops_frac": round(tf / bf16_tflops, 4), "gbs": round(gbs, 1),
                     "hbm_frac": round(gbs / hbm_gbs, 3),
                     "kernel": "stem_kernel (NCHW fp32 input)" if cp == 0 else "conv_tc_kernel"})
    return {"images_per_launch": batch, "shapes": rows,
            "tflops_all_shapes": round(tot_flops / (tot_ms * 1e-3) / 1e12, 2),
            "gbs_all_shapes": round(tot_bytes / (tot_ms * 1e-3) / 1e9, 1),
            "peak_tflops": bf16_tflops, "peak_gbs": hbm_gbs, "peak_source": src,
            "note": "FP32 activations as split bf16 pairs, 3 tcgen05 bf16 products per MAC (the tensor pipe "
                    "executes 3x the algorithmic FLOPs); parity: tests/test_gpu_conv_handle.py"}


def strong_leg(model, args, world, rank, local, barrier, max_over_ranks, gather_group):
    """The batch-64 benchmark as a fixed global batch: 64 images (seeds 1..64)
    split 64/N per GPU.  Device-resident time (CUDA events, max over ranks)
    and end to end: each step streams the rank's pinned fp32 input to its GPU
    (two batches in flight), copies the detections back and gathers every
    rank's detections into rank 0's host memory."""
    import torch

    import yb_weights as yw

    G, H = args.global_batch, args.hw
    per = G // world
    imgs = yw.make_batch(range(rank * per + 1, rank * per + per + 1), H, H)
    host_in = torch.from_numpy(imgs).pin_memory()
    d_in, d_out = model.plan_io(per, H, H)
    stream = torch.cuda.Stream()
    dev = host_in.to(f"cuda:{local}")
    torch.cuda.synchronize()
    model.forward_device(dev.data_ptr(), d_out, per, H, H, 300, stream.cuda_stream)
    torch.cuda.synchronize()
    del dev
    for _ in range(args.warmup):
        model.forward_device(d_in, d_out, per, H, H, 300, stream.cuda_stream)
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        model.forward_device(d_in, d_out, per, H, H, 300, stream.cuda_stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    outs = [torch.empty((per, 300, 6), dtype=torch.float32).pin_memory() for _ in range(2)]
    gathered = [torch.empty((per, 300, 6), dtype=torch.float32) for _ in range(world)] if rank == 0 else None

    def gather(t):
        if world == 1:
            gathered[0].copy_(t)
        else:
            import torch.distributed as dist

            dist.gather(t, gathered, dst=0, group=gather_group)

    def run(k):
        pending = []
        for i in range(k):
            if len(pending) == 2:
                t, o = pending.pop(0)
                model.wait(t)
                gather(o)
            o = outs[i % 2]
            pending.append((model.submit(host_in.data_ptr(), per, H, H, o.data_ptr()), o))
        for t, o in pending:
            model.wait(t)
            gather(o)

    run(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    run(args.steps)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    return {"metric": "images/sec YOLO26n 640x640 FP32, global batch 64 split across the GPUs",
            "value": G * args.steps / (dev_ms * 1e-3), "unit": UNIT, "ms_per_step": dev_ms / args.steps,
            "scaling": "strong", "images_per_gpu": per, "global_batch": G,
            "e2e": {"value": G * args.steps / e2e_s, "unit": UNIT,
                    "h2d_bytes_per_step": G * 3 * H * H * 4, "d2h_bytes_per_step": G * 300 * 6 * 4,
                    "mode": "streaming submit/wait (two batches in flight) of each rank's pinned fp32 shard, "
                            "detections copied back and gathered into rank 0's host memory every step"}}


CONFIG5_GLOBAL = 16
CONFIG5_HW = 1280
CONFIG5_CALIB = 4


def config5_leg(args, world, rank, local, tmpdir, barrier, max_over_ranks):
    """The s-width (channels x2) YOLO26 INT8 forward at 1280x1280, global
    batch 16 split 16/N per GPU: C2PSA attention over 1600 tokens in 4 heads
    of 64 channels, 33,600 anchors into the top-300 decode.  Weights: seeded
    random init (seed 0); INT8 scales from a device calibration over 4 seeded
    U[0,1) 1280x1280 images.  Device-resident time (CUDA events, max over
    ranks), end to end through the streaming API, and the conv_i8 roofline."""
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    L = yb.lib()
    G, H = CONFIG5_GLOBAL, CONFIG5_HW
    per = max(1, G // world)
    w = os.path.join(tmpdir, "yolo26s_seed0.bin")
    yw.write_bin(w, yw.random_state("s", 0))
    m = yb.Model(w, device=local)
    try:
        t0 = time.perf_counter()
        scales = m.calibrate_int8(yw.make_batch(range(30000, 30000 + CONFIG5_CALIB), H, H), apply=True)
        calib_s = time.perf_counter() - t0
        imgs = yw.make_batch(range(40000 + rank * per, 40000 + rank * per + per), H, H)
        host_in = torch.from_numpy(imgs).pin_memory()
        d_in, d_out = m.plan_io(per, H, H)
        stream = torch.cuda.Stream()
        dev = host_in.to(f"cuda:{local}")
        torch.cuda.synchronize()
        m.forward_device(dev.data_ptr(), d_out, per, H, H, 300, stream.cuda_stream)
        torch.cuda.synchronize()
        del dev
        for _ in range(args.warmup):
            m.forward_device(d_in, d_out, per, H, H, 300, stream.cuda_stream)
        torch.cuda.synchronize()
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(bus_id_of(local) if rank == 0 else None) as clk:
            ev0.record(stream)
            for _ in range(args.steps):
                m.forward_device(d_in, d_out, per, H, H, 300, stream.cuda_stream)
            ev1.record(stream)
            torch.cuda.synchronize()
        barrier()
        dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
        clocks = clk.summary() if rank == 0 else None
        es_s = timed_stream(m, host_in, per, H, args, barrier, max_over_ranks)
        n_ops = C.c_int()
        yb.check(L.yb_cuda_profile_ops(m.ctx, per, H, H, 300, 0, None, 0, C.byref(n_ops)), "yb_cuda_profile_ops")
        out = None
        if rank == 0:
            stats = (OpStat * n_ops.value)()
            yb.check(L.yb_cuda_profile_ops(m.ctx, per, H, H, 300, 3, stats, n_ops.value, C.byref(n_ops)),
                     "yb_cuda_profile_ops")
            conv = [s for s in stats if s.kind == 0]
            conv_ms = sum(s.ms for s in conv)
            conv_bytes = sum(s.bytes for s in conv)
            conv_ops = sum(s.flops for s in conv)
            per_kind = {}
            for s in stats:
                d = per_kind.setdefault(INT8_KINDS[s.kind], {"launches": 0, "ms": 0.0})
                d["launches"] += 1
                d["ms"] += s.ms
            hbm = peaks()[0]
            ach = conv_bytes / (conv_ms * 1e-3) / 1e9
            out = {"metric": "images/sec YOLO26s-width INT8 1280x1280, global batch 16 split across the GPUs",
                   "value": G * args.steps / (dev_ms * 1e-3) if world <= G else None, "unit": UNIT,
                   "ms_per_step": dev_ms / args.steps, "scaling": "strong", "images_per_gpu": per,
                   "global_batch": per * world, "dtype": "int8 (int32 accumulation)",
                   "calibration": {"images": CONFIG5_CALIB, "hw": H, "seconds": round(calib_s, 3),
                                   "scales": len(scales), "source": "device (FP32 forwards with statistics)"},
                   "e2e": {"value": per * world * args.steps / es_s, "unit": UNIT,
                           "h2d_bytes_per_step": per * world * 3 * H * H * 4,
                           "d2h_bytes_per_step": per * world * 300 * 6 * 4, "mode": STREAM_NOTE},
                   "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                "kernel": "conv_i8_kernel", "launches": len(conv),
                                "bytes_per_launch": conv_bytes / len(conv), "ms_per_launch": conv_ms / len(conv)},
                   "conv_tops": conv_ops / (conv_ms * 1e-3) / 1e12,
                   "forward_breakdown_ms": {k: round(v["ms"], 4) for k, v in per_kind.items()},
                   "gpu_launches": n_ops.value * args.steps, "clocks": clocks,
                   "parity": "tests/test_gpu_configs.py (s-width INT8 1280x1280, batch 2, bit-exact)"}
    finally:
        m.close()
    return out


class OpStat(C.Structure):
    _fields_ = [("kind", C.c_int), ("step", C.c_int), ("ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--hw", type=int, default=640)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-int8-sweep", action="store_true")
    ap.add_argument("--no-int8", action="store_true", help="skip the INT8 model leg")
    ap.add_argument("--global-batch", type=int, default=64, help="global batch of the strong-scaling leg")
    ap.add_argument("--no-strong", action="store_true", help="skip the global-batch-64 (strong scaling) leg")
    ap.add_argument("--no-config5", action="store_true", help="skip the s-width INT8 1280x1280 leg")
    ap.add_argument("--no-fp32-sweep", action="store_true", help="skip the FP32 convolution sweep")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
