#!/usr/bin/env python
"""Benchmark of the triangle pair stack (headline metric: pair-stack layers*N^2/s at N=1024).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configuration 5): B=1, N=1024, c_z=128, 8 layers of
[TriMulOut, TriMulIn, TriAttStart, TriAttEnd] with residual adds, all-ones mask, synthetic
z ~ N(0,1) and weights ~ N(0, 1/fan_in) (gate biases 1). One step = one full 8-layer
stack forward. The pair tensor (512 MB fp32) is larger than the 126 MB L2, so no flush is
needed between steps. The stack runs as one CUDA graph of 96 kernel launches; CUDA events
recorded between the kernels (captured into the graph) give each kernel's device time.

* ``value``: layers*N^2/s over all ranks with inputs resident in HBM (device timing, CUDA
  events, max over ranks).
* ``e2e``: the same metric through the public API with host buffers: every step copies z
  from pinned host memory, runs the stack and copies the full result back. On one GPU the
  copies run on their own streams, so the input copy of step s+1 and the result copy of
  step s overlap the compute of step s (two device buffer pairs); the one-stream serial
  figure is reported alongside (``e2e.serial``).
* ``roofline``: the dominant kernel against MEASURED_PEAKS.json.
* ``cpu_baseline``: the reference math (the fp32 PyTorch oracle) on this host's cores, on
  a row sample of one N=1024 layer (rank 0 at N=1 only).

``--impl reference`` times that CPU implementation alone (rank 0). Each step is one row
sample of one N=1024 layer (a quarter of the output rows by default); ``ms_per_step`` is the
wall time the step took, and ``value`` is the full-layer throughput estimated from the sample
(labelled as such in the line).

With --gpus N > 1 (torchrun, one process per GPU) the same N=1024 problem is row-sharded
over the ranks (``genie_tk.sharded``). By default the exchanges (the gathered or
channel-sharded planes of the multiplicative update, the triangle bias, the ending node's
pair transposes, which the attention blocks' K4e stores directly when a rank's rows are a
multiple of 128) are push kernels that store straight into the peers' buffers over NVLink,
with NCCL used only for set-up (``--exchange nccl`` runs them as NCCL collectives). The
scaling is strong: ``value`` is the one problem's layers*N^2/s, timed on each rank's stream
with CUDA events and reduced with MAX over ranks. After the timed region the ranks' output
shards are gathered on rank 0 and compared with a one-GPU run of the same stack on the same
input (``parity`` in the line).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import statistics
import subprocess
import sys
import tempfile

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "genie-tk_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "pair-stack layers*N^2/sec at N=1024, c_z=128"
UNIT = "layers*N^2/s"

# algorithmic work per launch (B=1): FLOPs for tensor-bound kernels, bytes for HBM-bound ones
def kernel_work(name: str, N: int, B: int = 1):
    P = B * N * N
    if name == "triatt_core":
        return "tensor", 4.0 * B * N ** 3 * 4 * 32          # QK^T + PV, H=4, d=32
    if name in ("trimul_contract", "trimul_contract_to"):
        return "tensor", 2.0 * B * N ** 3 * 128             # 128 channel GEMMs of N^3
    if name in ("trimul_project", "trimul_project_to"):
        return "hbm", P * (512 + 4 + 2 * 128 * 2)           # z fp32 + mask in, a, b fp16 out
    if name == "trimul_finish":
        return "hbm", P * (128 * 2 + 512 + 512)             # x fp16 + z fp32 in, z fp32 out
    if name == "triatt_project":
        return "hbm", P * (512 + 4 * 128 * 2 + 4 * 2)       # z in; q, k, v, g fp16 + bias out
    if name in ("triatt_finish", "triatt_finish_to"):
        return "hbm", P * (128 * 2 + 512 + 512)             # og fp16 + z in, z out
    raise KeyError(name)


def layer_flops(N: int) -> float:
    return 1536.0 * N + 722944.0  # per pair; see oracle.triangle_oracle.flops_per_pair("layer")


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clocks and throttle reasons of this process's GPU while the timed region runs.

    NVML (read-only queries) is polled every 20 ms from a thread, so even a timed region of
    a tenth of a second (8 GPUs x 10 steps) gets samples; without NVML, nvidia-smi samples at
    200 ms. The GPU is found by its UUID (then PCI bus id, then index), so a job that was
    given a subset of a node's GPUs samples its own."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event (throttle) reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, device=None):
        self.device = torch.device("cuda", 0) if device is None else torch.device(device)
        self.proc = None
        self.path = None
        self.thread = None
        self.samples = []  # (sm MHz, max sm MHz, reason bits)

    def _nvml_handle(self, nv):
        props = torch.cuda.get_device_properties(self.device)
        tries = []
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            tries.append(lambda: nv.nvmlDeviceGetHandleByUUID("GPU-" + str(uuid)))
        if hasattr(props, "pci_bus_id"):
            bus = f"{getattr(props, 'pci_domain_id', 0):08x}:{props.pci_bus_id:02x}:{getattr(props, 'pci_device_id', 0):02x}.0"
            tries.append(lambda: nv.nvmlDeviceGetHandleByPciBusId(bus))
        tries.append(lambda: nv.nvmlDeviceGetHandleByIndex(self.device.index or 0))
        for t in tries:
            try:
                return t()
            except Exception:
                continue
        return None

    def start(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._nvml_handle(nv)
            if h is None:
                raise RuntimeError("no NVML handle")
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.stop_flag = threading.Event()

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx, int(reasons(h))))
                    except Exception:
                        pass
                    self.stop_flag.wait(0.02)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        exe = shutil.which("nvidia-smi")
        if not exe:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.f = open(self.path, "w")
        self.proc = subprocess.Popen([exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)

    def stop(self):
        """This GPU's samples: a list of (sm MHz, max sm MHz, reason bits)."""
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            return list(self.samples)
        if not self.proc:
            return []
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        out = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) != (self.device.index or 0):
                    continue
                try:
                    sm, mxc = float(parts[1]), float(parts[2])
                except ValueError:
                    continue
                bits = 0
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        bits |= self.REASON_BITS[n]
                out.append((sm, mxc, bits))
        os.unlink(self.path)
        return out

    @classmethod
    def summary(cls, samples):
        """Median SM clock, max clock and the reasons seen, over samples of one or more GPUs."""
        if not samples:
            return None
        reasons = sorted(n for n, bit in cls.REASON_BITS.items() if any(s[2] & bit for s in samples))
        return {"sm_mhz": statistics.median(s[0] for s in samples), "sm_max_mhz": max(s[1] for s in samples),
                "reasons": reasons, "samples": len(samples)}


def make_stack(n_layers: int, device, seed: int = 1005):
    """Random-init weights of the cfg5 architecture: N(0, 1/fan_in), gate biases 1."""
    import genie_tk
    stack = genie_tk.TrianglePairStack(n_layers).to(device)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for name, p in stack.named_parameters():
            kind = name.split(".")[-1]
            if kind == "weight" and p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=gen) / math.sqrt(p.shape[1]))
            elif kind == "weight":
                p.fill_(1.0)       # LayerNorm gamma
            elif name.endswith("linear_a_g.bias") or name.endswith("linear_b_g.bias") or \
                    name.endswith("linear_g.bias"):
                p.fill_(1.0)       # gate biases
            else:
                p.zero_()
    return stack


def cpu_sample(N: int, rows: int, threads: int):
    """One N x N layer of the reference math on the host cores, from a row sample."""
    from oracle import triangle_oracle as O
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(4)
    z = torch.randn(1, N, N, 128, generator=gen)
    mask = torch.ones(1, N, N)
    pg = torch.Generator().manual_seed(1005)
    lp = {"tri_mul_out": O.make_trimul_params(128, 128, pg, gate_bias=1.0),
          "tri_mul_in": O.make_trimul_params(128, 128, pg, gate_bias=1.0),
          "tri_att_start": O.make_triatt_params(128, 128, 4, pg, gate_bias=1.0),
          "tri_att_end": O.make_triatt_params(128, 128, 4, pg, gate_bias=1.0)}
    return lambda: O.time_layer_sample(z, mask, lp, 4, rows)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank):
    """The reference arm: the reference's fp32 PyTorch math (oracle port) on all host cores.

    Each step times one row sample of one N x N layer: the row-independent parts of the four
    ops over all pairs, then ``--cpu-rows`` output rows of each op. ``ms_per_step`` is the
    measured wall time of a step. ``value`` is the estimated full-layer throughput: the
    per-row part scales linearly with the rows, so a layer takes sum(t_prepare + t_rows * N /
    rows); it is labelled a row-sample estimate (``value_kind``)."""
    import time
    if rank != 0:
        return None
    N = args.N
    threads = os.cpu_count() or 1
    fn = cpu_sample(N, args.cpu_rows, threads)
    for _ in range(args.warmup):
        fn()
    ests, walls = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        est, parts, tot = fn()
        walls.append(time.perf_counter() - t0)
        ests.append(est)
    layer_s = statistics.mean(ests)
    value = N * N / layer_s
    frac = min(1.0, args.cpu_rows / N)
    sample = (f"one {N}x{N} layer (4 ops) of the reference fp32 PyTorch math per step: row-independent parts "
              f"over all pairs plus {args.cpu_rows} of {N} output rows per op ({frac:.0%} of the rows); the "
              f"per-row part is scaled to {N} rows for the value")
    ms_step = statistics.mean(walls) * 1e3
    return {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "value_kind": f"row-sample estimate: {args.cpu_rows} of {N} rows timed per step, scaled to a full "
                          f"layer",
            "estimated_full_layer_ms": layer_s * 1e3,
            "estimated_full_stack_ms": layer_s * 1e3 * args.layers,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"cfg5 triangle pair stack, B=1 N={N} c_z=128, "
                                                        f"{args.layers} layers (CPU row sample of one layer)",
                                            "global_batch": 1, "seq_len": N, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                             "cpu": cpu_model(), "measured_s": round(sum(walls), 2)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_e2e(args, stack, mask, z_host, z_ref, device, world, B, L, N):
    """End-to-end steps through the public API (``TrianglePairStack.forward_into``) with host
    buffers. Every step copies its input z from pinned host memory to the device and its
    result back to pinned host memory, inside the timed region.

    Pipelined (the figure reported): two device input/output buffer pairs, one CUDA graph per
    pair; the host->device copy of step s+1 and the device->host copy of step s run on their
    own streams while step s computes (PCIe is full duplex), ordered by events so that no
    copy touches a buffer a step is still using. Serial (reported alongside): copy in, run,
    copy out on one stream, one step at a time."""
    cur = torch.cuda.current_stream(device)
    zin = [torch.empty_like(z_ref), torch.empty_like(z_ref)]
    zout = [torch.empty_like(z_ref), torch.empty_like(z_ref)]
    out_host = [torch.empty_like(z_host).pin_memory(), torch.empty_like(z_host).pin_memory()]
    graphs = []
    for b in range(2):
        zin[b].copy_(z_host)
        stack.forward_into(zin[b], zout[b], mask)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(device=device)
        cs.wait_stream(cur)
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                stack.forward_into(zin[b], zout[b], mask)
        cur.wait_stream(cs)
        graphs.append(g)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def timed(fn):
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        fn()
        e1.record(cur)
        torch.cuda.synchronize()
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms / args.steps

    def serial():
        for _ in range(args.steps):
            zin[0].copy_(z_host, non_blocking=True)
            graphs[0].replay()
            out_host[0].copy_(zout[0], non_blocking=True)

    h2d = torch.cuda.Stream(device=device)
    d2h = torch.cuda.Stream(device=device)

    def pipelined():
        K = args.steps
        in_ready = [torch.cuda.Event(), torch.cuda.Event()]
        step_done = [torch.cuda.Event(), torch.cuda.Event()]
        out_read = [torch.cuda.Event(), torch.cuda.Event()]
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        with torch.cuda.stream(h2d):
            zin[0].copy_(z_host, non_blocking=True)
            in_ready[0].record(h2d)
        for s in range(K):
            b = s & 1
            if s + 1 < K:
                nb = b ^ 1
                with torch.cuda.stream(h2d):
                    if s >= 1:
                        h2d.wait_event(step_done[nb])  # step s-1 has finished reading zin[nb]
                    zin[nb].copy_(z_host, non_blocking=True)
                    in_ready[nb].record(h2d)
            cur.wait_event(in_ready[b])
            if s >= 2:
                cur.wait_event(out_read[b])  # step s-2's result has left zout[b]
            graphs[b].replay()
            step_done[b].record(cur)
            with torch.cuda.stream(d2h):
                d2h.wait_event(step_done[b])
                out_host[b].copy_(zout[b], non_blocking=True)
                out_read[b].record(d2h)
        cur.wait_stream(d2h)
        cur.wait_stream(h2d)

    serial()  # warm-up
    ms_serial = timed(serial)
    h2d_bytes = z_host.numel() * 4
    serial_line = {"value": world * B * L * N * N / (ms_serial / 1e3), "ms_per_step": ms_serial}
    try:
        pipelined()  # warm-up of both graphs and streams
        ms = timed(pipelined)
        # the last step's result must equal the resident-input run's result
        last = out_host[(args.steps - 1) & 1]
        if not torch.equal(last[:, : min(N, 64)], z_ref[:, : min(N, 64)].cpu()):
            raise RuntimeError("pipelined result differs from the device-resident run")
    except RuntimeError as exc:  # report the serial figure rather than none
        return {"value": serial_line["value"], "unit": UNIT, "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": h2d_bytes, "ms_per_step": ms_serial, "mode": "serial",
                "pipelined_error": str(exc)[:200]}
    return {"value": world * B * L * N * N / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": h2d_bytes, "ms_per_step": ms,
            "mode": "pipelined: H2D of step s+1 and D2H of step s on their own streams, overlapping step s",
            "serial": serial_line}

def run_ours(args, rank, world, device):
    import genie_tk
    from genie_tk import ops, stack as stack_mod
    N, L, B = args.N, args.layers, 1
    torch.manual_seed(4)
    gen = torch.Generator(device="cpu").manual_seed(4)
    z_host = torch.randn(B, N, N, 128, generator=gen).pin_memory()
    mask = torch.ones(B, N, N, device=device)
    z0 = z_host.to(device)
    z = torch.empty_like(z0)
    stack = make_stack(L, device)
    stack.prepare(B, N, device)

    # capture one stack step into a graph, with an event between every pair of kernels
    labels = []
    events = []

    def hook(label):
        # a kernel runs between the event recorded with its label and the next event
        if label != "end":
            labels.append((label, len(events)))
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events.append(ev)

    stack.forward_into(z0, z, mask)  # tensor maps / attributes cached outside capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            stack._run(z0, z, mask, hook)
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize()
    n_kernels = len(labels)
    assert n_kernels == L * stack_mod.KERNELS_PER_LAYER

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ops.check_status(device)

    sampler = ClockSampler(device)
    sampler.start()
    per_kernel = {}
    timing_mode = "graph-events"
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        graph.replay()
        if timing_mode == "graph-events":
            # harvest this replay's per-kernel times (events are overwritten by the next replay)
            try:
                events[-1].synchronize()
                for lab, e in labels:
                    per_kernel.setdefault(lab, []).append(events[e].elapsed_time(events[e + 1]))
            except RuntimeError:
                timing_mode = "eager-events"
                per_kernel = {}
    t_stop.record()
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = t_start.elapsed_time(t_stop)
    clocks = ClockSampler.summary(sampler.stop())
    if timing_mode == "eager-events":
        for _ in range(args.steps):
            labels.clear()
            events.clear()
            stack._run(z0, z, mask, hook)
            torch.cuda.synchronize()
            for lab, e in labels:
                per_kernel.setdefault(lab, []).append(events[e].elapsed_time(events[e + 1]))
    status = ops.check_status(device)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * B * L * N * N / (ms_per_step / 1e3)

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, stack, mask, z_host, z, device, world, B, L, N)

    peaks = load_peaks()
    kernels = {}
    total_k = sum(sum(v) for v in per_kernel.values())
    for lab, times in per_kernel.items():
        launches = len(times)
        avg = sum(times) / launches
        bound, work = kernel_work(lab, N, B)
        if bound == "tensor":
            ach = work / (avg / 1e3) / 1e12
            peak = peaks["bf16_tflops"]
            unit = "TFLOP/s"
        else:
            ach = work / (avg / 1e3) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        kernels[lab] = {"launches_per_step": launches // args.steps, "avg_ms": round(avg, 4),
                        "share": round(sum(times) / total_k, 4), "bound": bound, "achieved": round(ach, 1),
                        "unit": unit, "frac": round(ach / peak, 4)}
    dom = max(kernels, key=lambda k: kernels[k]["share"])
    dk = kernels[dom]
    traffic, traffic_note = read_traffic(dom)
    roofline = {"kernel": dom, "bound": dk["bound"], "achieved": dk["achieved"],
                "peak": peaks["bf16_tflops"] if dk["bound"] == "tensor" else peaks["hbm_gbs"],
                "unit": dk["unit"], "frac": dk["frac"], "traffic": traffic, "traffic_source": traffic_note,
                "peak_source": peaks["source"] + " (MEASURED_PEAKS.json burst)" if peaks["source"] == "measured"
                else "fallback"}
    stack_tflops = B * N * N * L * layer_flops(N) / (ms_per_step / 1e3) / 1e12 * world
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 tensor-core operands, f32 accumulate / f32 residual stream",
            "data": "synthetic (z ~ N(0,1), weights ~ N(0,1/fan_in), all-ones mask)",
            "config": {"workload": f"cfg5 triangle pair stack: B={B}, N={N}, c_z=128, c=128, H=4, d=32, "
                                   f"{L} layers x [TriMulOut, TriMulIn, TriAttStart, TriAttEnd]",
                       "global_batch": B * world, "seq_len": N, "layers": L,
                       "parallelism": "replicas" if world > 1 else "single-gpu",
                       "l2": "inputs larger than L2 (z is 512 MB fp32); no flush"},
            "stack_tflops": round(stack_tflops, 1),
            "stack_frac_of_bf16_peak": round(stack_tflops / peaks["bf16_tflops"] / world, 4),
            "e2e": e2e, "gpu_launches": n_kernels * args.steps, "roofline": roofline, "kernels": kernels,
            "kernel_timing": timing_mode,
            "clocks": clocks, "status_word": status}
    return line


def run_sharded(args, rank, world, device):
    """The row-sharded stack over ``world`` ranks (strong scaling of one N x N problem)."""
    from genie_tk import ops
    from genie_tk.sharded import CudaStageOps, ShardedTrianglePairStack, TimedStageOps
    import torch.distributed as dist
    N, L, B = args.N, args.layers, 1
    gen = torch.Generator(device="cpu").manual_seed(4)
    z_full = torch.randn(B, N, N, 128, generator=gen)
    R = N // world
    z_host = z_full[:, rank * R:(rank + 1) * R].clone().pin_memory()
    del z_full
    mask = torch.ones(B, N, N, device=device)
    z0 = z_host.to(device)
    z = torch.empty_like(z0)
    stack = make_stack(L, device)
    so = TimedStageOps(CudaStageOps(device, push=args.push))
    shard = ShardedTrianglePairStack(stack, world, rank, stage_ops=so, trimul_exchange=args.trimul_exchange,
                                     exchange=args.exchange, k1_direct=args.k1_direct,
                                     fused_transpose=not args.separate_transpose, fused_x=not args.separate_x)
    if args.exchange == "peer":
        shard.connect(None, B, N, device)
    else:
        shard.prepare(B, N, device)

    def step(zin=None, hook=None, zout=None):
        so.hook = hook
        shard.forward_(z if zout is None else zout, mask, z_in=z0 if zin is None else zin, hook=hook)
        so.hook = None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_status(device)
    so.launches = 0

    sampler = ClockSampler(device)
    sampler.start()
    dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    dist.barrier()
    # every rank samples its own GPU; rank 0 reports all of them together
    per_rank = [None] * world
    dist.all_gather_object(per_rank, sampler.stop())
    clocks = ClockSampler.summary([x for r in per_rank for x in r])
    launches = so.launches
    elapsed = torch.tensor([t0.elapsed_time(t1)], device=device)
    dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    ms_per_step = float(elapsed.item()) / args.steps
    value = B * L * N * N / (ms_per_step / 1e3)

    # one more step with an event around every kernel and collective (not the timed run)
    labels, events = [], []

    def hook(label):
        if label != "end":
            labels.append((label, len(events)))
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events.append(ev)
    step(hook=hook)
    torch.cuda.synchronize()
    per = {}
    for lab, e in labels:
        per[lab] = per.get(lab, 0.0) + events[e].elapsed_time(events[e + 1])
    tot = sum(per.values())
    breakdown = {k: {"ms": round(v, 3), "share": round(v / tot, 4)} for k, v in sorted(per.items(),
                                                                                        key=lambda kv: -kv[1])}
    status = ops.check_status(device)

    e2e = None
    if not args.no_e2e:
        # Each rank copies its own row shard in from pinned host memory and its result out,
        # every step. Pipelined (the figure reported): two input and two output buffers, the
        # H2D of step s+1 and the D2H of step s on their own streams while step s runs; the
        # serial form (copy in, step, copy out on one stream) is reported beside it.
        cur = torch.cuda.current_stream(device)
        h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        out_host = [torch.empty_like(z_host).pin_memory() for _ in range(2)]
        zin, zout = [z0, torch.empty_like(z0)], [z, torch.empty_like(z)]

        def timed(fn):
            torch.cuda.synchronize()
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            fn()
            e1.record(cur)
            torch.cuda.synchronize()
            dist.barrier()
            t = torch.tensor([e0.elapsed_time(e1)], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item()) / args.steps

        def serial():
            for _ in range(args.steps):
                z0.copy_(z_host, non_blocking=True)
                step()
                out_host[0].copy_(z, non_blocking=True)

        def pipelined():
            K = args.steps
            in_ready = [torch.cuda.Event(), torch.cuda.Event()]
            step_done = [torch.cuda.Event(), torch.cuda.Event()]
            out_read = [torch.cuda.Event(), torch.cuda.Event()]
            h2d.wait_stream(cur)
            d2h.wait_stream(cur)
            with torch.cuda.stream(h2d):
                zin[0].copy_(z_host, non_blocking=True)
                in_ready[0].record(h2d)
            for s in range(K):
                b = s & 1
                if s + 1 < K:
                    nb = b ^ 1
                    with torch.cuda.stream(h2d):
                        if s >= 1:
                            h2d.wait_event(step_done[nb])  # step s-1 has finished reading zin[nb]
                        zin[nb].copy_(z_host, non_blocking=True)
                        in_ready[nb].record(h2d)
                cur.wait_event(in_ready[b])
                if s >= 2:
                    cur.wait_event(out_read[b])  # step s-2's result has left zout[b]
                step(zin[b], zout=zout[b])
                step_done[b].record(cur)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(step_done[b])
                    out_host[b].copy_(zout[b], non_blocking=True)
                    out_read[b].record(d2h)
            cur.wait_stream(d2h)
            cur.wait_stream(h2d)

        serial()  # warm-up
        ms_serial = timed(serial)
        serial_out = out_host[0].clone()
        pipelined()  # warm-up of the second buffers and the copy streams
        ms_pipe = timed(pipelined)
        # every step has the same input, so the last pipelined result equals the serial one
        same = torch.equal(out_host[(args.steps - 1) & 1], serial_out)
        bytes_step = z_host.numel() * 4 * world
        serial_line = {"value": B * L * N * N / (ms_serial / 1e3), "ms_per_step": ms_serial}
        e_ms = ms_pipe if same else ms_serial
        e2e = {"value": B * L * N * N / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": bytes_step,
               "d2h_bytes_per_step": bytes_step, "ms_per_step": e_ms,
               "mode": ("pipelined: H2D of step s+1 and D2H of step s on their own streams, overlapping step s"
                        if same else "serial (the pipelined result differed)"),
               "serial": serial_line, "note": "each rank copies its own row shard in and out"}
    parity = sharded_parity(stack, shard_step=step, z_out=z, rank=rank, world=world, device=device,
                            mask=mask, N=N, B=B)
    peaks = load_peaks()
    stack_tflops = B * N * N * L * layer_flops(N) / (ms_per_step / 1e3) / 1e12
    stage_kernels = ("triatt_core", "trimul_contract", "trimul_project", "trimul_project_to", "trimul_finish",
                     "triatt_project", "triatt_finish", "triatt_finish_to", "trimul_contract_to")
    dom = max((k for k in breakdown if k in stage_kernels), key=lambda k: breakdown[k]["ms"])
    bound, work = kernel_work(dom, N, B)
    calls = sum(1 for lab, _ in labels if lab == dom)
    avg_ms = per[dom] / calls
    work /= world  # each rank's launch covers its R = N / P rows
    if bound == "tensor":
        ach, peak, unit = work / (avg_ms / 1e3) / 1e12, peaks["bf16_tflops"], "TFLOP/s"
    else:
        ach, peak, unit = work / (avg_ms / 1e3) / 1e9, peaks["hbm_gbs"], "GB/s"
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 tensor-core operands, f32 accumulate / f32 residual stream",
            "data": "synthetic (z ~ N(0,1), weights ~ N(0,1/fan_in), all-ones mask)",
            "config": {"workload": f"cfg5 triangle pair stack: B={B}, N={N}, c_z=128, c=128, H=4, d=32, "
                                   f"{L} layers x [TriMulOut, TriMulIn, TriAttStart, TriAttEnd]",
                       "global_batch": B, "seq_len": N, "layers": L,
                       "parallelism": f"row-sharded over i, {world} ranks x {R} rows; exchanges: " + (
                           "peer push kernels over NVLink (NCCL for set-up only)" if args.exchange == "peer"
                           else "NCCL collectives"),
                       "trimul_exchange": shard.trimul_exchange, "exchange": args.exchange,
                       "k1_direct": bool(args.k1_direct and args.exchange == "peer" and shard.trimul_exchange == "channels"),
                       "attention_transpose": ("fused into K4e's stores" if args.exchange == "peer" and
                                               not args.separate_transpose and (N // world) % 128 == 0
                                               else "separate push"),
                       "x_scatter": ("fused into K2's stores" if args.exchange == "peer" and not args.separate_x and
                                     shard.trimul_exchange == "channels" and (N // world) % 128 == 0
                                     else "separate push"),
                       "push": args.push,
                       "l2": "inputs larger than L2 (each shard is >= 64 MB fp32); no flush"},
            "stack_tflops": round(stack_tflops, 1),
            "stack_frac_of_bf16_peak": round(stack_tflops / peaks["bf16_tflops"] / world, 4),
            "e2e": e2e, "gpu_launches": launches, "roofline": {
                "kernel": dom, "bound": bound, "achieved": round(ach, 1), "peak": peak, "unit": unit,
                "frac": round(ach / peak, 4), "traffic": None, "peak_source": peaks["source"],
                "note": "rank 0's eager per-kernel timing of one extra step"},
            "breakdown_rank0": breakdown, "parity": parity, "clocks": clocks, "status_word": status}
    shard.close()
    return line


def sharded_parity(stack, shard_step, z_out, rank, world, device, mask, N, B):
    """Correctness of the row-sharded run: one more sharded step (every rank), its output
    shards gathered on every rank, and on rank 0 a one-GPU run of the same stack (same
    weights) on the same full input, compared element by element. The one-GPU stack is the
    path the parity tests check against the fp32 oracle of the reference math."""
    import torch.distributed as dist
    shard_step()
    torch.cuda.synchronize()
    full = torch.empty((world,) + tuple(z_out.shape[1:]), dtype=z_out.dtype, device=device)
    dist.all_gather_into_tensor(full, z_out.contiguous())
    result = None
    if rank == 0:
        gen = torch.Generator(device="cpu").manual_seed(4)
        z_in = torch.randn(B, N, N, 128, generator=gen).to(device)
        ref = torch.empty_like(z_in)
        stack.forward_into(z_in, ref, mask)
        torch.cuda.synchronize()
        got = full.view(B, N, N, 128)
        d = (got - ref).abs()
        mx, mn = float(d.max()), float(d.mean())
        result = {"vs": "one-GPU TrianglePairStack run of the same weights and input on rank 0",
                  "max_abs": mx, "mean_abs": mn, "bitwise_equal": bool(torch.equal(got, ref)),
                  "finite": bool(torch.isfinite(got).all()),
                  "bar": {"max_abs": 2e-2, "mean_abs": 2e-3}, "ok": bool(mx <= 2e-2 and mn <= 2e-3)}
        del z_in, ref, d
    del full
    dist.barrier()
    return result


# CUDA sources each kernel is compiled from (its file and the shared device header)
KERNEL_SOURCES = {
    "triatt_core": ("triatt.cu", "gtk_sm100.cuh"), "triatt_project": ("triatt.cu", "gtk_sm100.cuh"),
    "triatt_finish": ("triatt.cu", "gtk_sm100.cuh"), "trimul_project": ("trimul.cu", "gtk_sm100.cuh"),
    "trimul_contract": ("trimul.cu", "gtk_sm100.cuh"), "trimul_finish": ("trimul.cu", "gtk_sm100.cuh"),
}
TRAFFIC_FILE = os.path.join(REPO, "profiles", "triatt_core_dram_traffic_stack_cfg5_N1024.txt")


def source_sha16(kernel):
    """First 16 hex digits of the SHA-256 of the CUDA sources ``kernel`` is built from."""
    import hashlib
    h = hashlib.sha256()
    for f in KERNEL_SOURCES.get(kernel, ()):
        with open(os.path.join(REPO, "genie-tk_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def read_traffic(kernel):
    """DRAM bytes per launch of ``kernel`` at the bench workload, from the committed ncu
    summary, and a note. The summary records the hash of the sources it was captured from;
    when the kernel's sources have changed since, the figure is stale and not reported."""
    vals, shas = {}, {}
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 3 and parts[0] == "source_sha16":
                    shas[parts[1]] = parts[2]
                elif len(parts) >= 2 and not line.startswith("#"):
                    vals[parts[0]] = float(parts[1])
    except OSError:
        return None, "no ncu capture committed"
    if kernel not in vals:
        return None, "no ncu capture of this kernel committed"
    if shas.get(kernel) != source_sha16(kernel):
        return None, "the committed ncu capture is of older kernel sources; not reported"
    return vals[kernel], "ncu dram__bytes_read.sum + dram__bytes_write.sum, per launch (" + \
        os.path.relpath(TRAFFIC_FILE, REPO) + ")"


def run_transition(args, device):
    """``--op transition``: the pair transition (LN -> 4x expand -> ReLU -> project) with the
    pair transform layer's residual and mask, p = (p + transition(p)) * mask, on one GPU
    (N^2 pairs per step, B = 1, seeded synthetic z and weights). Not the headline metric; it
    measures the pair-transition kernels against their HBM roofline and against the same
    math as unfused fp32 PyTorch ops on the GPU."""
    from genie_tk import ops
    N = args.N
    gen = torch.Generator().manual_seed(5)
    z = torch.randn(1, N, N, 128, generator=gen).to(device)
    mask = torch.ones(1, N, N, device=device)
    # seeded PairTransition parameters: LayerNorm near identity, weights N(0, 1/fan_in),
    # small biases (linear_2 is not the reference's zero init, so the update is not zero)
    p = {"layer_norm.weight": 1.0 + 0.1 * torch.randn(128, generator=gen),
         "layer_norm.bias": 0.1 * torch.randn(128, generator=gen),
         "linear_1.weight": torch.randn(512, 128, generator=gen) / math.sqrt(128),
         "linear_1.bias": 0.1 * torch.randn(512, generator=gen),
         "linear_2.weight": torch.randn(128, 512, generator=gen) / math.sqrt(512),
         "linear_2.bias": 0.1 * torch.randn(128, generator=gen)}
    p = {k: v.to(device) for k, v in p.items()}
    packed = ops.pack_transition(p, device)
    out = torch.empty_like(z)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms = timed(lambda: ops.transition_forward(z, mask, packed, out=out, add_residual=True), args.steps)
    torch.backends.cuda.matmul.allow_tf32 = False
    lw, lb = p["layer_norm.weight"], p["layer_norm.bias"]

    def torch_path():
        h = torch.relu(torch.nn.functional.linear(torch.nn.functional.layer_norm(z, (128,), lw, lb),
                                                  p["linear_1.weight"], p["linear_1.bias"]))
        return (z + torch.nn.functional.linear(h, p["linear_2.weight"], p["linear_2.bias"])) * mask.unsqueeze(-1)

    ms_torch = timed(torch_path, max(2, args.steps // 4))
    diff = float((out - torch_path()).abs().max())
    peaks = load_peaks()
    bytes_pair = 512 + 1024 + 1024 + 512 + 512 + 4  # z in, h out | h in, z in, out, mask
    gbs = N * N * bytes_pair / (ms / 1e3) / 1e9
    return {"metric": "pair transition N^2/s (residual + mask, one layer)", "value": N * N / (ms / 1e3),
            "unit": "N^2/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
            "higher_is_better": True, "dtype": "f16 tensor-core operands, f32 accumulate / f32 residual",
            "data": "synthetic (z ~ N(0,1), seeded weights)", "config": {"workload": f"pair transition, B=1, N={N}"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_pair": bytes_pair},
            "torch_fp32_unfused_ms": ms_torch, "max_abs_diff_vs_torch_fp32": diff,
            "status_word": ops.check_status(device)}


def run_embed(args, device, c_s: int = 384):
    """``--op embed``: the pair embedding producer (p_ij = Linear(2 c_s, 128)([s_i ; s_j]),
    p_mask = m_i m_j) for one N x N grid, against HBM (512 + 4 B written per pair) and
    against the reference's own operations (expand, cat, nn.Linear in fp32) on the GPU."""
    from genie_tk import ops
    N = args.N
    gen = torch.Generator().manual_seed(6)
    s = torch.randn(1, N, c_s, generator=gen).to(device)
    mask = torch.ones(1, N, device=device)
    w = (torch.randn(128, 2 * c_s, generator=gen) / (2 * c_s) ** 0.5).to(device)
    b = (0.1 * torch.randn(128, generator=gen)).to(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms = timed(lambda: ops.pair_embed(s, mask, w, b), args.steps)
    torch.backends.cuda.matmul.allow_tf32 = False

    def torch_path():
        s_i = s.unsqueeze(2).expand(-1, -1, N, -1)
        s_j = s.unsqueeze(1).expand(-1, N, -1, -1)
        return torch.nn.functional.linear(torch.cat([s_i, s_j], dim=-1), w, b), mask.unsqueeze(1) * mask.unsqueeze(2)

    ms_torch = timed(torch_path, max(2, args.steps // 4))
    diff = float((ops.pair_embed(s, mask, w, b)[0] - torch_path()[0]).abs().max())
    peaks = load_peaks()
    gbs = N * N * (512 + 4) / (ms / 1e3) / 1e9
    return {"metric": "pair embedding N^2/s (c_s = %d)" % c_s, "value": N * N / (ms / 1e3), "unit": "N^2/s",
            "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "n_gpus": 1, "higher_is_better": True,
            "dtype": "f32", "data": "synthetic", "config": {"workload": f"pair embedding, B=1, N={N}, c_s={c_s}"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_pair": 516},
            "torch_fp32_reference_ops_ms": ms_torch, "max_abs_diff_vs_torch_fp32": diff}


def claim_stdout():
    """Keep the process's stdout for the one JSON result line. Everything else written to
    file descriptor 1 -- NCCL's version banner at communicator set-up, library messages,
    stray prints -- goes to stderr instead. Returns the stream for the result."""
    sys.stdout.flush()
    result = os.fdopen(os.dup(1), "w", buffering=1)
    os.dup2(2, 1)
    return result


def main():
    result = claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--N", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--cpu-rows", type=int, default=256,
                    help="output rows per op timed by the CPU reference math (scaled to N rows)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="multi-GPU exchanges: peer-memory push kernels over NVLink, or NCCL collectives")
    ap.add_argument("--trimul-exchange", default="auto", choices=["auto", "gather", "channels"],
                    help="multi-GPU exchange of the multiplicative update (auto: the channel shards when "
                         "their x exchange is fused into the contraction's stores, else gather for <= 3 GPUs)")
    ap.add_argument("--op", default="stack", choices=["stack", "transition", "embed"],
                    help="stack: the headline workload (default); transition / embed: the pair-transition or "
                         "pair-embedding kernels alone")
    ap.add_argument("--separate-x", action="store_true",
                    help="peer exchange, channel shards: K2 then the x push, instead of K2 storing into the owners")
    ap.add_argument("--separate-transpose", action="store_true",
                    help="peer exchange: K4e then a transpose push, instead of K4e storing transposed into the peers")
    ap.add_argument("--push", default="kernel", choices=["kernel", "dma"],
                    help="peer exchanges: slab pushes with the push kernel or the copy engines")
    ap.add_argument("--k1-direct", action="store_true",
                    help="peer exchanges, channel mode: K1 writes the a/b channel shards straight into the "
                         "peers' buffers instead of a separate push")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), file=result, flush=True)
        return 0

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.op in ("transition", "embed"):
        print(json.dumps(run_transition(args, device) if args.op == "transition" else run_embed(args, device)),
              file=result, flush=True)
        return 0
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    line = run_sharded(args, rank, world, device) if world > 1 else run_ours(args, rank, world, device)
    if rank == 0 and world == 1 and not args.no_cpu:
        fn = cpu_sample(args.N, args.cpu_rows, os.cpu_count() or 1)
        # repeat the row sample until about 10 s of CPU work has been timed (at most 5 times)
        ests, measured = [], 0.0
        while measured < 10.0 and len(ests) < 5:
            est, parts, tot = fn()
            ests.append(est)
            measured += tot
        est = statistics.mean(ests)
        line["cpu_baseline"] = {"value": args.N * args.N / est, "unit": UNIT, "cores": os.cpu_count() or 1,
                                "kind": "port", "cpu": cpu_model(), "measured_s": round(measured, 2),
                                "sample": f"{len(ests)} x one {args.N}x{args.N} layer of the reference fp32 "
                                          f"PyTorch math (oracle port): row-independent parts over all pairs "
                                          f"plus {args.cpu_rows} output rows per op, per-row part scaled to "
                                          f"{args.N} rows; mean of the per-layer estimates"}
    if rank == 0:
        print(json.dumps(line), file=result, flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
