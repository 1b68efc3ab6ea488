"""Graph-forward throughput of the B200 executor on PyFlame IR graphs.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload all|fused|mlp|gemm_chain|encoder|convstack]
                    [--impl ours|reference] [--precision tf32x3|bf16] [--scaling strong|weak]

One run measures all five workload graphs (the default `--workload all`) and
prints ONE JSON line.  Its top-level keys are the GEMM chain's (Linear
4096->16384, GELU, Linear 16384->4096 on 8192 rows: the largest single-GPU
configuration); `workloads` carries the same record for every graph:
`value`, `ms_per_step`, `roofline` (dominant kernels' algorithmic work over
their share of the timed step, against the measured peak), `cpu_baseline`,
`e2e`, `clocks`, `gpu_launches`, and for the tensor-core graphs a `bf16`
sub-record (the optional bf16 mode, measured against the bf16 peak).

One step evaluates one batch of a graph.  `value` is whole-job samples/s
with inputs resident in HBM (CudaExecutor.execute_device: device pointers
bound to the graph's INPUT nodes, weights registered with set_resident,
outputs written in place), timed with CUDA events on the executor's stream,
max over ranks.  `e2e` is the same metric through the public host-buffer call
CudaExecutor.execute_streamed: every step copies the batch in from pinned host
memory and every output back, chunk copies overlapping compute.

Multi-GPU (torchrun, one process per GPU; `--scaling strong`, the default):
the global batch of each configuration is split along dim 0, B/N samples per
rank.  Weights are uploaded by rank 0 and broadcast once over NCCL before
timing, then registered as each rank's resident constants.  No collective
runs inside the timed regions.  In `e2e` every rank copies its host shard in
and writes its outputs into its own rows of ONE shared pinned host result
(a /dev/shm mapping pinned in every rank with cudaHostRegister): that write
is the output gather.  The MLP (batch 64 per launch) is not split: each GPU
runs its own batch of 64 (weak), as its record says.  `--scaling weak` gives
every rank the full batch instead.

`--impl reference` times PyFlame's own CPU code for the path (and the oracle
port where PyFlame has none) on the host cores, on bounded samples.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "graph fwd samples/sec at 1/2/4/8 B200; % of HBM / tensor-core roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = ["fused", "mlp", "gemm_chain", "encoder", "convstack"]
HEADLINE = "gemm_chain"
# full-size configurations: the global batch (split across ranks under strong scaling)
FULL = {
    "fused": dict(rows=8192, cols=4096),
    "mlp": dict(batch=64),
    "gemm_chain": dict(rows=8192),
    "encoder": dict(batch=32, seq=512),
    "convstack": dict(batch=256),
}
BATCH_KEY = {"fused": "rows", "mlp": "batch", "gemm_chain": "rows", "encoder": "batch", "convstack": "batch"}
WEAK_ONLY = {"mlp"}          # one 64-sample launch per GPU: never split
BF16 = ("gemm_chain", "encoder", "convstack")
# chunks of a rank's batch in the streamed e2e measurement (best of 2/4/8 on
# B200 at one GPU), never below MIN_CHUNK samples per chunk
E2E_CHUNKS = {"fused": 8, "mlp": 1, "gemm_chain": 8, "encoder": 2, "convstack": 8}
MIN_CHUNK = {"fused": 512, "mlp": 64, "gemm_chain": 256, "encoder": 2, "convstack": 16}
# timed steps when --steps is not given (about a second of device time each)
DEFAULT_STEPS = {"fused": 4000, "mlp": 4000, "gemm_chain": 100, "encoder": 300, "convstack": 300}
# CPU samples per step (bounded: a few seconds of host work each)
CPU_SAMPLE = {
    "fused": dict(rows=8192, cols=4096),
    "mlp": dict(batch=2048),
    "gemm_chain": dict(rows=16),
    "encoder": dict(batch=1, seq=512),
    "convstack": dict(batch=4),
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return FALLBACK_PEAKS, "fallback"


def profiled_traffic(workload):
    """DRAM bytes (read + write) per launch of the workload's dominant kernel,
    from the ncu summaries kept under profiles/ (a line
    `traffic_per_launch_bytes[<workload>] = <bytes>`), or None."""
    import re
    pat = re.compile(r"traffic_per_launch_bytes\[(\w+)\]\s*=\s*(\d+)")
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for m in pat.finditer(f.read_text()):
            if m.group(1) == workload:
                return int(m.group(2))
    return None


def ensure_built():
    from pyflame_b200 import _native
    if not _native.LIB_PATH.exists():
        from pyflame_b200 import build
        build.build()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region,
    plus read-only NVML queries about every half millisecond from this process
    (nvidia-smi's own interval is 50 ms)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.nvml = []
        self._stop = threading.Event()
        self._poller = None
        self.n0 = 0

    def start_polling(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:
                # the CUDA device's own NVML handle (NVML ignores CUDA_VISIBLE_DEVICES)
                pr = torch.cuda.get_device_properties(self.gpu)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(
                    f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0".encode())
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            return
        self._stop.clear()

        def run():
            while not self._stop.is_set():
                try:
                    self.nvml.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx, reasons(h)))
                except Exception:
                    return
                time.sleep(0.0005)

        self._poller = threading.Thread(target=run, daemon=True)
        self._poller.start()

    def stop_polling(self):
        self._stop.set()
        if self._poller:
            self._poller.join(timeout=2)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first_sample(self, timeout: float = 5.0):
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)
        self.n0 = len(self.lines)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.n0:]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        for clk, cmax, bits in self.nvml:
            sm.append(float(clk))
            mx = max(mx, float(cmax))
            for n, b in self.REASON_BITS.items():
                if bits & b:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_workload(name, **kw):
    from pyflame_b200 import workloads
    return workloads.BUILDERS[name](**kw)


class Dist:
    """Rank/world from the torchrun environment; NCCL process group for N > 1."""

    def __init__(self):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([float(v)], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def broadcast(self, t):
        if self.world > 1:
            import torch.distributed as dist
            dist.broadcast(t, src=0)

    def close(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


class SharedPinned:
    """One host array shared by every rank of this node (a /dev/shm mapping),
    each rank's rows pinned in that rank's process with cudaHostRegister, so
    device->host copies of all ranks land in one result."""

    def __init__(self, d: Dist, tag: str, shape, rows_lo: int, rows_hi: int):
        import torch
        self.d = d
        self.path = Path("/dev/shm") / f"pyflame_b200_{os.environ.get('MASTER_PORT', 'x')}_{tag}"
        nbytes = int(np.prod(shape)) * 4
        if d.rank == 0:
            with open(self.path, "wb") as f:
                f.truncate(nbytes)
        d.barrier()
        self.full = np.memmap(self.path, dtype=np.float32, mode="r+", shape=tuple(shape))
        self.mine = self.full[rows_lo:rows_hi]
        ptr = self.mine.ctypes.data
        lo = ptr // 4096 * 4096
        hi = -(-(ptr + self.mine.nbytes) // 4096) * 4096
        self.reg = (lo, hi - lo)
        rt = torch.cuda.cudart()
        rc = rt.cudaHostRegister(lo, hi - lo, 0)
        if int(rc) != 0:
            raise RuntimeError(f"cudaHostRegister of the shared result failed ({rc})")

    def close(self):
        import torch
        torch.cuda.cudart().cudaHostUnregister(self.reg[0])
        del self.mine
        del self.full
        self.d.barrier()
        if self.d.rank == 0:
            self.path.unlink(missing_ok=True)


def _shm_free() -> int:
    try:
        st = os.statvfs("/dev/shm")
        return st.f_bavail * st.f_frsize
    except OSError:
        return 0


def _chunks_for(name, shard):
    c = max(1, min(E2E_CHUNKS[name], shard // MIN_CHUNK[name]))
    while shard % c:
        c -= 1
    return c


def _roofline(name, w, kernels, ms_per_step, precision, pk, pk_kind):
    """Algorithmic work of the dominant kernel(s) per step over their average
    duration in the timed region: the CUDA-event step time apportioned by each
    kernel's share of device time in a profiled step of the same plan."""
    total = sum(ms for _, ms in kernels) or 1e-9
    top = max(kernels, key=lambda k: k[1]) if kernels else ("", 0.0)
    if w.flops:
        bound, unit = "tensor", "TFLOP/s"
        dom = sum(ms for n, ms in kernels if n.startswith(("gemm", "conv gemm", "attention", "small")))
        dom_ms = ms_per_step * dom / total
        achieved = w.flops / (dom_ms / 1e3) / 1e12 if dom else 0.0
        peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        if precision == "tf32x3":
            peak = peak / 2.0 / 3.0  # tf32 is half the bf16 rate; three products per output term
        source = f"{pk_kind} bf16 sustained" + (" / 2 / 3 for 3xTF32" if precision == "tf32x3" else "")
        share = dom / total
    else:
        bound, unit = "hbm", "GB/s"
        dom_ms = ms_per_step * top[1] / total
        achieved = w.bytes / (dom_ms / 1e3) / 1e9 if top[1] else 0.0
        peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        source = f"{pk_kind} hbm copy"
        share = top[1] / total
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak if peak else None,
            "traffic": profiled_traffic(name) if precision == "tf32x3" else None,
            "peak_source": source, "kernel": top[0], "kernel_share": share, "dominant_avg_ms_timed": dom_ms}


def measure(name, args, d: Dist, precision="tf32x3", with_e2e=True, with_cpu=True):
    """One workload on this rank: device-resident timing, profiled shares,
    streamed host-buffer e2e.  Returns the record (meaningful on rank 0)."""
    import torch

    import pyflame_b200 as pf

    world, rank = d.world, d.rank
    key = BATCH_KEY[name]
    glob = FULL[name][key]
    strong = args.scaling == "strong" and name not in WEAK_ONLY and world > 1
    if strong and glob % world:
        raise SystemExit(f"{name}: global batch {glob} does not split over {world} ranks")
    shard = glob // world if strong else glob
    w = build_workload(name, **{**FULL[name], key: shard})
    g, out_ids = w.graph(), w.output_ids()
    # batch inputs: this rank's rows of the global batch (strong), or its own full batch (weak)
    if strong and rank > 0:
        gw = build_workload(name, **FULL[name])
        lo = rank * shard
        for iname, t in w.inputs.items():
            t.node().set_constant_data(np.ascontiguousarray(gw.inputs[iname].node().constant_data()[lo:lo + shard]))
        del gw
    elif world > 1 and not strong:
        for t in w.inputs.values():
            t.node().set_constant_data(t.node().constant_data() + np.float32(rank))
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(device_id=d.local, precision=precision))
    bind, keep = {}, []
    for t in w.inputs.values():
        dv = torch.from_numpy(np.array(t.node().constant_data(), copy=True)).cuda()
        keep.append(dv)
        bind[t.node().id()] = dv.data_ptr()
    # weights: rank 0's copy broadcast once over NCCL, then each rank's resident constants
    weights = {}
    for nid, arr in sorted(w.weights().items()):
        dv = torch.from_numpy(np.array(arr, copy=True)).cuda() if rank == 0 else \
            torch.empty(arr.shape, dtype=torch.float32, device="cuda")
        d.broadcast(dv)
        weights[nid] = dv
    for nid, dv in weights.items():
        ex.set_resident(g.node(nid), dv.data_ptr())
    outs = [torch.empty(t.shape, dtype=torch.float32, device="cuda") for t in w.outputs]
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def step():
        return ex.execute_device(g, bind, out_ids, [o.data_ptr() for o in outs], stream=sp)

    torch.cuda.synchronize()
    steps = args.steps if args.steps is not None else DEFAULT_STEPS[name]
    for _ in range(max(args.warmup, 3)):
        r = step()
    torch.cuda.synchronize()
    launches = r.kernel_launches
    d.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    with ClockSampler(d.local) as clk:
        clk.wait_first_sample()
        clk.start_polling()
        ev[0].record(stream)
        for i in range(steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
        clk.stop_polling()
    d.barrier()
    per_step = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total_ms = d.max(ev[0].elapsed_time(ev[-1]))
    ms_per_step = total_ms / steps
    value = shard * world * steps / (total_ms / 1e3)  # whole-job samples (strong: the global batch)

    # per-kernel device times of one profiled step of the same plan on the same stream
    prof = pf.CudaExecutor(pf.CudaExecutor.Config(device_id=d.local, precision=precision, enable_profiling=True))
    for nid, dv in weights.items():
        prof.set_resident(g.node(nid), dv.data_ptr())
    prof.execute_device(g, bind, out_ids, [o.data_ptr() for o in outs], stream=sp)
    torch.cuda.synchronize()
    kernels = prof.last_profile()
    prof.close()

    e2e = None
    if with_e2e and not args.no_e2e:
        e2e = measure_e2e(name, args, d, w, ex, shard, strong, weights)
    ex.close()
    del keep, weights, outs
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    pk, pk_kind = peaks()
    rec = {"value": value, "unit": "samples/s", "ms_per_step": ms_per_step, "steps": steps,
           "scaling": "strong" if strong else "weak",
           "config": {"workload": name, **FULL[name], **w.meta, key: glob if strong else shard,
                      "per_gpu_batch": shard,
                      "parallelism": f"dp{world}" + (" (global batch split across GPUs)" if strong else
                                                     " (one full batch per GPU)" if world > 1 else ""),
                      "l2": "inputs larger than L2" if name == "fused" else "weights resident",
                      "precision": precision},
           "roofline": _roofline(name, w, kernels, ms_per_step, precision, pk, pk_kind),
           "clocks": clk.summary(), "gpu_launches": launches * steps, "launches_per_step": launches,
           "kernels": [{"name": n, "ms": round(ms, 4)} for n, ms in kernels],
           "step_ms_min": min(per_step), "step_ms_max": max(per_step)}
    if e2e is not None:
        rec["e2e"] = e2e
    if with_cpu and world == 1 and rank == 0 and not args.no_cpu:
        rec["cpu_baseline"] = cpu_baseline(name)
    return rec


def measure_e2e(name, args, d: Dist, w, ex, shard, strong, weights):
    """Samples/s through CudaExecutor.execute_streamed with host buffers: each
    step copies this rank's batch in from pinned memory and writes every
    output into this rank's rows of the result (one shared pinned host array
    over all ranks at N > 1), max over ranks."""
    import torch
    world = d.world
    key = BATCH_KEY[name]
    n_e2e = max(3, min(args.steps if args.steps is not None else 20, 20))
    pinned_in = {iname: torch.from_numpy(np.array(t.node().constant_data(), copy=True)).pin_memory()
                 for iname, t in w.inputs.items()}
    shared = []
    out_np = []
    # one shared result needs room for every rank's outputs in /dev/shm (the
    # same free space seen by every rank); otherwise each rank writes its rows
    # into its own pinned buffer
    need = sum(int(np.prod(t.shape)) * 4 * world for t in w.outputs)
    use_shared = world > 1 and d.max(0.0 if _shm_free() >= need + (64 << 20) else 1.0) == 0.0
    for k, t in enumerate(w.outputs):
        if use_shared:
            full_shape = [t.shape[0] * world, *t.shape[1:]]
            sh = SharedPinned(d, f"{name}_{k}", full_shape, d.rank * t.shape[0], (d.rank + 1) * t.shape[0])
            shared.append(sh)
            out_np.append(sh.mine)
        else:
            out_np.append(torch.empty(t.shape, dtype=torch.float32).pin_memory().numpy())
    h2d = sum(p.numel() * 4 for p in pinned_in.values())
    d2h = sum(o.nbytes for o in out_np)
    chunks = _chunks_for(name, shard)
    cw = build_workload(name, **{**FULL[name], key: shard // chunks})
    # the chunk graph's weights are the same device buffers (same seeded layers, same order)
    for (cnid, _), (nid, dv) in zip(sorted(cw.weights().items()), sorted(weights.items())):
        ex.set_resident(cw.graph().node(cnid), dv.data_ptr())
    c_in = {cw.inputs[iname].node().id(): pinned_in[iname].numpy() for iname in cw.inputs}
    c_out = cw.output_ids()
    for _ in range(2):
        r = ex.execute_streamed(cw.graph(), c_in, c_out, out_np)
    assert r.h2d_bytes == h2d and r.d2h_bytes == d2h, (r.h2d_bytes, h2d, r.d2h_bytes, d2h)
    d.barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        ex.execute_streamed(cw.graph(), c_in, c_out, out_np)
    dt = d.max(time.perf_counter() - t0)
    glob_samples = shard * world
    e2e = {"value": glob_samples * n_e2e / dt, "unit": "samples/s", "h2d_bytes_per_step": h2d * world,
           "d2h_bytes_per_step": d2h * world, "ms_per_step": dt / n_e2e * 1e3, "steps": n_e2e,
           "chunks_per_gpu": chunks,
           "api": "CudaExecutor.execute_streamed (pfc_executor_execute_streamed), pinned host buffers",
           "gather": ("every rank's outputs into its rows of one shared pinned host result" if use_shared else
                      "each rank's outputs into its own pinned host buffer (/dev/shm too small for one result)"
                      if world > 1 else "single GPU")}
    if world == 1:
        # the plain host-buffer call for comparison: upload, compute, download in sequence
        for iname, t in w.inputs.items():
            t.node().set_constant_data(pinned_in[iname].numpy(), copy=False)
        w.graph().version += 1
        for _ in range(2):
            rr = ex.execute(w.graph(), w.output_ids(), out=out_np)
            assert rr.success, rr.error_message
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            ex.execute(w.graph(), w.output_ids(), out=out_np)
        ds = time.perf_counter() - t0
        e2e["serial"] = {"value": shard * n_e2e / ds, "ms_per_step": ds / n_e2e * 1e3,
                         "api": "CudaExecutor.execute (pfc_executor_execute)"}
    for sh in shared:
        sh.close()
    return e2e


def run_ours(args):
    ensure_built()
    d = Dist()
    names = WORKLOADS if args.workload == "all" else [args.workload]
    recs = {}
    for name in names:
        recs[name] = measure(name, args, d, precision=args.precision)
        if args.workload == "all" and args.precision == "tf32x3" and name in BF16 and not args.no_bf16:
            b = measure(name, args, d, precision="bf16", with_e2e=False, with_cpu=False)
            recs[name]["bf16"] = {k: b[k] for k in ("value", "ms_per_step", "roofline", "clocks", "gpu_launches")}
    if d.rank == 0:
        head = HEADLINE if HEADLINE in recs else names[0]
        h = recs[head]
        line = {
            "metric": METRIC, "value": h["value"], "unit": "samples/s", "n_gpus": d.world, "steps": h["steps"],
            "warmup": args.warmup, "ms_per_step": h["ms_per_step"], "higher_is_better": True,
            "scaling": h["scaling"], "vs_baseline": None,
            "dtype": "f32" if args.precision == "tf32x3" else "bf16",
            "data": "synthetic (seeded numpy: inputs seed 42, layers 43+i)",
            "config": h["config"], "roofline": h["roofline"], "cpu_baseline": h.get("cpu_baseline"),
            "e2e": h.get("e2e"), "clocks": h["clocks"], "gpu_launches": h["gpu_launches"],
            "workloads": recs,
        }
        print(json.dumps(line), flush=True)
    d.close()


# ---------------------------------------------------------------------------
# CPU: PyFlame's own code for the path, on the host cores
# ---------------------------------------------------------------------------

class CpuFused:
    """The fused graph on a row sample with PyFlame's CPU code, z computed
    once: the reference executor (executor.cpp:205-524) evaluates
    z = sigmoid(x*y+0.5) - relu(x); ops::sum_dim_cpu / mean_dim_cpu /
    max_dim_cpu (reduction.cpp:49-121) reduce its rows; LayerNorm, which
    PyFlame has no CPU code for, is the oracle restatement applied to that z
    (a one-node graph), one oracle thread per shard.  Rows are split into one
    shard per host thread.  Inputs and graphs are made once; step() times
    only the evaluation."""

    def __init__(self, rows, cols, threads):
        import pyflame_b200 as pf
        from oracle import oracle as O
        self.O = O
        self.ref = O.Reference() if O.Reference.available() else None
        self.kind = "reference" if self.ref else "port"
        self.rows, self.cols, self.threads = rows, cols, threads
        rng = np.random.default_rng(42)
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        y = np.random.default_rng(43).standard_normal((rows, cols), dtype=np.float32)
        self.shards = []
        for sh in np.array_split(np.arange(rows), threads):
            pf.reset_graph()
            xs, ys = pf.tensor(x[sh]), pf.tensor(y[sh])
            z = pf.sigmoid(xs * ys + 0.5) - pf.relu(xs)
            pf.reset_graph()
            zin = pf.Tensor.input(np.zeros((len(sh), cols), np.float32))
            ln = pf.nn.LayerNorm(cols)(zin)
            self.shards.append((z, zin, ln))

    def _work(self, i):
        z, zin, ln = self.shards[i]
        self.O.set_threads(1)
        if self.ref is not None:
            zz = self.ref.execute_cpu(z.graph(), [z.node().id()])[z.node().id()]
            self.ref.reduce_dim("sum", zz, 1)
            self.ref.reduce_dim("mean", zz, 1)
            self.ref.reduce_dim("max", zz, 1)
        else:
            zz = self.O.run(z.graph(), [z.node().id()])[z.node().id()]
            self.O.run(z.graph(), [z.sum(1).node().id(), z.mean(1).node().id(), z.max(1).node().id()])
        zin.node().set_constant_data(zz, copy=False)
        zin.graph().version += 1
        self.O.run(ln.graph(), [ln.node().id()])

    def step(self):
        import concurrent.futures as cf
        with cf.ThreadPoolExecutor(self.threads) as pool:
            t0 = time.perf_counter()
            list(pool.map(self._work, range(len(self.shards))))
            return time.perf_counter() - t0


class CpuOracle:
    """Graphs PyFlame's CPU executor cannot evaluate (broadcast bias adds,
    Conv2d, BatchNorm, LayerNorm, pools, batched matmul) through the oracle
    port on all host threads, on a bounded batch sample."""

    def __init__(self, workload, threads):
        from oracle import oracle as O
        self.O = O
        self.kind = "port"
        self.w = build_workload(workload, **CPU_SAMPLE[workload])
        self.threads = threads

    def step(self):
        self.O.set_threads(self.threads)
        t0 = time.perf_counter()
        self.O.run(self.w.graph(), self.w.output_ids())
        return time.perf_counter() - t0


def cpu_runner(workload, threads):
    if workload == "fused":
        s = CPU_SAMPLE["fused"]
        return CpuFused(s["rows"], s["cols"], threads)
    return CpuOracle(workload, threads)


def _sample_units(workload):
    return CPU_SAMPLE[workload][BATCH_KEY[workload]]


def cpu_baseline(workload):
    threads = os.cpu_count() or 1
    try:
        r = cpu_runner(workload, threads)
        r.step()  # warm
        dt = r.step()
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "samples/s", "error": str(e)}
    return {"value": _sample_units(workload) / dt, "unit": "samples/s", "cores": threads, "kind": r.kind,
            "ms_per_sample_step": dt * 1e3,
            "sample": f"{workload} {CPU_SAMPLE[workload]} per step (samples are independent)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    names = WORKLOADS if args.workload == "all" else [args.workload]
    steps = args.steps if args.steps is not None else 5
    recs = {}
    for name in names:
        r = cpu_runner(name, threads)
        for _ in range(max(args.warmup, 0)):
            r.step()
        times = [r.step() for _ in range(steps)]
        units = _sample_units(name)
        v = units / statistics.median(times)
        recs[name] = {"value": v, "unit": "samples/s", "ms_per_step": statistics.mean(times) * 1e3, "steps": steps,
                      "config": {"workload": name, **FULL[name], "sample": CPU_SAMPLE[name]},
                      "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": r.kind,
                                       "sample": f"{name} {CPU_SAMPLE[name]} per step"},
                      "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    head = HEADLINE if HEADLINE in recs else names[0]
    h = recs[head]
    line = {"impl": "reference", "metric": METRIC, "value": h["value"], "unit": "samples/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": h["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy)",
            "config": h["config"], "cpu_baseline": h["cpu_baseline"], "e2e": h["e2e"], "workloads": recs}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps per workload (default: about a second of device time each)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="all", choices=["all", *WORKLOADS])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="tf32x3", choices=["tf32x3", "bf16"])
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurements")
    ap.add_argument("--no-bf16", action="store_true", help="skip the bf16 sub-records")
    ap.add_argument("--size", action="append", default=[], metavar="KEY=INT",
                    help="override a workload size (e.g. rows=1024) for small profiling runs of one "
                         "--workload; the default sizes are the benchmark configuration")
    args = ap.parse_args()
    for kv in args.size:
        k, v = kv.split("=")
        if args.workload == "all" or k not in FULL[args.workload]:
            ap.error(f"--size needs one --workload with a size '{k}'")
        FULL[args.workload][k] = int(v)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
