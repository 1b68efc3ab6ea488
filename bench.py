"""Graph-forward throughput of the B200 executor on PyFlame IR graphs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload fused|mlp|gemm_chain|encoder|convstack]
                    [--impl ours|reference]

One step evaluates one batch of the workload's graph.  `value` is whole-job
samples/s with inputs resident in HBM (CudaExecutor.execute_device, device
pointers bound to the graph's INPUT nodes, outputs written in place); `e2e`
is the same metric through the public host-buffer call with inputs copied
from pinned host memory and all outputs read back every step:
CudaExecutor.execute_streamed (the batch as micro-batches whose copies
overlap compute), and under `e2e.serial` CudaExecutor.execute (one upload,
compute, download in sequence); a batch too small to split (the MLP's 64
samples) takes execute alone.  Multi-GPU runs (torchrun, one process per
GPU) give every rank its own full batch (weak scaling): weights are broadcast
once from rank 0 over NCCL and registered as each rank's resident constants
(CudaExecutor.set_resident); no collective runs inside the timed region.
`--impl reference` times PyFlame's own CPU code for the path on the host
cores instead.
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

# full-size configurations (the fused elementwise+reduction graph is the headline)
FULL = {
    "fused": dict(rows=8192, cols=4096),
    "mlp": dict(batch=64),
    "gemm_chain": dict(rows=8192),
    "encoder": dict(batch=32, seq=512),
    "convstack": dict(batch=256),
}
# micro-batches of the end-to-end host-buffer measurement (execute_streamed)
# chunks of the batch in the streamed e2e measurement, each the best of 2/4/8 measured on B200
E2E_CHUNKS = {"fused": 8, "mlp": 1, "gemm_chain": 8, "encoder": 2, "convstack": 8}
# CPU-baseline samples (bounded, seconds of CPU work)
CPU_SAMPLE = {
    "fused": dict(rows=8192, cols=4096),
    "mlp": dict(batch=64),
    "gemm_chain": dict(rows=16),
    "encoder": dict(batch=1, seq=512),
    "convstack": dict(batch=2),
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
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
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.nvml = []  # (sm MHz, max MHz, clock-event reason bits) read in-process
        self._stop = threading.Event()
        self._poller = None

    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def start_polling(self):
        """Read the SM clock and clock-event reasons through NVML about every
        half millisecond until stop_polling(): a timed region of a few
        milliseconds still gets samples (nvidia-smi's own interval is 50 ms).
        Read-only queries; no GPU setting is touched."""
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
        """nvidia-smi needs a moment to start; begin timing once it samples."""
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
        for ln in self.lines[getattr(self, "n0", 0):]:
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


def leaf_weights(w):
    """Resident constant leaves (weights) of the workload graph, by node id."""
    g = w.outputs[0].graph()
    out = {}
    input_ids = {t.node().id() for t in w.inputs.values()}
    for n in g.topological_order([t.node() for t in w.outputs]):
        if not n.is_operation() and n.id() not in input_ids and n.has_constant_data() and n.numel() > 1:
            a = n.constant_data()
            if np.all(a == a.flat[0]):
                continue  # a constant of equal values stays a scalar in the plan
            out[n.id()] = a
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    ensure_built()
    import pyflame_b200 as pf

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    w = build_workload(args.workload, **FULL[args.workload])
    g = w.outputs[0].graph()
    out_ids = [t.node().id() for t in w.outputs]
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(device_id=local, precision=args.precision))

    # batch inputs in HBM (each rank its own batch) and weights: broadcast from rank 0 once
    bind = {}
    keep = []
    for name, t in w.inputs.items():
        arr = t.node().constant_data()
        if world > 1:
            arr = arr + np.float32(rank)  # distinct data per rank
        d = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
        keep.append(d)
        bind[t.node().id()] = d.data_ptr()
    # weights: uploaded by rank 0, broadcast once over NCCL, then registered as
    # the executors' resident constants (their tensor-core operands are
    # prepared once and kept)
    weights = {}
    for nid, arr in leaf_weights(w).items():
        d = torch.from_numpy(np.ascontiguousarray(arr)).cuda() if rank == 0 else \
            torch.empty(arr.shape, dtype=torch.float32, device="cuda")
        if world > 1:
            dist.broadcast(d, src=0)
        keep.append(d)
        weights[nid] = d
    for nid, d in weights.items():
        ex.set_resident(g.node(nid), d.data_ptr())
    outs = [torch.empty(t.shape, dtype=torch.float32, device="cuda") for t in w.outputs]
    # a dedicated stream: the executor runs its work on it and the events are recorded on it
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    assert sp != 0

    def step():
        return ex.execute_device(g, bind, out_ids, [o.data_ptr() for o in outs], stream=sp)

    torch.cuda.synchronize()  # inputs and weights were uploaded on the default stream
    for _ in range(max(args.warmup, 3)):
        r = step()
    torch.cuda.synchronize()
    launches_per_step = r.kernel_launches
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clk:
        clk.wait_first_sample()
        clk.start_polling()
        ev[0].record(stream)
        for i in range(args.steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
        clk.stop_polling()
    per_step = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    if world > 1:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * w.samples * args.steps / (total_ms / 1e3)

    # the dominant kernel: per-kernel device times from a profiled run on the same stream
    prof = pf.CudaExecutor(pf.CudaExecutor.Config(device_id=local, precision=args.precision,
                                                  enable_profiling=True))
    for nid, d in weights.items():
        prof.set_resident(g.node(nid), d.data_ptr())
    prof.execute_device(g, bind, out_ids, [o.data_ptr() for o in outs], stream=sp)
    torch.cuda.synchronize()
    kernels = prof.last_profile()
    prof.close()

    # end to end through the public host-buffer API, inputs from pinned host memory
    e2e = None
    if rank == 0 and not args.no_e2e:
        pinned_in = {}
        for name, t in w.inputs.items():
            pt = torch.from_numpy(t.node().constant_data()).pin_memory()
            t.node().set_constant_data(pt.numpy(), copy=False)
            pinned_in[name] = pt
        g.version += 1  # payload pointers changed: rebuild the native graph description
        pinned_out = [torch.empty(t.shape, dtype=torch.float32).pin_memory() for t in w.outputs]
        out_np = [p.numpy() for p in pinned_out]
        h2d = sum(t.node().constant_data().nbytes for t in w.inputs.values())
        d2h = sum(o.nbytes for o in out_np)
        n_e2e = max(3, min(args.steps, 20))
        # (a) one execute call per step: upload, compute, download in sequence
        for _ in range(2):
            rr = ex.execute(g, out_ids, out=out_np)
            assert rr.success, rr.error_message
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            rr = ex.execute(g, out_ids, out=out_np)
        dt_serial = time.perf_counter() - t0
        # (b) execute_streamed: the same batch as micro-batches of one chunk
        # graph, each chunk's compute overlapping the next upload and the
        # previous download
        serial = {"value": w.samples * n_e2e / dt_serial, "ms_per_step": dt_serial / n_e2e * 1e3,
                  "api": "CudaExecutor.execute (pfc_executor_execute)"}
        chunks = E2E_CHUNKS[args.workload]
        if chunks > 1:
            key = next(iter(FULL[args.workload]))  # the batch-size key (rows / batch)
            cw = build_workload(args.workload, **{**FULL[args.workload], key: FULL[args.workload][key] // chunks})
            cg = cw.outputs[0].graph()
            c_in = {cw.inputs[name].node().id(): pinned_in[name].numpy() for name in cw.inputs}
            c_out = [t.node().id() for t in cw.outputs]
            for _ in range(2):
                ex.execute_streamed(cg, c_in, c_out, out_np)
            t0 = time.perf_counter()
            for _ in range(n_e2e):
                ex.execute_streamed(cg, c_in, c_out, out_np)
            dt = time.perf_counter() - t0
            e2e = {"value": w.samples * n_e2e / dt, "unit": "samples/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "ms_per_step": dt / n_e2e * 1e3, "steps": n_e2e,
                   "api": f"CudaExecutor.execute_streamed (pfc_executor_execute_streamed), {chunks} chunks, "
                          "pinned host buffers",
                   "serial": serial}
        else:
            # a batch too small to split: one execute call per step
            e2e = {"value": serial["value"], "unit": "samples/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "ms_per_step": serial["ms_per_step"], "steps": n_e2e,
                   "api": serial["api"] + ", pinned host buffers"}

    if rank == 0:
        pk, pk_kind = peaks()
        total_kernel_ms = sum(ms for _, ms in kernels) or 1e-9
        top = max(kernels, key=lambda k: k[1]) if kernels else ("", 0.0)
        # Algorithmic work of the dominant kernel(s) per step divided by their
        # average duration in the timed region: the per-step time measured with
        # CUDA events on the launching stream, apportioned by each kernel's
        # share of device time in a profiled step of the same plan.
        if w.flops:
            bound, unit = "tensor", "TFLOP/s"
            gemm_ms = sum(ms for name, ms in kernels if name.startswith(("gemm", "conv gemm", "attention")))
            dom_ms = ms_per_step * gemm_ms / total_kernel_ms
            achieved = w.flops / (dom_ms / 1e3) / 1e12 if gemm_ms else 0.0
            # kernels run inside a long loop: the sustained GEMM figure
            peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
            if args.precision == "tf32x3":
                peak = peak / 2.0 / 3.0  # tf32 is half the bf16 rate; three products per output term
        else:
            bound, unit = "hbm", "GB/s"
            dom_ms = ms_per_step * top[1] / total_kernel_ms
            achieved = w.bytes / (dom_ms / 1e3) / 1e9 if top[1] else 0.0
            peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        traffic = profiled_traffic(args.workload)
        cpu = cpu_baseline(args.workload) if (world == 1 and not args.no_cpu) else None
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if args.precision == "tf32x3" else "bf16",
            "data": "synthetic (seeded numpy: inputs seed 42, layers 43+i)",
            "config": {"workload": args.workload, **FULL[args.workload], **w.meta,
                       "parallelism": f"dp{world} (weak: one full batch per GPU)",
                       "l2": "inputs larger than L2" if args.workload == "fused" else "weights resident",
                       "precision": args.precision},
            "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak if peak else None, "traffic": traffic,
                         "peak_source": f"{pk_kind}" + (" (bf16/2/3 for 3xTF32)" if bound == "tensor" else ""),
                         "kernel": top[0], "kernel_avg_ms_timed": dom_ms, "kernel_ms_profiled_once": top[1],
                         "kernel_share": top[1] / total_kernel_ms},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "kernels": [{"name": n, "ms": round(ms, 4)} for n, ms in kernels],
            "step_ms_min": min(per_step), "step_ms_max": max(per_step),
        }
        print(json.dumps(line), flush=True)
    ex.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU: PyFlame's own code for the path, on the host cores
# ---------------------------------------------------------------------------

def _cpu_fused_step(rows, cols, threads):
    """The fused graph on a row sample with PyFlame's CPU code: the reference
    executor (executor.cpp:205-524) evaluates z = sigmoid(x*y+0.5) - relu(x);
    ops::sum_dim_cpu / mean_dim_cpu / max_dim_cpu (reduction.cpp:49-121)
    reduce rows; LayerNorm, which PyFlame has no CPU code for, comes from the
    oracle restatement.  Rows are split across threads."""
    import concurrent.futures as cf

    import pyflame_b200 as pf
    from oracle import oracle as O

    use_ref = O.Reference.available()
    ref = O.Reference() if use_ref else None
    rng = np.random.default_rng(42)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    y = rng.standard_normal((rows, cols), dtype=np.float32)
    shards = np.array_split(np.arange(rows), threads)
    graphs = []
    for sh in shards:
        pf.reset_graph()
        xs, ys = pf.tensor(x[sh]), pf.tensor(y[sh])
        z = pf.sigmoid(xs * ys + 0.5) - pf.relu(xs)
        ln = pf.nn.LayerNorm(cols)(z)
        graphs.append((z, ln))

    def work(i):
        z, ln = graphs[i]
        g = z.graph()
        if use_ref:
            zz = ref.execute_cpu(g, [z.node().id()])[z.node().id()]
            ref.reduce_dim("sum", zz, 1)
            ref.reduce_dim("mean", zz, 1)
            ref.reduce_dim("max", zz, 1)
        O.run(g, [ln.node().id()])

    with cf.ThreadPoolExecutor(threads) as pool:
        t0 = time.perf_counter()
        list(pool.map(work, range(len(graphs))))
        dt = time.perf_counter() - t0
    return rows / dt, ("reference" if use_ref else "port")


def _cpu_oracle_step(workload, threads):
    import pyflame_b200 as pf  # noqa: F401
    from oracle import oracle as O
    w = build_workload(workload, **CPU_SAMPLE[workload])
    g = w.outputs[0].graph()
    os.environ["ORACLE_THREADS"] = str(threads)
    t0 = time.perf_counter()
    O.run(g, [t.node().id() for t in w.outputs])
    dt = time.perf_counter() - t0
    return w.samples / dt, "port"


def cpu_step(workload, threads):
    if workload == "fused":
        s = CPU_SAMPLE["fused"]
        return _cpu_fused_step(s["rows"], s["cols"], threads)
    return _cpu_oracle_step(workload, threads)


def cpu_baseline(workload):
    threads = os.cpu_count() or 1
    try:
        cpu_step(workload, threads)  # warm
        v, kind = cpu_step(workload, threads)
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "samples/s", "error": str(e)}
    sample = CPU_SAMPLE[workload]
    return {"value": v, "unit": "samples/s", "cores": threads, "kind": kind,
            "sample": f"{workload} {sample} per step (rows/images/sequences are independent)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(max(args.warmup, 0)):
        cpu_step(args.workload, threads)
    vals, kind = [], "port"
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, kind = cpu_step(args.workload, threads)
        vals.append(v)
    wall = time.perf_counter() - t0
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy)",
            "config": {"workload": args.workload, **FULL[args.workload], "sample": CPU_SAMPLE[args.workload]},
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": kind,
                             "sample": f"{args.workload} {CPU_SAMPLE[args.workload]} per step"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: about 2 s of device time for the workload)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="fused", choices=sorted(FULL))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="tf32x3", choices=["tf32x3", "bf16"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurement")
    ap.add_argument("--size", action="append", default=[], metavar="KEY=INT",
                    help="override a workload size (e.g. rows=1024) for small profiling runs; "
                         "the default sizes are the benchmark configuration")
    args = ap.parse_args()
    for kv in args.size:
        k, v = kv.split("=")
        if k not in FULL[args.workload]:
            ap.error(f"{args.workload} has no size '{k}' (sizes: {', '.join(FULL[args.workload])})")
        FULL[args.workload][k] = int(v)
    if args.steps is None:
        args.steps = {"fused": 20000, "mlp": 20000, "gemm_chain": 200, "encoder": 100, "convstack": 100}[
            args.workload] if args.impl == "ours" else 5
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
