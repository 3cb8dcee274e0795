"""Benchmark of the `cuda` target on its headline workload: ResNet-50 (BASELINE configs 0 and 4).

Default arm (our backend), one process per GPU (``torchrun`` for N > 1, batch-sharded replicas,
weak scaling: every GPU runs its own batch of ``--batch`` images, no collectives on the data path):

* ``value``: whole-job img/s of the compiled ResNet-50 (O3 graph, CUDA Graph replay) with the
  inputs resident in HBM, timed with CUDA events on the model's stream over ``--steps`` replays
  after ``--warmup`` untimed ones, max over ranks;
* ``e2e``: the same through the public API ``CudaCompiledModel.run`` from pinned host memory
  (host->device input copy, replay, device->host logits copy every step; the input is uploaded
  in four slices whose copies overlap the stem and layer1 of the earlier slices);
* ``roofline``: the dominant kernel (the implicit-GEMM convolution / GEMM launches) from one
  eagerly launched pass with CUDA events around every launch, against MEASURED_PEAKS.json;
* ``latency_b1``: batch-1 p50 latency (public API and device-only replay);
* ``bert``: BERT-base sequence-128 batch-32 seq/s, device-timed replays and
  through ``run``;
* ``cpu_baseline``: the reference's own C backend (gcc + OpenMP) on this host's cores, on a
  bounded batch.

``--impl reference`` runs the reference's C backend (the unmodified reference, installed in
baseline/_ref, through its public ``compile_graph`` API) on the same workload on the host CPU.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "ml-graph-compiler_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "ResNet-50 b256 img/s (fp32 semantics, O3 graph)"
UNIT = "img/s"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """Sample SM clocks, power and clock-event (throttle) reasons every 20 ms while the timed
    region runs, through NVML (the GPU found by its PCI bus id), else ``nvidia-smi -lms``."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.device = device
        self.samples: list[tuple[float, float, set[str]]] = []  # (sm MHz, max MHz, reasons)
        self.proc: subprocess.Popen | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._nvml = None
        self._handle = None

    def _open_nvml(self) -> bool:
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            try:
                self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self._nvml = pynvml
            return True
        except Exception:
            return False

    def _poll_nvml(self) -> None:
        nv, h = self._nvml, self._handle
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = int(get_reasons(h))
                self.samples.append((sm, mx, {k for k, v in self.REASONS.items() if bits & v}))
            except Exception:
                pass
            self._stop.wait(0.02)

    def _poll_smi(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((sm, mx, {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))

    def __enter__(self) -> "Clocks":
        if self._open_nvml():
            self._thread = threading.Thread(target=self._poll_nvml, daemon=True)
        else:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._thread = threading.Thread(target=self._poll_smi, daemon=True)
            except OSError:
                self.proc = None
        if self._thread is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        sm = [x[0] for x in self.samples]
        reasons = sorted(set().union(*[x[2] for x in self.samples])) if self.samples else []
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max((x[1] for x in self.samples), default=None), "reasons": reasons,
                "samples": len(sm), "source": "nvml" if self._nvml is not None else "nvidia-smi"}


def measured_traffic(batch: int) -> int | None:
    """DRAM bytes (read + write) of one step's GEMM launches, from the committed ncu summary
    (measured at batch 32, scaled by the batch)."""
    f = ROOT / "profiles" / "resnet50_step_launches.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_bytes_per_step_b32:"):
            return int(int(line.split(":")[1]) * batch / 32)
    return None


def build_r50(batch: int, seed: int = 4):
    from mgc_cuda import zoo
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    g = zoo.resnet50(batch=batch, seed=0)
    optimize(g, "O3")
    schedule(g)
    return g


def bert_throughput(precision: str, device: int, steps: int, warmup: int) -> dict:
    """BERT-base, sequence 128, batch 32 (the metric's seq/s): CUDA Graph
    replays with resident inputs timed with CUDA events on the model's stream, and the same
    through ``run`` from pinned host buffers (token ids and mask uploaded, every output read back
    each step)."""
    import torch

    from mgc_cuda import zoo
    from mgc_cuda.runtime import compile_graph
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    batch, seq = 32, 128
    g = zoo.bert(batch=batch, seq=seq, seed=2)
    optimize(g, "O3")
    schedule(g)
    # the planner's naive strategy, as for ResNet-50: every buffer its own memory (3.0 GB), so no
    # attention operand read through strides lies under a GEMM's output and needs a copy first
    m = compile_graph(g, precision=precision, device=device, strategy="naive")
    feeds = zoo.feeds(g, 2)
    outs = m.run(feeds)
    stream = torch.cuda.ExternalStream(m.stream)
    for _ in range(warmup):
        m.run_device(sync=False)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        m.run_device(sync=False)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # end to end with pinned host buffers, as for ResNet-50
    pinned_in = {}
    for k, v in feeds.items():
        buf = torch.empty(v.shape, dtype=torch.from_numpy(np.ascontiguousarray(v)).dtype, pin_memory=True).numpy()
        buf[...] = v
        pinned_in[k] = buf
    pinned_out = {}
    for k, v in outs.items():
        pinned_out[k] = torch.empty(v.shape, dtype=torch.from_numpy(np.ascontiguousarray(v)).dtype, pin_memory=True).numpy()
    for _ in range(2):
        m.run(pinned_in, out=pinned_out)
    t0 = time.perf_counter()
    for _ in range(steps):
        m.run(pinned_in, out=pinned_out)
    e2e_s = (time.perf_counter() - t0) / steps
    m.close()
    return {
        "metric": "BERT-base seq128 seq/s (batch 32, O3 graph)", "value": round(batch / (ms / 1e3), 2),
        "unit": "seq/s", "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup,
        "e2e": {"value": round(batch / e2e_s, 2), "unit": "seq/s",
                "h2d_bytes_per_step": int(sum(np.asarray(v).nbytes for v in feeds.values())),
                "d2h_bytes_per_step": int(sum(np.asarray(v).nbytes for v in outs.values()))},
        "l2": "weights (hi + lo TF32 parts) and activations stream through HBM every step, larger than L2",
        "memory_plan": "naive",
    }


def cpu_reference_run(batch: int, steps: int, warmup: int) -> dict:
    """The reference C backend on this host: compile_graph(O3 graph) with gcc + OpenMP."""
    os.environ.setdefault("MGC_CC", "/usr/bin/gcc")
    from mgc_cuda import _reference  # noqa: F401  (the unmodified reference, baseline/_ref)
    from ml_graph_compiler.codegen import compile_graph as c_compile

    g = build_r50(batch)
    x = np.random.default_rng(4).standard_normal((batch, 3, 224, 224)).astype(np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        model = c_compile(g, cache_dir=tmp)
        times = model.benchmark({"image": x}, warmup=warmup, repeat=steps)
        threads = model.max_threads()
        openmp = model.openmp
    p50 = statistics.median(times)
    return {"value": batch / p50, "p50_s": p50, "cores": threads, "openmp": openmp, "batch": batch,
            "times": times}


def run_reference_arm(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    batch = args.ref_batch
    try:
        r = cpu_reference_run(batch, args.steps, args.warmup)
    except Exception as exc:  # the reference could not be built or run on this host
        print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
        return
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["p50_s"] * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"resnet50 O3, C backend (gcc+OpenMP), batch {batch} per step",
                   "batch_per_step": batch, "threads": r["cores"], "openmp": r["openmp"]},
        "cpu_baseline": {"value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "reference",
                         "sample": f"ResNet-50 O3 batch {batch}, {args.steps} timed runs"},
        "e2e": {"value": round(r["value"], 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=256, help="images per GPU per step")
    ap.add_argument("--precision", default="tf32", choices=["tf32", "strict", "fp32"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-batch", type=int, default=16, help="images per step of the CPU reference arm")
    ap.add_argument("--cpu-batch", type=int, default=8, help="images of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--no-bert", action="store_true", help="skip the BERT-base seq/s measurement")
    ap.add_argument("--strategy", default="naive", choices=["greedy_by_size", "first_fit", "naive"],
                    help="the reference planner's memory strategy for the benchmark model; naive gives every "
                         "buffer its own memory (11.7 GB arena at batch 256), which lets run() upload the image in "
                         "slices that overlap the stem and layer1")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch

    from mgc_cuda.replicas import ReplicaGroup

    group = ReplicaGroup(backend="nccl", timeout_s=300)
    world, rank, local = group.world, group.rank, group.local_rank
    torch.cuda.set_device(local)

    from mgc_cuda.lowering import algorithmic_cost
    from mgc_cuda.runtime import compile_graph
    from ml_graph_compiler import ops

    pk = peaks()
    g = build_r50(args.batch)
    flops, nbytes = algorithmic_cost(g)
    model = compile_graph(g, precision=args.precision, device=local, strategy=args.strategy)
    x = np.random.default_rng(4 + rank).standard_normal((args.batch, 3, 224, 224)).astype(np.float32)
    # resident input for the device-timed loop
    model.run({"image": x})
    stream = torch.cuda.ExternalStream(model.stream)

    barrier = group.barrier

    for _ in range(args.warmup):
        model.run_device(sync=False)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            model.run_device(sync=False)
        end.record(stream)
        end.synchronize()
    barrier()
    ms = group.max(start.elapsed_time(end))
    ms_per_step = ms / args.steps
    value = world * args.batch * args.steps / (ms / 1e3)

    # end to end through the public API, pinned host buffers
    pinned_in = torch.empty((args.batch, 3, 224, 224), dtype=torch.float32, pin_memory=True).numpy()
    pinned_in[...] = x
    pinned_out = torch.empty((args.batch, 1000), dtype=torch.float32, pin_memory=True).numpy()
    for _ in range(2):
        model.run({"image": pinned_in}, out={"logits": pinned_out})
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.run({"image": pinned_in}, out={"logits": pinned_out})
    e2e_s = group.max(time.perf_counter() - t0)
    e2e = world * args.batch * args.steps / e2e_s

    # dominant kernel: per-launch CUDA events (eager pass), GEMM-family nodes
    prof_runs = 3
    per_node = [0.0] * len(g.nodes)
    for _ in range(prof_runs):
        for i, (_, _, s) in enumerate(model.profile()):
            per_node[i] += s / prof_runs
    gemm_nodes = [i for i, n in enumerate(g.nodes) if n.op in ("FusedConv", "FusedGemm", "Conv", "Gemm", "MatMul")]
    gemm_s = sum(per_node[i] for i in gemm_nodes)
    gemm_flops = sum(ops.flops(g.nodes[i]) for i in gemm_nodes)
    launches = sum(1 for r in model.lowered.launches if r.kind == 1)
    tf32_peak = pk["bf16_tflops"] / 2.0
    achieved = gemm_flops / gemm_s / 1e12 if gemm_s > 0 else 0.0
    step_bound_s = max(flops / (tf32_peak * 1e12), nbytes / (pk["hbm_gbs"] * 1e9))
    total_prof = sum(per_node)

    line: dict = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"resnet50 v1.5 O3, batch {args.batch} per GPU, CUDA Graph replay",
            "batch_per_gpu": args.batch, "precision": args.precision, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (input 154 MB, activations 1.8 GB per step)",
            "flops_per_step_per_gpu": flops, "algorithmic_bytes_per_step_per_gpu": nbytes,
            "memory_plan": f"{args.strategy} ({model.lowered.arena_bytes / 1e9:.2f} GB arena)",
            "upload_slices": model.slices,
        },
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": int(pinned_in.nbytes),
                "d2h_bytes_per_step": int(pinned_out.nbytes)},
        "gpu_launches": model.launch_count * args.steps,
        "roofline": {
            "bound": "tensor", "achieved": round(achieved, 3), "peak": round(tf32_peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / tf32_peak, 4), "traffic": measured_traffic(args.batch),
            "traffic_note": "DRAM read+write bytes of the 54 GEMM launches of one step (ncu, batch 32, "
                            "scaled by the batch; profiles/resnet50_step_launches.md)",
            "kernel": "implicit-GEMM conv/GEMM launches (54 per step)",
            "peak_note": f"dense TF32 = half the {pk['source']} bf16 cuBLAS rate",
            "gemm_share_of_step": round(gemm_s / total_prof, 4) if total_prof else None,
            "gemm_launches": launches,
        },
        "step_roofline": {"bound_ms": round(step_bound_s * 1e3, 4), "frac": round(step_bound_s * 1e3 / ms_per_step, 4),
                          "note": "max(FLOPs / TF32 peak, algorithmic bytes / HBM peak) / measured step"},
        "clocks": clocks.summary(),
    }
    model.close()

    if rank == 0 and world == 1 and not args.no_latency:
        g1 = build_r50(1)
        m1 = compile_graph(g1, precision=args.precision, device=local)
        x1 = np.random.default_rng(0).standard_normal((1, 3, 224, 224)).astype(np.float32)
        for _ in range(10):
            m1.run({"image": x1})
        ts = []
        for _ in range(100):
            t0 = time.perf_counter()
            m1.run({"image": x1})
            ts.append(time.perf_counter() - t0)
        s1 = torch.cuda.ExternalStream(m1.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dts = []
        for _ in range(50):
            e0.record(s1)
            m1.run_device(sync=False)
            e1.record(s1)
            e1.synchronize()
            dts.append(e0.elapsed_time(e1))
        line["latency_b1"] = {"p50_ms": round(statistics.median(ts) * 1e3, 4),
                              "device_p50_ms": round(statistics.median(dts), 4), "unit": "ms"}
        m1.close()

    if rank == 0 and world == 1 and not args.no_bert:
        line["bert"] = bert_throughput(args.precision, local, steps=20, warmup=3)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_reference_run(args.cpu_batch, 5, 1)
            line["cpu_baseline"] = {"value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "reference",
                                    "sample": f"reference C backend (gcc+OpenMP), ResNet-50 O3 batch {args.cpu_batch}, "
                                              "p50 of 5 runs"}
        except Exception as exc:
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                                    "sample": f"failed: {type(exc).__name__}: {exc}"[:200]}
    if rank == 0:
        print(json.dumps(line))
    group.close()


if __name__ == "__main__":
    main()
