"""Benchmark of the `cuda` target on its headline workload: ResNet-50 (BASELINE configs 0 and 4).

Default arm (our backend), one process per GPU (``torchrun`` for N > 1, batch-sharded replicas,
no collective on the data path):

* ``value``: whole-job img/s of the compiled ResNet-50 (O3 graph on the reference planner's
  default memory plan, CUDA Graph replay) at ``--batch`` images per GPU (weak scaling), inputs
  resident in HBM, timed with CUDA events on the model's stream over ``--steps`` replays after
  ``--warmup`` untimed ones, max over ranks;
* ``e2e``: the same through the public API ``CudaCompiledModel.run`` from pinned host memory
  (host->device input copy, replay, device->host logits copy every step; the input is uploaded
  in four slices whose copies overlap the first layers of the earlier slices);
* ``roofline``: the dominant kernel family (the implicit-GEMM convolution / GEMM launches) from
  one eagerly launched pass with CUDA events around every launch, against MEASURED_PEAKS.json;
* ``fixed_total_batch``: BASELINE config 4 as a fixed total batch (256 and 1024 images) sharded
  over the N GPUs (strong scaling), whole-job img/s;
* at N = 1 also: the naive memory plan, strict (3xTF32) mode, batch-1 latency, and the other
  BASELINE configs (MobileNetV2 b128, BERT-base b32 and b1, GPT-2 b16);
* ``cpu_baseline``: the reference's own C backend (gcc + OpenMP, every host thread) on a bounded
  sample of the workload.

``--impl reference`` runs the reference's C backend (the unmodified reference, installed in
baseline/_ref, through its public ``compile_graph`` API) on the same workload on the host CPU,
every host thread, on rank 0 only.
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


def measured_traffic(batch: int) -> tuple[int | None, str]:
    """DRAM bytes (read + write) of one step's GEMM launches from the committed ncu summary:
    per-form captures at batch 256 summed over the step's launches
    (profiles/resnet50_b256_gemm_traffic.md), scaled to `batch` when that differs; else None."""
    f = ROOT / "profiles" / "resnet50_b256_gemm_traffic.md"
    if f.exists():
        for line in f.read_text().splitlines():
            if line.startswith("traffic_bytes_per_step_b256:"):
                v = int(line.split(":")[1])
                note = "ncu at batch 256" + ("" if batch == 256 else f", scaled to batch {batch}")
                return int(v * batch / 256), note
    return None, "no batch-256 capture committed"


def prepared(name: str, **kw):
    """A benchmark model (mgc_cuda.zoo: the BASELINE configs built in the reference IR with
    seeded random-init weights) through the reference's O3 pipeline and scheduler."""
    from mgc_cuda import zoo
    from ml_graph_compiler.passes import optimize
    from ml_graph_compiler.schedule import schedule

    g = zoo.MODELS[name](**kw)
    optimize(g, "O3")
    schedule(g)
    return g


def build_r50(batch: int):
    """ResNet-50 v1.5 (BASELINE configs 0 and 4): weights of config 0 (seed 0)."""
    return prepared("resnet50", batch=batch, seed=0)


def host_threads() -> int:
    """Host threads this process may run on (the CPU affinity, not the machine's core count)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def pinned_like(a: np.ndarray) -> np.ndarray:
    """A page-locked host copy of `a` (asynchronous host<->device copies)."""
    import torch

    buf = torch.empty(a.shape, dtype=torch.from_numpy(np.ascontiguousarray(a[:0])).dtype, pin_memory=True).numpy()
    buf[...] = a
    return buf


def device_ms(model, steps: int, warmup: int, group=None, clocks=None) -> float:
    """Milliseconds per replay of the model's CUDA Graph with its inputs resident, CUDA events on
    the model's stream, `warmup` untimed replays first; with a replica group, a barrier on both
    sides and the max over ranks."""
    import torch

    stream = torch.cuda.ExternalStream(model.stream)
    for _ in range(warmup):
        model.run_device(sync=False)
    if group is not None:
        group.barrier()
    else:
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks is not None:
        clocks.__enter__()
    e0.record(stream)
    for _ in range(steps):
        model.run_device(sync=False)
    e1.record(stream)
    e1.synchronize()
    if clocks is not None:
        clocks.__exit__(None, None, None)
    ms = e0.elapsed_time(e1)
    if group is not None:
        group.barrier()
        ms = group.max(ms)
    return ms / steps


def e2e_s(model, feeds: dict, steps: int, group=None) -> tuple[float, int, int]:
    """(seconds per call, H2D bytes, D2H bytes) of ``run`` from pinned host buffers: every call
    copies the inputs in, replays the graph and copies every output back."""
    pinned_in = {k: pinned_like(np.asarray(v)) for k, v in feeds.items()}
    outs = model.run(pinned_in)
    pinned_out = {k: pinned_like(v) for k, v in outs.items()}
    for _ in range(2):
        model.run(pinned_in, out=pinned_out)
    if group is not None:
        group.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        model.run(pinned_in, out=pinned_out)
    dt = time.perf_counter() - t0
    if group is not None:
        dt = group.max(dt)
    return (dt / steps, int(sum(a.nbytes for a in pinned_in.values())),
            int(sum(a.nbytes for a in pinned_out.values())))


def measure(name: str, kw: dict, units: int, unit: str, precision: str, device: int, steps: int, warmup: int,
            strategy: str = "greedy_by_size", seed: int = 0, e2e: bool = True, group=None) -> dict:
    """Device-timed throughput (and, with `e2e`, through ``run`` from pinned host buffers) of one
    benchmark model; `units` images or sequences per replay."""
    from mgc_cuda import zoo
    from mgc_cuda.runtime import compile_graph

    g = prepared(name, **kw)
    m = compile_graph(g, precision=precision, device=device, strategy=strategy)
    try:
        feeds = zoo.feeds(g, seed)
        m.run(feeds)  # inputs resident for the device-timed replays
        ms = device_ms(m, steps, warmup, group)
        world = group.world if group is not None else 1
        out = {"value": round(world * units / (ms / 1e3), 2), "unit": unit, "ms_per_step": round(ms, 4),
               "steps": steps, "warmup": warmup, "precision": precision, "memory_plan": strategy,
               "gpu_launches_per_step": m.launch_count}
        if e2e:
            s, hi, ho = e2e_s(m, feeds, steps, group)
            out["e2e"] = {"value": round(world * units / s, 2), "unit": unit, "h2d_bytes_per_step": hi,
                          "d2h_bytes_per_step": ho}
        return out
    finally:
        m.close()


def latency(name: str, kw: dict, precision: str, device: int, seed: int) -> dict:
    """Batch-1 p50 latency: through ``run`` (host buffers, wall clock) and device-only replays."""
    import torch

    from mgc_cuda import zoo
    from mgc_cuda.runtime import compile_graph

    g = prepared(name, **kw)
    m = compile_graph(g, precision=precision, device=device)
    try:
        feeds = zoo.feeds(g, seed)
        for _ in range(10):
            m.run(feeds)
        ts = []
        for _ in range(100):
            t0 = time.perf_counter()
            m.run(feeds)
            ts.append(time.perf_counter() - t0)
        s1 = torch.cuda.ExternalStream(m.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dts = []
        for _ in range(50):
            e0.record(s1)
            m.run_device(sync=False)
            e1.record(s1)
            e1.synchronize()
            dts.append(e0.elapsed_time(e1))
        return {"p50_ms": round(statistics.median(ts) * 1e3, 4), "device_p50_ms": round(statistics.median(dts), 4),
                "unit": "ms", "precision": precision}
    finally:
        m.close()


def cpu_reference_run(batch: int, steps: int, warmup: int) -> dict:
    """The reference C backend on this host: compile_graph(O3 graph) with gcc + OpenMP on every
    host thread this process may use (set explicitly: torchrun exports OMP_NUM_THREADS=1)."""
    os.environ.setdefault("MGC_CC", "/usr/bin/gcc")
    from mgc_cuda import _reference  # noqa: F401  (the unmodified reference, baseline/_ref)
    from ml_graph_compiler.codegen import compile_graph as c_compile

    g = build_r50(batch)
    x = np.random.default_rng(4).standard_normal((batch, 3, 224, 224)).astype(np.float32)
    threads = host_threads()
    with tempfile.TemporaryDirectory() as tmp:
        model = c_compile(g, cache_dir=tmp)
        model.set_threads(threads)
        times = model.benchmark({"image": x}, warmup=warmup, repeat=steps)
        used = model.max_threads()
        openmp = model.openmp
    p50 = statistics.median(times)
    return {"value": batch / p50, "p50_s": p50, "cores": used, "openmp": openmp, "batch": batch, "times": times}


def headline_config(batch: int, world: int) -> dict:
    """The workload of the headline line, identical in both arms (each arm's arithmetic is in
    its ``details``)."""
    return {"workload": f"resnet50 v1.5 O3 (BASELINE config 4), batch {batch} per GPU, fp32 tensors",
            "batch_per_gpu": batch, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (input 154 MB, activations 1.8 GB per step at batch 256)"}


def run_reference_arm(args: argparse.Namespace) -> None:
    """The reference's own implementation of the path (its C backend, the CPU) on the same
    workload: every timed step runs the whole per-GPU batch. Rank 0 only; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        r = cpu_reference_run(args.batch, args.steps, args.warmup)
    except Exception as exc:  # the reference could not be built or run on this host
        print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
        return
    sample = (f"reference C backend (gcc + OpenMP, {r['cores']} threads, {cpu_model()}), ResNet-50 O3 batch "
              f"{args.batch}, p50 of {args.steps} runs after {args.warmup} warm-up runs")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["p50_s"] * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(args.batch, args.gpus),
        "details": {"precision": "fp32 (C backend)", "threads": r["cores"], "cpu": cpu_model()},
        "cpu_baseline": {"value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "reference",
                         "sample": sample, "cpu": cpu_model(), "openmp": r["openmp"]},
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
    ap.add_argument("--cpu-batch", type=int, default=64, help="images of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the headline line: no other configs or modes")
    ap.add_argument("--strategy", default="greedy_by_size", choices=["greedy_by_size", "first_fit", "naive"],
                    help="the reference planner's memory strategy for the headline model (its default, "
                         "greedy_by_size, as the cuda target's north star asks; the naive plan is measured beside it)")
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
    model.run({"image": x})  # resident input for the device-timed loop
    clocks = Clocks(local)
    ms_per_step = device_ms(model, args.steps, args.warmup, group, clocks)
    value = world * args.batch / (ms_per_step / 1e3)
    e2e_step, h2d, d2h = e2e_s(model, {"image": x}, args.steps, group)
    e2e = world * args.batch / e2e_step

    # dominant kernel family: per-launch CUDA events (eager pass), GEMM-family nodes
    prof_runs = 3
    per_node = [0.0] * len(g.nodes)
    for _ in range(prof_runs):
        for i, (_, _, s) in enumerate(model.profile()):
            per_node[i] += s / prof_runs
    gemm_nodes = [i for i, n in enumerate(g.nodes) if n.op in ("FusedConv", "FusedGemm", "Conv", "Gemm", "MatMul")]
    gemm_s = sum(per_node[i] for i in gemm_nodes)
    gemm_flops = sum(ops.flops(g.nodes[i]) for i in gemm_nodes)
    paths = model.gemm_paths()
    tf32_peak = pk["bf16_tflops"] / 2.0
    achieved = gemm_flops / gemm_s / 1e12 if gemm_s > 0 else 0.0
    step_bound_s = max(flops / (tf32_peak * 1e12), nbytes / (pk["hbm_gbs"] * 1e9))
    total_prof = sum(per_node)
    traffic, traffic_src = measured_traffic(args.batch)

    line: dict = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(args.batch, world),
        "details": {
            "precision": args.precision,
            "memory_plan": f"{args.strategy} ({model.lowered.arena_bytes / 1e9:.2f} GB arena)",
            "upload_slices": model.slices, "flops_per_step_per_gpu": flops,
            "algorithmic_bytes_per_step_per_gpu": nbytes,
            "gemm_records": {"tcgen05": sum(1 for p in paths if p[3] == "tcgen05"),
                             "simt": sum(1 for p in paths if p[3] == "simt")},
        },
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": model.launch_count * args.steps,
        "roofline": {
            "bound": "tensor", "achieved": round(achieved, 3), "peak": round(tf32_peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / tf32_peak, 4),
            "traffic": traffic,
            "traffic_note": f"DRAM read + write bytes of one step's GEMM launches, the unit `achieved` is "
                            f"measured over ({traffic_src}; profiles/resnet50_b256_gemm_traffic.md)",
            "kernel": "implicit-GEMM conv/GEMM launches (umma_gemm_kernel forms)",
            "peak_note": f"dense TF32 = half the {pk['source']} bf16 cuBLAS burst rate (of {pk['source']})",
            "gemm_share_of_step": round(gemm_s / total_prof, 4) if total_prof else None,
            "gemm_launches": len(gemm_nodes),
        },
        "step_roofline": {"bound_ms": round(step_bound_s * 1e3, 4), "frac": round(step_bound_s * 1e3 / ms_per_step, 4),
                          "note": "max(FLOPs / TF32 peak, algorithmic bytes / HBM peak) / measured step"},
        "clocks": clocks.summary(),
    }
    model.close()
    del model

    # BASELINE config 4 as a fixed total batch sharded over the GPUs (strong scaling): every rank
    # runs total / N images per step
    fixed: dict = {}
    for total in (256, 1024):
        if total % world:
            continue
        if total == args.batch * world and args.strategy == "greedy_by_size":
            fixed[f"b{total}"] = {"value": round(value, 2), "ms_per_step": round(ms_per_step, 4), "per_gpu": args.batch,
                                  "e2e": line["e2e"]["value"]}
            continue
        r = measure("resnet50", {"batch": total // world, "seed": 0}, total // world, UNIT, args.precision, local,
                    min(args.steps, 20), 3, seed=4 + rank, e2e=True, group=group)
        fixed[f"b{total}"] = {"value": r["value"], "ms_per_step": r["ms_per_step"], "per_gpu": total // world,
                              "e2e": r["e2e"]["value"]}
    line["fixed_total_batch"] = {**fixed, "unit": UNIT, "scaling": "strong",
                                 "note": "whole-job img/s with the total batch split over the GPUs"}

    extras = rank == 0 and world == 1 and not args.no_extras
    if extras:
        steps = min(args.steps, 20)
        other = "naive" if args.strategy != "naive" else "greedy_by_size"
        r = measure("resnet50", {"batch": args.batch, "seed": 0}, args.batch, UNIT, args.precision, local, steps, 3,
                    strategy=other, seed=4)
        line[f"{other}_plan"] = r
        line["strict"] = {
            "resnet50_b256": measure("resnet50", {"batch": 256, "seed": 0}, 256, UNIT, "strict", local, steps, 3,
                                     seed=4, e2e=False),
            "latency_b1": latency("resnet50", {"batch": 1, "seed": 0}, "strict", local, 0),
            "bert_b32": measure("bert", {"batch": 32, "seq": 128, "seed": 2}, 32, "seq/s", "strict", local, steps, 3,
                                strategy="naive", seed=2, e2e=False),
        }
        line["latency_b1"] = latency("resnet50", {"batch": 1, "seed": 0}, args.precision, local, 0)
        line["configs"] = {
            "mobilenet_v2_b1": latency("mobilenet_v2", {"batch": 1, "seed": 1}, args.precision, local, 1),
            "mobilenet_v2_b128": measure("mobilenet_v2", {"batch": 128, "seed": 1}, 128, UNIT, args.precision, local,
                                         steps, 3, seed=1),
            "bert_b1": measure("bert", {"batch": 1, "seq": 128, "seed": 2}, 1, "seq/s", args.precision, local, steps,
                               3, seed=2),
            "bert_b32": measure("bert", {"batch": 32, "seq": 128, "seed": 2}, 32, "seq/s", args.precision, local, steps,
                                3, strategy="naive", seed=2),
            "gpt2_b1": latency("gpt2", {"batch": 1, "seq": 128, "seed": 3}, args.precision, local, 3),
            "gpt2_b16": measure("gpt2", {"batch": 16, "seq": 128, "seed": 3}, 16, "seq/s", args.precision, local,
                                steps, 3, seed=3),
        }
        line["bert"] = {"metric": "BERT-base seq128 seq/s (batch 32, O3 graph)", **line["configs"]["bert_b32"]}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_reference_run(args.cpu_batch, 3, 1)
            line["cpu_baseline"] = {
                "value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "reference",
                "sample": f"reference C backend (gcc + OpenMP), ResNet-50 O3 batch {args.cpu_batch} of the "
                          f"{args.batch}-image workload, p50 of 3 runs", "cpu": cpu_model()}
        except Exception as exc:
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": host_threads(), "kind": "reference",
                                    "sample": f"failed: {type(exc).__name__}: {exc}"[:200]}
    if rank == 0:
        print(json.dumps(line))
    group.close()


if __name__ == "__main__":
    main()
