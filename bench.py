#!/usr/bin/env python3
"""Benchmark of the B200 inference-kernel path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the configuration the metric is quoted on): the BF16 GEMM shape sweep
C[M,N] = A[M,K] * B[N,K]^T with M in {1,16,128,1024,8192} crossed with
(N,K) in {(4096,4096),(14336,4096),(4096,14336),(6144,4096)}, A ~ N(0,1), B ~ N(0,0.02),
bf16 in/out, fp32 accumulation.  One step = one pass over the 20 GEMMs.  At N GPUs the
weights are column-sharded (each rank owns N/G rows of every B and computes that slice of
C; no collective), so the total work is fixed: strong scaling.

Prints ONE JSON line (rank 0).  `value` is TFLOP/s of the whole job with operands resident
in HBM; `e2e` is the same metric through the drop-in ModelNew.forward with host buffers
(H2D of A and B and D2H of C inside the timed region); `roofline` describes the dominant
kernel (the tensor-core GEMM of the M >= 1024 shapes), timed live with CUDA events around
each of its launches; `cpu_baseline` is the CPU oracle (the reference's PyTorch path) on a
bounded number of passes over the same 20 shapes on this machine's host cores.

`ops` holds one record per operator configuration of the metric (GEMM 4096^3, the two
flash-attention shapes, the Mixtral-like MoE, the fine-grained MoE at 1/64/512/8192 tokens):
device time per call under CUDA-graph replay with the L2 flushed between calls, TFLOP/s or
GB/s, and the roofline fraction of the operator and of its dominant kernel.  With N > 1
GPUs `ops` holds what shards: attention over batch x KV heads (no collective) and the MoE
expert-parallel over the N GPUs (tokens/s of the whole job).

--impl reference times the CPU path alone over the same 20 shapes, on rank 0, as the
reference arm.
"""
from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

M_VALUES = (1, 16, 128, 1024, 8192)
NK_VALUES = ((4096, 4096), (14336, 4096), (4096, 14336), (6144, 4096))
SEED = 20260312
WORKLOAD = "gemm_bf16_shape_sweep (M in {1,16,128,1024,8192} x (N,K) in {(4096,4096),(14336,4096),(4096,14336),(6144,4096)})"
METRIC = "BF16 TFLOP/s per op (GEMM, FA fwd, fused MoE) and % of B200 dense peak"
CPU_SECONDS = 15.0  # CPU work spent on the baseline passes
DENSE_M = 1024  # shapes with M >= DENSE_M run the tensor-core-bound kernel


def sweep_shapes():
    return [(m, n, k) for m in M_VALUES for (n, k) in NK_VALUES]


def flops(shapes) -> float:
    return float(sum(2.0 * m * n * k for (m, n, k) in shapes))


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi during the timed region (reads only; changes no setting)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._pump, daemon=True)
        self.thread.start()

    def _pump(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()  # the exact process started above
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        # "under load" = samples drawing at least half of the highest power seen
        top = max(power) if power else 0.0
        loaded = [c for c, w in zip(sm, power) if w >= 0.5 * top] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "power_w_max": top or None,
                "samples": len(sm), "samples_under_load": len(loaded), "reasons": sorted(reasons)}


# --------------------------------------------------------------------------- CPU arm
def sweep_config(world: int) -> dict:
    """The `config` object of the JSON line: the same for both arms, so that their values
    are rates over the same work."""
    return {
        "workload": WORKLOAD, "shapes": len(sweep_shapes()), "flop_per_step": flops(sweep_shapes()),
        "parallelism": f"column-sharded over N x{world}, no collective" if world > 1 else "one device",
        "l2": "inputs larger than L2: one step cycles through about 1.8 GB of operands and results",
        "seed": SEED,
    }


class CpuSweep:
    """The CPU oracle GEMM (the reference's torch.matmul(A, B.T) path with fp32
    accumulation) over all 20 shapes of the sweep; one pass = one step."""

    def __init__(self):
        import torch

        from oracle import gemm_oracle

        self.torch, self.oracle = torch, gemm_oracle
        g = torch.Generator().manual_seed(SEED)
        self.weights = {nk: (torch.randn(nk, generator=g) * 0.02).to(torch.bfloat16) for nk in NK_VALUES}
        self.acts = {(m, k): torch.randn((m, k), generator=g).to(torch.bfloat16)
                     for m in M_VALUES for k in (4096, 14336)}
        self.shapes = sweep_shapes()
        gemm_oracle.gemm_reference(self.acts[(16, 4096)], self.weights[(4096, 4096)])  # warm the thread pool

    def one_pass(self) -> float:
        t0 = time.perf_counter()
        for (m, n, k) in self.shapes:
            self.oracle.gemm_reference(self.acts[(m, k)], self.weights[(n, k)])
        return time.perf_counter() - t0


def time_cpu_sweep(max_seconds: float):
    """Passes over the 20 shapes until `max_seconds` of CPU work have run (at least one);
    returns (TFLOP/s of the best pass, its seconds, threads, passes)."""
    import torch

    sweep = CpuSweep()
    best, total, passes = None, 0.0, 0
    while passes == 0 or (total < max_seconds and passes < 50):
        dt = sweep.one_pass()
        best = dt if best is None else min(best, dt)
        total += dt
        passes += 1
    return flops(sweep.shapes) / best / 1e12, best, torch.get_num_threads(), passes


def host_cores() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    # torchrun exports OMP_NUM_THREADS=1 to its workers; the CPU arm uses every core it may
    torch.set_num_threads(host_cores())
    sweep = CpuSweep()
    times = []
    for i in range(args.warmup + args.steps):
        dt = sweep.one_pass()
        if i >= args.warmup:
            times.append(dt)
    mean = sum(times) / len(times)
    tf = flops(sweep.shapes) / mean / 1e12
    threads = torch.get_num_threads()
    sample = ("each step = one pass over all 20 shapes of the sweep (the b200 arm's step), CPU oracle: "
              "torch fp32 matmul of the bf16 operands")
    line = {
        "impl": "reference", "metric": METRIC, "value": tf, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": sweep_config(args.gpus),
        "cpu_baseline": {"value": tf, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tf, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- per-operator records
def measure_ops(args, pkg, dist, dev, rank, world, peaks) -> dict:
    """The `ops` object of the JSON line.  One GPU: every operator configuration of the
    metric.  Several GPUs: what shards -- attention over batch x KV heads with no collective,
    the MoE expert-parallel with this library's peer-memory dispatch and return."""
    import torch

    steps = max(3, min(args.steps, 10))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    ops: dict = {}
    if world == 1:
        builder = CaseBuilder(pkg, dev)
        for name in OPS_CASES:
            c = builder.build(name)
            ms, ms_min = time_replays(torch, c["call"], steps, 3, flush)
            rec = op_record(c, ms, ms_min, peaks, steps)
            add_stage_roofline(rec, c, peaks)
            ops[name] = rec
            del c
        del builder
        torch.cuda.empty_cache()
        return ops

    # ---- attention shards: each rank runs the kernel on its own (batch, KV-head) rectangle
    for name, (B, S, Hq, Hkv, causal) in (("c3a", (8, 4096, 32, 8, True)), ("c3b", (2, 16384, 16, 16, False))):
        try:
            sh = pkg.sharding.attention_shard(B, Hkv, world, rank)
        except ValueError as err:
            ops[f"{name}_sharded"] = {"skipped": str(err)}
            continue
        Bl, Hkl = sh.b1 - sh.b0, sh.hk1 - sh.hk0
        Hql = Hkl * (Hq // Hkv)
        g = torch.Generator(device=dev).manual_seed(SEED + rank)
        mk = lambda h: torch.randn((Bl, S, h, 128), device=dev, dtype=torch.float32, generator=g).to(torch.bfloat16)  # noqa: E731
        q, k, v = mk(Hql), mk(Hkl), mk(Hkl)
        out = torch.empty_like(q)
        ms, ms_min = time_replays(torch, lambda: pkg.flash_attn(q, k, v, causal=causal, out=out), steps, 3, flush)
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        fl = 2.0 * B * Hq * S * (S + 1) * 128 if causal else 4.0 * B * Hq * S * S * 128
        ops[f"{name}_sharded"] = {
            "case": f"fa:{B}x{S}x{Hq}x{Hkv}x{'causal' if causal else 'full'}", "n_gpus": world, "ms": ms,
            "tflops": fl / ms / 1e9, "frac_of_n_gpu_peak": fl / ms / 1e9 / (world * peaks["bf16_tflops"]),
            "parallelism": f"batch x KV-head rectangles, {Bl} x {Hkl} per rank, no collective",
            "timing": "CUDA graph replay per rank, L2 flushed, max over ranks of the median"}
        del q, k, v, out
    torch.cuda.empty_cache()
    # ---- expert-parallel MoE
    for dims in ("c4", "c5_t8192", "c5_t512", "c5_t64"):
        T, _, _, E, _ = (int(x) for x in EP_PRESETS[dims].split("x"))
        if T % world or E % world:
            continue
        # A failure on one rank (a barrier wait that ran out, a capture that failed) must not
        # leave the others waiting in a collective: every rank records its outcome, then all
        # ranks agree on it.
        try:
            rec = measure_ep(pkg, dist, dev, rank, world, dims, steps=steps, warmup=3, graph=not args.ep_eager)
            failed = 0
        except Exception as exc:  # noqa: BLE001 - reported in the record
            rec = {"case": f"ep:{dims}", "n_gpus": world, "error": f"{type(exc).__name__}: {exc}"[:300]}
            failed = 1
        torch.cuda.synchronize()
        flag = torch.tensor([failed], device=dev, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if int(flag.item()) and "error" not in rec:
            rec = {"case": f"ep:{dims}", "n_gpus": world, "error": "another rank failed during this case"}
        if int(flag.item()):
            pkg.clear_status()
        ops[f"moe_ep_{dims}"] = rec
        torch.cuda.empty_cache()
    return ops


# --------------------------------------------------------------------------- GPU arm
def run_b200_arm(args) -> None:
    import torch

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device: the B200 path has no CPU fallback")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        # NCCL prints its version banner on stdout when NCCL_DEBUG is VERSION or WARN;
        # stdout carries the one JSON line only
        if os.environ.get("NCCL_DEBUG", "").upper() in ("VERSION", "WARN"):
            del os.environ["NCCL_DEBUG"]
        import torch.distributed as dist_mod

        dist = dist_mod
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=240))

    import __graft_entry__ as entry

    if rank == 0:
        entry.build()
    if dist is not None:
        dist.barrier()
    pkg = importlib.import_module(entry.PACKAGE_NAME)
    pkg._cabi.load()
    from importlib import util as _util

    spec = _util.spec_from_file_location(
        "b200_gemm_model", REPO / entry.PACKAGE_NAME / "datasets" / "inference" / "gemm" / "b200" / "model.py")
    gemm_model = _util.module_from_spec(spec)
    spec.loader.exec_module(gemm_model)
    model = gemm_model.ModelNew()
    gemm = pkg.gemm_pipeline_transposed_b
    pkg.clear_status()

    # ---- synthetic operands, resident in HBM; this rank's column shard of every B ----
    shapes = sweep_shapes()
    g = torch.Generator(device=dev).manual_seed(SEED)
    acts = {(m, k): torch.randn((m, k), device=dev, dtype=torch.float32, generator=g).to(torch.bfloat16)
            for m in M_VALUES for k in (4096, 14336)}
    weights = {}
    for (n, k) in NK_VALUES:
        n_local = n // world
        if n_local * world != n:
            raise RuntimeError(f"N={n} does not split over {world} GPUs")
        w = (torch.randn((n, k), device=dev, dtype=torch.float32, generator=g) * 0.02).to(torch.bfloat16)
        weights[(n, k)] = w[rank * n_local:(rank + 1) * n_local].contiguous()
        del w
    outs = {(m, n, k): torch.empty((m, n // world), device=dev, dtype=torch.bfloat16) for (m, n, k) in shapes}
    footprint = sum(t.numel() * 2 for d in (acts, weights, outs) for t in d.values())

    def step(record=None):
        for (m, n, k) in shapes:
            if record is not None and m >= DENSE_M:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                gemm(acts[(m, k)], weights[(n, k)], outs[(m, n, k)])
                e1.record()
                record.append((e0, e1))
            else:
                gemm(acts[(m, k)], weights[(n, k)], outs[(m, n, k)])

    def sync_all():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step()
    sync_all()

    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.25)

    # one step = one replay of a CUDA graph holding the 20 launches (the reference's own
    # timer replays captured graphs too: scripts/benchmark/cudagraph_timer.py:33-55)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    sync_all()

    # ---- timed region: exactly K steps, device-timed, max over ranks ----
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sync_all()
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    sync_all()
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    total_flops = flops(shapes)  # whole job: all ranks' column shards together
    value = total_flops / (ms_per_step * 1e-3) / 1e12

    # ---- the same K steps launched eagerly with a CUDA-event pair around every launch of
    #      the dominant kernel (events cannot be read back from inside a graph replay) ----
    dense_events: list = []
    for _ in range(args.steps):
        step(dense_events)
    sync_all()

    # dominant kernel: the persistent tcgen05 GEMM of the M >= 1024 shapes
    dense_shapes = [s for s in shapes if s[0] >= DENSE_M]
    dense_ms = sum(e0.elapsed_time(e1) for (e0, e1) in dense_events)
    dense_launches = len(dense_events)
    dense_flops_local = flops(dense_shapes) / world * args.steps
    achieved = dense_flops_local / (dense_ms * 1e-3) / 1e12
    peaks = load_peaks()

    # ---- end to end through the drop-in ModelNew.forward with host buffers ----
    # Every step uploads each of its 14 distinct inputs (10 activation matrices, 4 weight
    # shards) once from pinned host memory, runs the 20 GEMMs through ModelNew.forward as
    # their operands land, and reads all 20 results back.  Upload, compute and read-back run
    # on three streams so that the two DMA directions and the GEMMs overlap.
    host_a = {key: t_.cpu().pin_memory() for key, t_ in acts.items()}
    host_b = {key: t_.cpu().pin_memory() for key, t_ in weights.items()}
    host_c = {key: torch.empty(t_.shape, dtype=t_.dtype).pin_memory() for key, t_ in outs.items()}
    dev_a = {key: torch.empty_like(t_, device=dev) for key, t_ in host_a.items()}
    dev_b = {key: torch.empty_like(t_, device=dev) for key, t_ in host_b.items()}
    h2d = sum(t_.numel() * 2 for t_ in host_a.values()) + sum(t_.numel() * 2 for t_ in host_b.values())
    d2h = sum(host_c[s].numel() * 2 for s in shapes)
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream(dev)
    # upload order = order of first use by the sweep
    upload_order = []
    for (m, n, k) in shapes:
        for item in (("a", (m, k)), ("b", (n, k))):
            if item not in upload_order:
                upload_order.append(item)

    def e2e_step():
        ready = {}
        up.wait_stream(main)       # the previous step's GEMMs have finished with the device inputs
        with torch.cuda.stream(up):
            for kind, key in upload_order:
                (dev_a if kind == "a" else dev_b)[key].copy_((host_a if kind == "a" else host_b)[key],
                                                             non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(up)
                ready[(kind, key)] = ev
        for (m, n, k) in shapes:
            main.wait_event(ready[("a", (m, k))])
            main.wait_event(ready[("b", (n, k))])
            c = model(dev_a[(m, k)], dev_b[(n, k)])
            done = torch.cuda.Event()
            done.record(main)
            down.wait_event(done)
            with torch.cuda.stream(down):
                host_c[(m, n, k)].copy_(c, non_blocking=True)
                c.record_stream(down)
        main.wait_stream(down)     # the step ends when its last result is on the host

    e2e_steps = max(1, min(args.steps, 5))
    e2e_step()
    sync_all()
    start.record()
    for _ in range(e2e_steps):
        e2e_step()
    end.record()
    sync_all()
    t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e2e_steps
    e2e_value = total_flops / (e2e_ms * 1e-3) / 1e12

    # free the sweep's operands before the per-operator cases
    del host_a, host_b, host_c, dev_a, dev_b, graph
    acts.clear()
    weights.clear()
    outs.clear()
    torch.cuda.empty_cache()

    ops = {} if args.no_ops else measure_ops(args, pkg, dist, dev, rank, world, peaks)

    clocks = sampler.stop() if sampler else None
    status = pkg.device_status()
    if status != 0:
        raise RuntimeError(f"device status word is {status:#x}: a kernel wait gave up")

    if rank == 0:
        cpu_tf, cpu_s, cpu_threads, cpu_passes = (None, None, None, 0)
        if world == 1:
            torch.set_num_threads(host_cores())
            cpu_tf, cpu_s, cpu_threads, cpu_passes = time_cpu_sweep(CPU_SECONDS)
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": sweep_config(world),
            "step": "one CUDA-graph replay of the 20 GEMM launches",
            "footprint_bytes_per_rank": footprint,
            "roofline": {
                "kernel": "gemm_bf16_pair_kernel<STAGES=6>, cta_group::2 256x256 tiles (M >= 1024 shapes)", "bound": "tensor",
                "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"], "peak_source": f"{peaks['source']} burst bf16 GEMM",
                "launches_timed": dense_launches, "avg_launch_ms": dense_ms / max(1, dense_launches),
                "timing": "CUDA events around each launch, K eager steps right after the graph-replayed timed region",
                "traffic": TRAFFIC_OVER_ALGORITHMIC * sum(
                    2.0 * (m * k + n * k / world + m * n / world) for (m, n, k) in dense_shapes) / len(dense_shapes),
                "traffic_note": "DRAM bytes per launch: ncu capture of gemm:4096x8192x4096 (216.2 MB measured vs "
                                "167.8 MB algorithmic) scaled by algorithmic bytes to the average dense launch",
            },
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms, "steps": e2e_steps,
                    "api": "datasets/inference/gemm/b200/model.py ModelNew.forward"},
            "gpu_launches": len(shapes) * args.steps,
            "clocks": clocks,
            "ops": ops,
        }
        if cpu_tf is not None:
            line["cpu_baseline"] = {
                "value": cpu_tf, "unit": "TFLOP/s", "cores": cpu_threads, "kind": "port",
                "sample": f"{cpu_passes} pass(es) over all 20 shapes of the sweep (the same step as the GPU arm), best pass {cpu_s:.2f} s",
            }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# --------------------------------------------------------------------------- single cases
CASE_PRESETS = {
    "c1": "gemm:4096x4096x4096", "c3a": "fa:8x4096x32x8xcausal", "c3b": "fa:2x16384x16x16xfull",
    "c4": "moe:4096x4096x14336x8x2xrouter", "c5_t1": "moe:1x7168x2048x256x8",
    "c5_t64": "moe:64x7168x2048x256x8", "c5_t512": "moe:512x7168x2048x256x8",
    "c5_t8192": "moe:8192x7168x2048x256x8",
}
CASE_PRESETS.update({"fp8_t64": "moe8:64x7168x2048x32x4", "fp8_t512": "moe8:512x7168x2048x32x4",
                     "bf16_t64": "moe:64x7168x2048x32x4", "bf16_t512": "moe:512x7168x2048x32x4"})
# the metric's five configurations, then the reference's own MoE format (fp8 codes + block scales,
# its table shape: 32 experts, top-4) beside the same shape in bf16
OPS_CASES = ("c1", "c3a", "c3b", "c4", "c5_t1", "c5_t64", "c5_t512", "c5_t8192",
             "bf16_t64", "bf16_t512", "fp8_t64", "fp8_t512")


class CaseBuilder:
    """Seeded device-resident inputs and a zero-argument call for one operator case
    (`gemm:MxNxK`, `fa:BxSxHqxHkvx{causal|full}`, `moe:TxHxIxExK[xrouter]` or a preset).
    Expert weights are cached per (E, H, I) so the fine-grained MoE's 21 GiB are drawn once."""

    def __init__(self, pkg, dev):
        import torch

        self.torch, self.pkg, self.dev = torch, pkg, dev
        self.g = torch.Generator(device=dev).manual_seed(SEED)
        self._weights: dict = {}

    def randn_bf16(self, shape, std=1.0):
        t = self.torch
        return (t.randn(shape, device=self.dev, dtype=t.float32, generator=self.g) * std).to(t.bfloat16)

    def expert_weights(self, E, H, I):
        key = (E, H, I)
        if key not in self._weights:
            t = self.torch
            self._weights.clear()  # one set at a time: the largest is 21 GiB
            w13 = t.empty((E, 2 * I, H), device=self.dev, dtype=t.bfloat16)
            w2 = t.empty((E, H, I), device=self.dev, dtype=t.bfloat16)
            for e in range(E):  # per expert: keeps the fp32 temporaries small
                w13[e] = self.randn_bf16((2 * I, H), 0.02)
                w2[e] = self.randn_bf16((H, I), 0.02)
            self._weights[key] = (w13, w2)
        return self._weights[key]

    def build(self, case: str) -> dict:
        t, pkg = self.torch, self.pkg
        case = CASE_PRESETS.get(case, case)
        kind, _, dims = case.partition(":")
        parts = dims.split("x")
        c = {"case": case, "kind": kind, "stages": None}
        if kind == "gemm":
            m, n, k = (int(x) for x in parts)
            a, b = self.randn_bf16((m, k)), self.randn_bf16((n, k), 0.02)
            out = t.empty((m, n), device=self.dev, dtype=t.bfloat16)
            c.update(call=lambda: pkg.gemm_pipeline_transposed_b(a, b, out), flop=2.0 * m * n * k,
                     bytes=2.0 * (m * k + n * k + m * n), launches=1,
                     bound="tensor" if m > 128 else "hbm",
                     kernel="gemm_bf16_pair_kernel<6,256>" if m > 128 else "gemm_bf16_kernel<swap, split-K>")
        elif kind == "fa":
            B, S, Hq, Hkv = (int(x) for x in parts[:4])
            causal = parts[4] == "causal"
            q, kk, v = self.randn_bf16((B, S, Hq, 128)), self.randn_bf16((B, S, Hkv, 128)), self.randn_bf16((B, S, Hkv, 128))
            out = t.empty_like(q)
            c.update(call=lambda: pkg.flash_attn(q, kk, v, causal=causal, out=out),
                     flop=2.0 * B * Hq * S * (S + 1) * 128 if causal else 4.0 * B * Hq * S * S * 128,
                     bytes=2.0 * B * S * 128 * (2 * Hq + 2 * Hkv), launches=1, bound="tensor",
                     kernel="fa_fwd_kernel",
                     flop_convention="true causal work 2*B*Hq*S*(S+1)*D" if causal else "4*B*Hq*S^2*D")
        elif kind == "moe":
            T, H, I, E, K = (int(x) for x in parts[:5])
            router = len(parts) > 5 and parts[5] == "router"
            x = self.randn_bf16((T, H))
            w13, w2 = self.expert_weights(E, H, I)
            w_router = self.randn_bf16((E, H), 0.02) if router else None
            logits = None if router else t.randn((T, E), device=self.dev, dtype=t.float32, generator=self.g)
            op = pkg.moe.FusedMoE(tokens=T, hidden=H, inter=I, experts=E, topk=K, device=self.dev)
            call = lambda: op.forward(x, w13, w2, w_router=w_router, logits=logits)  # noqa: E731
            call()
            t.cuda.synchronize()
            touched = int((op.routes.expert_counts > 0).sum().item())
            rows_per_expert = T * K / E
            c.update(call=call, flop=6.0 * T * K * H * I + (2.0 * T * H * E if router else 0.0),
                     bytes=3.0 * H * I * 2 * touched + 2.0 * T * H * 2, launches=8 if router else 7,
                     bound="tensor" if rows_per_expert >= 200 else "hbm", kernel="gemm_bf16_kernel<grouped, gated>",
                     tokens=T, experts_touched=touched,
                     stages=lambda: op.stage_times(x, w13, w2, w_router=w_router, logits=logits),
                     stage_work={"gemm_w13_silu": (4.0 * T * K * H * I, 2.0 * 2 * I * H * touched),
                                 "gemm_w2": (2.0 * T * K * H * I, 2.0 * H * I * touched)})
        elif kind == "moe8":
            # fp8 e4m3 codes + fp32 block scales with the harness' distributions
            # (scripts/benchmark/backend_moe.py:86-210), through the fp8 tensor-core kernels
            T, H, I, E, K = (int(x) for x in parts[:5])
            f8 = t.float8_e4m3fn
            rnd = lambda shape: t.randn(shape, device=self.dev, dtype=t.float32, generator=self.g)  # noqa: E731
            x_q = (rnd((T, H)) + 0.1).to(f8)
            x_s = (rnd((T, H // 128)) * 2e-2 + 1e-1).clamp_min_(1e-8)
            tv, ti = t.topk(rnd((T, E)), k=K, dim=-1)
            ids, wts = ti.to(t.int32).contiguous(), t.softmax(tv, dim=-1).contiguous()
            key = ("f8", E, H, I)
            if key not in self._weights:
                self._weights.clear()
                w13 = t.empty((E, 2 * I, H), device=self.dev, dtype=f8)
                w2 = t.empty((E, H, I), device=self.dev, dtype=f8)
                for e in range(E):
                    w13[e] = (rnd((2 * I, H)) * 8.0).to(f8)
                    w2[e] = (rnd((H, I)) * 8.0).to(f8)
                s13 = (rnd((E, (2 * I // 128) * (H // 128))) * 2e-3 + 1e-2).clamp_min_(1e-8)
                s2 = (rnd((E, (H // 128) * (I // 128))) * 2e-3 + 1e-2).clamp_min_(1e-8)
                self._weights[key] = (w13, s13, w2, s2)
            w13, s13, w2, s2 = self._weights[key]
            op = pkg.moe.FusedMoEFp8(tokens=T, hidden=H, inter=I, experts=E, topk=K, device=self.dev)
            call = lambda: op.forward_routed(x_q, x_s, ids, wts, w13, s13, w2, s2)  # noqa: E731
            call()
            t.cuda.synchronize()
            touched = int((op.routes.expert_counts > 0).sum().item())
            c.update(call=call, flop=6.0 * T * K * H * I, bytes=3.0 * H * I * touched + T * H + 2.0 * T * H,
                     launches=6, bound="hbm", kernel="moe_fp8_grouped_kernel (kind::f8f6f4)", tokens=T,
                     experts_touched=touched)
        else:
            raise SystemExit(f"unknown case {case!r}")
        return c


def time_replays(torch, call, steps: int, warmup: int, flush, eager: bool = False):
    """Median / minimum device time (ms) of `call`, captured in a CUDA graph and replayed
    (like the reference's timer, scripts/benchmark/cudagraph_timer.py:33-55), with a write
    larger than L2 between timed calls."""
    for _ in range(max(warmup, 1)):
        call()
    torch.cuda.synchronize()
    run = call
    if not eager:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            call()
        torch.cuda.synchronize()
        run = graph.replay
    times = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times), min(times)


def op_record(c: dict, ms: float, ms_min: float, peaks: dict, steps: int, eager: bool = False) -> dict:
    """One entry of `ops`: rates from the algorithmic work and the roofline that bounds it."""
    tf, gbs = c["flop"] / ms / 1e9, c["bytes"] / ms / 1e6
    tensor = c["bound"] == "tensor"
    achieved, peak = (tf, peaks["bf16_tflops"]) if tensor else (gbs, peaks["hbm_gbs"])
    rec = {
        "case": c["case"], "ms": ms, "ms_min": ms_min, "tflops": tf, "gbs": gbs,
        "algorithmic_flop": c["flop"], "algorithmic_bytes": c["bytes"], "launches_per_call": c["launches"],
        "steps": steps, "timing": "eager launches" if eager else "CUDA graph replay, 256 MB write between calls",
        "roofline": {"kernel": c["kernel"], "bound": c["bound"], "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s" if tensor else "GB/s", "frac": achieved / peak,
                     "of": f"{peaks['source']} peak", "scope": "whole operator (all its launches)"},
    }
    if "flop_convention" in c:
        rec["flop_convention"] = c["flop_convention"]
    if "tokens" in c:
        rec["tokens_per_s"] = c["tokens"] / ms * 1e3
        rec["experts_touched"] = c["experts_touched"]
    return rec


def add_stage_roofline(rec: dict, c: dict, peaks: dict) -> None:
    """MoE: the dominant kernel (the gated expert GEMM) timed alone with CUDA events."""
    if not c.get("stages"):
        return
    stages = c["stages"]()
    rec["stage_ms"] = stages
    tensor = c["bound"] == "tensor"
    for name, (fl, by) in c["stage_work"].items():
        ms = stages[name]
        achieved = fl / ms / 1e9 if tensor else by / ms / 1e6
        peak = peaks["bf16_tflops"] if tensor else peaks["hbm_gbs"]
        rec.setdefault("kernel_roofline", {})[name] = {
            "bound": c["bound"], "achieved": achieved, "peak": peak, "unit": "TFLOP/s" if tensor else "GB/s",
            "frac": achieved / peak, "avg_launch_ms": ms, "launches_timed": 5,
            "timing": "CUDA events around the launch, eager, median of 5"}


def run_case(args) -> None:
    """One operator case on one GPU, e.g. for profiling or for the per-configuration numbers:
         --case gemm:MxNxK | c1
         --case fa:BxSxHqxHkvx{causal|full} | c3a | c3b
         --case moe:TxHxIxExK[xrouter] | c4 | c5_t1 | c5_t64 | c5_t512 | c5_t8192
    Prints one JSON line with the device time per call (CUDA events, L2 flushed between calls)."""
    import torch

    import __graft_entry__ as entry

    entry.build()
    pkg = importlib.import_module(entry.PACKAGE_NAME)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    pkg.clear_status()
    peaks = load_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    c = CaseBuilder(pkg, dev).build(args.case)
    ms, ms_min = time_replays(torch, c["call"], args.steps, args.warmup, flush, eager=args.eager)
    line = op_record(c, ms, ms_min, peaks, args.steps, eager=args.eager)
    line["frac_tensor_peak"] = line["tflops"] / peaks["bf16_tflops"]
    line["frac_hbm_peak"] = line["gbs"] / peaks["hbm_gbs"]
    add_stage_roofline(line, c, peaks)
    line["status"] = pkg.device_status()
    print(json.dumps(line), flush=True)


EP_PRESETS = {"c4": "4096x4096x14336x8x2", "c5_t1": "1x7168x2048x256x8", "c5_t64": "64x7168x2048x256x8",
              "c5_t512": "512x7168x2048x256x8", "c5_t8192": "8192x7168x2048x256x8"}


def measure_ep(pkg, dist, dev, rank, world, dims: str, *, steps: int, warmup: int, transport: str = "peer",
               sync: str = "signals", graph: bool = True, fused_return: bool = False, phases: bool = False) -> dict:
    """Expert-parallel MoE forward over all ranks of the job: tokens T/G and experts E/G per
    rank.  Device time per forward = max over ranks (CUDA events around `steps` forwards).
    Every rank must call this; the record is meaningful on every rank."""
    import torch

    T, H, I, E, K = (int(x) for x in EP_PRESETS.get(dims, dims).split("x")[:5])
    if E % world or T % world:
        raise SystemExit(f"T={T}, E={E} do not split over {world} ranks")
    Tl, El = T // world, E // world
    g = torch.Generator(device=dev).manual_seed(SEED + rank)

    def randn_bf16(shape, std=1.0):
        return (torch.randn(shape, device=dev, dtype=torch.float32, generator=g) * std).to(torch.bfloat16)

    x = randn_bf16((Tl, H))
    logits = torch.randn((Tl, E), device=dev, dtype=torch.float32, generator=g)
    w13 = torch.empty((El, 2 * I, H), device=dev, dtype=torch.bfloat16)
    w2 = torch.empty((El, H, I), device=dev, dtype=torch.bfloat16)
    for e in range(El):
        w13[e] = randn_bf16((2 * I, H), 0.02)
        w2[e] = randn_bf16((H, I), 0.02)
    if transport == "peer":
        ep = pkg.moe_ep.PeerExpertParallelMoE(tokens_local=Tl, hidden=H, inter=I, experts=E, topk=K, device=dev,
                                              fused_return=fused_return, sync=sync)
    else:
        ops = pkg.moe_ep.CudaOps(dev, tokens_global=T, experts=E, topk=K)
        ep = pkg.moe_ep.ExpertParallelMoE(experts=E, topk=K, ops=ops)
    for _ in range(max(warmup, 2)):
        ep.forward(x, w13, w2, logits=logits)
    dist.barrier()
    torch.cuda.synchronize()
    # With the peer transport and signal barriers a forward contains no collective-library
    # call, so it replays as one CUDA graph.  (A graph holding NCCL collectives kept the
    # communicator from shutting down at exit: those forwards are launched eagerly.)
    run = lambda: ep.forward(x, w13, w2, logits=logits)  # noqa: E731
    timing = "eager launches"
    cuda_graph = None
    if graph:
        if transport != "peer" or sync != "signals":
            raise SystemExit("graph replay needs the peer transport with signal barriers")
        cuda_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cuda_graph):
            run()
        torch.cuda.synchronize()
        dist.barrier()
        run = cuda_graph.replay
        timing = "CUDA graph replay"
        run()
        torch.cuda.synchronize()
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    dist.barrier()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del run
    cuda_graph = None  # release the graph before the process group goes away
    torch.cuda.synchronize()
    fl = 6.0 * T * K * H * I
    rec = {"case": f"ep:{dims}", "n_gpus": world, "ms": ms, "tokens_per_s": T / ms * 1e3,
           "tflops": fl / ms / 1e9, "tokens": T, "experts": E, "topk": K, "steps": steps,
           "parallelism": f"expert-parallel x{world}, tokens {Tl}/rank, experts {El}/rank",
           "transport": ("dispatch/return kernels storing into peer memory over NVLink, no host read"
                         if transport == "peer" else
                         "NCCL all_to_all_single, one host read of the per-expert counts per forward"),
           "timing": timing + ", device time = max over ranks"}
    if phases:
        # phase breakdown of one more forward on this rank (events between the phases)
        marks: list = []
        ep.forward(x, w13, w2, logits=logits, marks=marks)
        torch.cuda.synchronize()
        rec["phase_ms_rank0"] = {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(marks, marks[1:])}
    del ep
    torch.cuda.synchronize()
    dist.barrier()
    return rec


def run_ep_case(args) -> None:
    """--case ep:TxHxIxExK or ep:c4 / ep:c5_tN under torchrun; rank 0 prints one JSON line."""
    import torch
    import torch.distributed as dist

    import __graft_entry__ as entry

    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if os.environ.get("NCCL_DEBUG", "").upper() in ("VERSION", "WARN"):
        del os.environ["NCCL_DEBUG"]  # its version banner goes to stdout, which carries the JSON line
    dist.init_process_group("nccl", device_id=dev)
    if rank == 0:
        entry.build()
    dist.barrier()
    pkg = importlib.import_module(entry.PACKAGE_NAME)
    pkg._cabi.load()
    pkg.clear_status()
    rec = measure_ep(pkg, dist, dev, rank, world, args.case.split(":", 1)[1], steps=args.steps,
                     warmup=args.warmup, transport=args.transport, sync=args.ep_sync, graph=args.ep_graph,
                     fused_return=args.fused_return, phases=True)
    rec["status"] = pkg.device_status()
    if rank == 0:
        print(json.dumps(rec), flush=True)
    dist.destroy_process_group()


# DRAM traffic of the dominant kernel relative to its algorithmic bytes, from the ncu capture
# summarised in profiles/gemm_pair_4096x8192x4096_ncu.md (168.5 MB read + 47.7 MB written
# against 2(MK+NK+MN) = 167.8 MB).
TRAFFIC_OVER_ALGORITHMIC = 216.2 / 167.8


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--transport", choices=("peer", "nccl"), default="peer",
                    help="--case ep:*: how rows cross GPUs")
    ap.add_argument("--ep-sync", choices=("signals", "nccl"), default="signals",
                    help="--case ep:* --transport peer: how the GPUs synchronise")
    ap.add_argument("--ep-graph", action="store_true",
                    help="--case ep:* with --transport peer --ep-sync signals: replay the forward as a CUDA graph")
    ap.add_argument("--fused-return", action="store_true",
                    help="--case ep:* --transport peer: the second expert GEMM's epilogue stores rows to their home GPU")
    ap.add_argument("--eager", action="store_true", help="--case: time eager launches instead of graph replays")
    ap.add_argument("--case", default=None, help="run one operator case instead of the sweep (see run_case)")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-operator records (`ops`) of the JSON line")
    ap.add_argument("--ep-eager", action="store_true",
                    help="N > 1: launch the expert-parallel forwards of `ops` eagerly instead of replaying a CUDA graph")
    args = ap.parse_args()
    if args.case and args.case.startswith("ep:"):
        run_ep_case(args)
    elif args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_b200_arm(args)


if __name__ == "__main__":
    main()
