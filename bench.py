"""Benchmark of the HFFN sparse FFN hot path on B200: one JSON line on rank 0.

Default workload (``--workload fwd``): the Pythia-410M-shape synthetic HFFN layer of the benchmark plan, d_model 1024,
d_ff 4096, 512-of-1024 supports per neuron (50 %), N = 4096 tokens per GPU per step, float32. A step is one forward
of the layer over one batch: the up kernel (+ bias + GELU) then the down kernel, launched through the C ABI on inputs
resident in HBM (the tensor-core pair by the runtime's policy; ``--path cuda_cores`` forces the gather kernels).
Other workloads: ``fwd_bf16`` (the same in bfloat16 storage); ``train`` (the training step: d_model 2048, d_ff 8192,
80 %, N = 8192, MSE loss, backward and AdamW); ``decode`` (24 Pythia-410M-shape FFN layers x 8 tokens per step,
the prepared decode path in a CUDA graph, HBM roofline); ``pythia410m`` (the model: prefill and greedy decode, HFFN
arm and dense arm).

Timing: W warm-up steps, then exactly K timed steps bracketed by a barrier and a device synchronisation; every step
is timed with CUDA events on the launching stream and the L2 is flushed (a 512 MiB write) between steps, outside the
events (workloads whose per-step inputs exceed L2 say so instead). ``e2e``: the same metric through the public API
with host batches in pinned memory, copied in and the outputs copied back every step (``HostPipeline`` overlaps the
copies with the kernels). Multi-GPU (torchrun, one process per GPU): the forward is neuron-sharded (each rank holds a
slice of the hidden neurons and sends every rank's batch through it: NCCL all-gather / reduce-scatter, or
``--transport peer`` for the NVLink peer-memory pipeline); training is data-parallel with a gradient all-reduce;
``decode`` runs replicas. Weak scaling: each rank brings its own batch; the time is the max over ranks.

``--impl reference`` times the reference's own x86 AVX2 kernel (compiled from the reference sources into
``oracle/_ref``) on this host's cores, on the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 512 << 20
WORKLOADS = {
    "fwd": {"case": "c2_1024_4096_k512", "n": 4096, "dtype": "fp32"},
    "fwd_bf16": {"case": "c2_1024_4096_k512", "n": 4096, "dtype": "bf16"},
    "train": {"case": "c3_2048_8192_k1638", "n": 8192, "dtype": "fp32"},
    "train_small": {"case": "c3_2048_8192_k1638", "n": 1024, "dtype": "fp32"},
    "pythia410m": {"case": "c4_1024_4096_k512", "n": 8 * 512, "dtype": "bf16", "batch": 8, "prompt": 512,
                   "decode": 128},
    "decode": {"case": "c4_1024_4096_k512", "n": 8, "dtype": "bf16", "layers": 24},
}
# DRAM bytes (read + write) per launch of the dominant kernel from one `ncu --set full` capture of the same workload
# on a B200 (dram__bytes_read.sum + dram__bytes_write.sum); the command and the figures are in the named summary under
# profiles/. Keyed by (workload, kernel); a kernel without a capture reports null.
NCU_TRAFFIC = {
    ("fwd", "tc_gemm_up"): (142.489e6 + 96.618e6, "profiles/fwd_tensor_cores_c2_fp32.md"),
    ("fwd_bf16", "tc_gemm_up"): (16.834e6 + 0.433e6, "profiles/fwd_tensor_cores_c2_bf16.md"),
}
CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
               "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
               "clocks_event_reasons.sw_power_cap")


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index: int) -> None:
        self.index, self.proc, self.rows = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={CLOCK_QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        time.sleep(0.15)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[k] for r in self.rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def reference_arm(args, workload: dict) -> dict:
    """The reference x86 kernel on this host's cores: each step a bounded sample of the workload's tokens."""
    from hffn_b200 import synth
    from oracle import x86ref
    case = synth.CASES[workload["case"]]
    unit = "tokens/s"
    metric = f"HFFN FFN layer tokens/s ({'forward' if args.workload != 'train' else 'train step'}, {workload['dtype']})"
    if args.workload != "fwd" or not x86ref.available():
        why = "oracle/_ref not built" if not x86ref.available() else \
            "the reference x86 kernel is float32 inference only; no CPU arm for this workload"
        return {"impl": "reference", "unavailable": why, "metric": metric}
    layer = synth.make_layer(case)
    threads = len(os.sched_getaffinity(0))
    kernel = x86ref.X86Kernel(layer, threads=threads)
    sample = args.ref_tokens
    x = synth.make_input(case, workload["n"])[:sample]
    for _ in range(args.warmup):
        kernel.forward(x)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        kernel.forward(x)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload["case"], "tokens_per_step": sample, "parallelism": f"{threads} host threads"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "reference",
                             "sample": f"{sample} of the {workload['n']} tokens per step, dual route, <=96-token chunks"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_baseline(workload: dict, seconds: float) -> dict | None:
    """The reference x86 kernel on a bounded sample of the workload (rank 0, N = 1)."""
    from hffn_b200 import synth
    from oracle import x86ref
    if not x86ref.available() or workload["dtype"] != "fp32" or workload["case"] != "c2_1024_4096_k512":
        return None
    case = synth.CASES[workload["case"]]
    threads = len(os.sched_getaffinity(0))
    kernel = x86ref.X86Kernel(synth.make_layer(case), threads=threads)
    x = synth.make_input(case, workload["n"])
    chunk = 512
    kernel.forward(x[:chunk])
    tokens, start = 0, time.perf_counter()
    while time.perf_counter() - start < seconds:
        lo = tokens % workload["n"]
        kernel.forward(x[lo:lo + chunk])
        tokens += chunk
    elapsed = time.perf_counter() - start
    return {"value": tokens / elapsed, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{tokens} tokens in 512-token slices of the workload's batch, {elapsed:.1f} s"}


def algorithmic(case, n: int, elem: int) -> dict:
    """Algorithmic bytes and FLOPs of the two forward kernels per launch (minimal traffic of each kernel)."""
    e_up = case.d_ff * case.up_degree
    e_down = case.d_ff * case.down_degree
    up_bytes = n * case.d_model * elem + e_up * (2 + elem) + case.d_ff * (elem + 4) + 4 + case.d_ff * n * elem
    down_bytes = case.d_ff * n * elem + e_down * (2 + elem) + case.d_model * (elem + 4) + 4 + n * case.d_model * elem
    return {"up": {"bytes": up_bytes, "flops": 2.0 * e_up * n}, "down": {"bytes": down_bytes, "flops": 2.0 * e_down * n}}


def fp32_gemm_peak(torch) -> float:
    """Measured FP32 CUDA-core GEMM throughput (cuBLAS SGEMM 8192^3, TF32 off, best of 5), TFLOP/s."""
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    c = a @ b
    best = float("inf")
    for _ in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        torch.mm(a, b, out=c)
        end.record()
        end.synchronize()
        best = min(best, start.elapsed_time(end) / 1e3)
    del a, b, c
    return 2 * 8192 ** 3 / best / 1e12


def canonical(layer, torch) -> dict:
    return {k: torch.from_numpy(getattr(layer, k).copy()) for k in
            ("b_up", "up_offsets", "up_idx", "up_val", "b_down", "down_offsets", "down_idx", "down_val")}


def rank_input(case, n: int, rank: int) -> np.ndarray:
    """Rank 0's batch is the workload's seeded input; rank k > 0 draws its own from [seed, n, 1000 + k]."""
    from hffn_b200 import synth
    if rank == 0:
        return synth.make_input(case, n)
    rng = np.random.default_rng([case.seed, n, 1000 + rank])
    return np.ascontiguousarray(rng.standard_normal((n, case.d_model)).astype(np.float32))


def setup_dist(torch):
    import datetime

    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    return rank, world, local, device


def max_over_ranks(torch, values: list[float], world: int, device) -> list[float]:
    import torch.distributed as dist
    t = torch.tensor(values, device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def gpu_arm(args, workload: dict) -> dict | None:
    import torch
    import torch.distributed as dist

    from hffn_b200 import _native as native
    from hffn_b200 import synth
    from hffn_b200.distributed import sharded_runtime
    from hffn_b200.runtime import HFFNLayer, HFFNRuntime

    rank, world, local, device = setup_dist(torch)
    if args.workload.startswith("train"):
        return train_arm(args, workload, rank, world, local, device)
    if args.workload == "pythia410m":
        return pythia_arm(args, workload, rank, world, local, device)
    if args.workload == "decode":
        return decode_arm(args, workload, rank, world, local, device)
    case = synth.CASES[workload["case"]]
    n = workload["n"]
    dtype = torch.float32 if workload["dtype"] == "fp32" else torch.bfloat16
    elem = 4 if dtype == torch.float32 else 2
    layer = synth.make_layer(case)
    tensor_cores = False if args.path == "cuda_cores" else None
    if world == 1:
        t = torch.from_numpy
        kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets),
                                         t(layer.up_idx), t(layer.up_val), t(layer.b_down), t(layer.down_offsets),
                                         t(layer.down_idx), t(layer.down_val))
        runtime, shard, (lo, hi) = HFFNRuntime([kl], device, dtype, tensor_cores=tensor_cores), None, (0, case.d_ff)
    else:
        runtime, shard, (lo, hi) = sharded_runtime(case.d_model, canonical(layer, torch), device, dtype,
                                                   tensor_cores=tensor_cores, segments=args.segments,
                                                   comm_sms=args.comm_sms, transport=args.transport, push=args.push)
    if args.path == "tensor_cores":
        runtime.force("tc", "tc")
    d, f_local = case.d_model, hi - lo
    n_kernel = n * world                       # a shard runs every rank's batch through its neurons
    x_host = torch.from_numpy(rank_input(case, n, rank)).to(dtype).pin_memory()
    x = x_host.to(device)
    x_all = torch.from_numpy(np.concatenate([rank_input(case, n, k) for k in range(world)])).to(dtype).to(device) \
        if world > 1 else x
    runtime.forward(0, x_all)
    up, down = runtime.modes(n_kernel)
    code, struct = runtime._code, runtime._structs[0]
    stream = torch.cuda.current_stream(device)
    handle = stream.cuda_stream
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=device)
    tc = up == "tc"
    ptr = lambda v: None if v is None else v.data_ptr()  # noqa: E731
    if tc:
        dense, work, err = runtime._dense[0], runtime._tc_work.data_ptr(), runtime._err.data_ptr()
        if dtype == torch.float32:
            x_split, act_hi = work, work + 2 * n_kernel * d * 4
            act_lo = act_hi + n_kernel * f_local * 4
        else:
            x_split, act_hi, act_lo = None, work, None

    def kernels(marks):
        """The two kernels of one forward of the local runtime over x_all, an event between them."""
        if tc:
            native.check(native.lib.hffn_up_tc(code, x_all.data_ptr(), ptr(dense["up_hi"]), ptr(dense["up_lo"]),
                                               struct.b_up, act_hi, act_lo, None, x_split, err, d, f_local,
                                               n_kernel, handle), "hffn_up_tc")
            marks[1].record(stream)
            native.check(native.lib.hffn_down_tc(code, act_hi, act_lo, ptr(dense["down_hi"]), ptr(dense["down_lo"]),
                                                 struct.b_down, runtime._y.data_ptr(), err, d, f_local, n_kernel,
                                                 handle), "hffn_down_tc")
            return
        native.check(native.lib.hffn_up(code, native.UP_CODES[up], x_all.data_ptr(), struct.up_offsets,
                                        struct.up_idx, struct.up_val, struct.b_up, runtime._act.data_ptr(), None, d,
                                        f_local, n_kernel, handle), "hffn_up")
        marks[1].record(stream)
        native.check(native.lib.hffn_down(code, native.DOWN_CODES[down], runtime._act.data_ptr(), struct.out_offsets,
                                          struct.out_hidden, struct.out_val, struct.b_down, runtime._y.data_ptr(), d,
                                          f_local, n_kernel, handle), "hffn_down")

    def events(k):
        return [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(k)]

    # kernel loop: the local forward's two kernels, per-kernel events (the roofline's timing); for one GPU it is
    # also the timed step
    for marks in events(args.warmup):
        flush.zero_()
        marks[0].record(stream)
        kernels(marks)
    kernel_events = events(args.steps)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        for marks in kernel_events:
            flush.zero_()
            marks[0].record(stream)
            kernels(marks)
            marks[2].record(stream)
        torch.cuda.synchronize(device)
        step_events = None
        if world > 1 and args.transport == "peer":
            # the sharded steps as one pipelined stream of batches (forward_many): batch k's gathers and batch
            # k - 2's deliveries run on the copy engines during batch k - 1's GEMMs; each step's working set
            # (gathered batches, activations, partial outputs) exceeds L2, which is not flushed inside the stream
            shard.forward_many([x] * args.warmup)
            dist.barrier()
            torch.cuda.synchronize(device)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            shard.forward_many([x] * args.steps)
            b.record(stream)
            torch.cuda.synchronize(device)
            step_ms_pipelined = a.elapsed_time(b) / args.steps
        elif world > 1:
            # the sharded step: broadcast / compute / reduce pipeline over the ranks' batches
            for _ in range(args.warmup):
                flush.zero_()
                shard.forward(x)
            step_events = events(args.steps)
            dist.barrier()
            torch.cuda.synchronize(device)
            for marks in step_events:
                flush.zero_()
                marks[0].record(stream)
                shard.forward(x)
                marks[2].record(stream)
            torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    up_ms = [e[0].elapsed_time(e[1]) for e in kernel_events]
    down_ms = [e[1].elapsed_time(e[2]) for e in kernel_events]
    step_ms = [e[0].elapsed_time(e[2]) for e in (step_events or kernel_events)]
    if world > 1 and args.transport == "peer":
        step_ms = [step_ms_pipelined] * args.steps

    # end to end through the public API: every step copies its batch from pinned host memory to the device, runs the
    # forward and copies the output back to pinned host memory; HostPipeline overlaps step k's kernels with the copy
    # in of step k + 1 and the copy out of step k - 1. Timed from the first copy in to the last copy out. Run twice:
    # as a user runs it, and with the 512 MiB L2 flush queued before every step's kernels (the flush's own time
    # included: an upper bound on what a cold L2 costs).
    from hffn_b200.pipeline import HostPipeline, runtime_forward
    if world == 1:
        device_forward = runtime_forward(runtime, 0)
    else:
        def device_forward(x_dev, out):
            out.copy_(shard.forward(x_dev))
    x_hosts = [torch.from_numpy(rank_input(case, n, rank + 97 * k)).to(dtype).pin_memory() for k in range(2)]
    y_hosts = [torch.empty(n, d, dtype=dtype).pin_memory() for _ in range(max(args.steps, args.warmup))]

    def e2e_run(flushed: bool) -> float:
        forward = device_forward
        if flushed:
            def forward(x_dev, out):
                flush.zero_()
                device_forward(x_dev, out)
        pipe = HostPipeline(forward, d, d, n, dtype, device)
        pipe.run([x_hosts[k % 2] for k in range(args.warmup)], y_hosts[:args.warmup])
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        pipe.run([x_hosts[k % 2] for k in range(args.steps)], y_hosts[:args.steps], wait=False)
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    e2e_ms = [e2e_run(False)]
    e2e_flushed_ms = e2e_run(True)
    e2e_ok = all(torch.equal(y_hosts[k], y_hosts[k % 2]) for k in range(2, args.steps))
    total_s, e2e_s, e2e_flushed_s = max_over_ranks(torch, [sum(step_ms) / 1e3, sum(e2e_ms) / 1e3,
                                                          e2e_flushed_ms / 1e3], world, device)
    pk, pk_source = peaks()
    fp32_peak = fp32_gemm_peak(torch) if rank == 0 else None
    errors = runtime.device_errors()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    local_case = type(case)(case.name, d, f_local, case.up_degree, case.down_degree, False, case.seed)
    alg = algorithmic(local_case, n_kernel, elem)
    kernel_ms = {"up": statistics.mean(up_ms), "down": statistics.mean(down_ms)}
    top = max(kernel_ms, key=kernel_ms.get)
    seconds = kernel_ms[top] / 1e3
    achieved_gbs = alg[top]["bytes"] / seconds / 1e9
    achieved_tflops = alg[top]["flops"] / seconds / 1e12
    hbm = {"achieved_gbs": achieved_gbs, "peak_gbs": pk["hbm_gbs"], "frac": achieved_gbs / pk["hbm_gbs"],
           "algorithmic_bytes": alg[top]["bytes"]}
    if tc:
        passes = 3 if elem == 4 else 1
        dense_flops = 2.0 * n_kernel * f_local * d * passes
        pipe_peak = pk["bf16_tflops"] / (2 if elem == 4 else 1)
        traffic, traffic_source = NCU_TRAFFIC.get((args.workload, f"tc_gemm_{top}"), (None, None)) \
            if world == 1 else (None, None)
        roofline = {"bound": "tensor", "kernel": f"tc_gemm_{top}", "achieved": achieved_tflops,
                    "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved_tflops / pk["bf16_tflops"],
                    "traffic": traffic, "traffic_source": traffic_source,
                    "algorithmic_flops": alg[top]["flops"], "launch_ms": kernel_ms[top],
                    "peak_source": pk_source,
                    "tensor_pipe": {"kind": "tf32 x3 (3xTF32 split)" if elem == 4 else "bf16",
                                    "executed_tflops": dense_flops / seconds / 1e12, "peak_tflops": pipe_peak,
                                    "peak_note": "tf32 = half the measured bf16 peak (nominal ratio)" if elem == 4
                                    else "measured bf16 burst",
                                    "frac": dense_flops / seconds / 1e12 / pipe_peak},
                    "hbm": hbm}
        launches_per_kernel_step = 3 if elem == 4 else 2
    else:
        roofline = {"bound": "hbm", "kernel": f"{top}_{up if top == 'up' else down}", "achieved": achieved_gbs,
                    "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved_gbs / pk["hbm_gbs"], "traffic": None,
                    "algorithmic_bytes": alg[top]["bytes"], "launch_ms": kernel_ms[top], "peak_source": pk_source,
                    "fp32_cuda_cores": {"achieved_tflops": achieved_tflops, "peak_tflops": fp32_peak,
                                        "frac": achieved_tflops / fp32_peak if fp32_peak else None,
                                        "peak_source": "cuBLAS SGEMM 8192^3 TF32 off, measured in this run"}}
        launches_per_kernel_step = 2
    tokens = n * world * args.steps
    line = {
        "metric": f"HFFN FFN layer tokens/s (forward, {workload['dtype']})",
        "value": tokens / total_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total_s / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if elem == 4 else "bf16", "data": "synthetic",
        "config": {"workload": f"{case.name}: d_model {d}, d_ff {case.d_ff}, support {case.up_degree}, "
                               f"N {n} tokens per GPU per step", "modes": [up, down],
                   "parallelism": "single" if world == 1 else
                   f"neuron-sharded x{world} (NVLink peer memory, pipelined over batches: copy-engine gathers, "
                   f"partial outputs delivered into the owners' slots by "
                   f"{'the down GEMM epilogue' if args.push == 'store' else 'copy engines'})" if args.transport == "peer"
                   else
                   f"neuron-sharded x{world} (all-gather / reduce-scatter pipeline over NCCL, "
                   f"{shard.segments} segments, {shard.comm_sms} SMs left to NCCL)",
                   "l2": "flushed between steps (512 MiB write)"},
        "roofline": roofline,
        "fp32_gemm_peak_tflops": fp32_peak,
        "kernels_ms": kernel_ms,
        "e2e": {"value": n * world * args.steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": x_hosts[0].numel() * elem, "d2h_bytes_per_step": y_hosts[0].numel() * elem,
                "pipelined": "copy in of step k+1 and copy out of step k-1 overlap step k's kernels (HostPipeline)",
                "l2": "not flushed: every step's batch arrives by a fresh host-to-device copy and the step's working "
                      "set (x, split x, act, dense weights, y) exceeds L2",
                "value_l2_flushed": n * world * args.steps / e2e_flushed_s,
                "outputs_repeatable": e2e_ok},
        "gpu_launches": launches_per_kernel_step * args.steps,
        "device_errors": errors,
        "clocks": clocks.summary(),
    }
    if world > 1:
        line["kernel_loop_ms_per_step"] = statistics.mean(a + b for a, b in zip(up_ms, down_ms))
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(workload, args.cpu_seconds)
    return line


def train_arm(args, workload: dict, rank: int, world: int, local: int, device) -> dict | None:
    """The MSE training step (d_model 2048, d_ff 8192, 80 %, N per GPU), data parallel over ranks."""
    import torch
    import torch.distributed as dist

    from hffn_b200 import synth
    from hffn_b200.distributed import DataParallelTrainer
    from hffn_b200.runtime import HFFNLayer, HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime

    case = synth.CASES[workload["case"]]
    n = workload["n"]
    layer = synth.make_layer(case)
    t = torch.from_numpy
    kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                     t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                     t(layer.down_val))
    runtime = HFFNRuntime([kl], device, tensor_cores=False if args.path == "cuda_cores" else None)
    train = HFFNTrainRuntime(runtime, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, max_tokens=n,
                             store_gradients=world > 1,
                             tensor_cores={"cuda_cores": False, "tensor_cores": True}.get(args.path))
    tc = train.uses_tensor_cores(0, n)
    train.reserve(n)
    x_host = t(rank_input(case, n, rank)).pin_memory()
    target_host = t(synth.make_target(case, n) if rank == 0 else rank_input(case, n, rank + 500)).pin_memory()
    x, target = x_host.to(device), target_host.to(device)
    dp = DataParallelTrainer(train) if world > 1 else None
    step = (lambda: dp.step_mse(0, x, target)) if dp else (lambda: train.step_mse(0, x, target))
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        step()
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        for a, b in marks:
            a.record(stream)
            loss = step()
            b.record(stream)
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in marks]
    loss_host = torch.empty(1, dtype=loss.dtype).pin_memory()
    e2e_ms = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        x.copy_(x_host, non_blocking=True)
        target.copy_(target_host, non_blocking=True)
        loss = step()
        loss_host.copy_(loss, non_blocking=True)
        b.record(stream)
        b.synchronize()
        e2e_ms.append(a.elapsed_time(b))
    total_s, e2e_s = max_over_ranks(torch, [sum(step_ms) / 1e3, sum(e2e_ms) / 1e3], world, device)
    pk, pk_source = peaks()
    fp32_peak = fp32_gemm_peak(torch) if rank == 0 else None
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    e = case.d_ff * case.up_degree
    flops = 12.0 * e * n                       # forward 2 x 2En, backward 2x the forward
    step_bytes = (4 * n * case.d_model * 4      # x, target, gy, gx
                  + 2 * case.d_ff * n * 4 * 2   # z written and read
                  + 2 * e * 6 * 2               # both supports (index + value), forward and backward
                  + 2 * e * 24)                 # AdamW: p, m, v read and written, both value arrays
    seconds = total_s / args.steps
    achieved = step_bytes / seconds / 1e9
    if tc:
        dense_flops = 6 * 2.0 * case.d_model * case.d_ff * n * 3      # six GEMMs, three tf32 passes each
        roofline = {"bound": "tensor", "kernel": "whole step (six tcgen05 GEMMs)", "achieved": flops / seconds / 1e12,
                    "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": flops / seconds / 1e12 / pk["bf16_tflops"],
                    "traffic": None, "algorithmic_flops": flops, "peak_source": pk_source,
                    "tensor_pipe": {"kind": "tf32 x3 (3xTF32 split)", "executed_tflops": dense_flops / seconds / 1e12,
                                    "peak_tflops": pk["bf16_tflops"] / 2,
                                    "peak_note": "tf32 = half the measured bf16 peak (nominal ratio)",
                                    "frac": dense_flops / seconds / 1e12 / (pk["bf16_tflops"] / 2)},
                    "hbm": {"achieved_gbs": achieved, "peak_gbs": pk["hbm_gbs"], "frac": achieved / pk["hbm_gbs"],
                            "algorithmic_bytes": step_bytes},
                    "fp32_cuda_cores": {"achieved_tflops": flops / seconds / 1e12, "peak_tflops": fp32_peak,
                                        "frac": flops / seconds / 1e12 / fp32_peak if fp32_peak else None}}
    else:
        roofline = {"bound": "hbm", "kernel": "whole step", "achieved": achieved, "peak": pk["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": None,
                    "algorithmic_bytes": step_bytes, "peak_source": pk_source,
                    "fp32_cuda_cores": {"achieved_tflops": flops / seconds / 1e12, "peak_tflops": fp32_peak,
                                        "frac": flops / seconds / 1e12 / fp32_peak if fp32_peak else None}}
    return {
        "metric": "HFFN FFN layer tokens/s (train step, fp32)", "value": n * world * args.steps / total_s,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * seconds, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{case.name}: d_model {case.d_model}, d_ff {case.d_ff}, support {case.up_degree}, "
                               f"N {n} tokens per GPU per step, MSE loss, AdamW",
                   "path": "tensor_cores" if tc else "cuda_cores",
                   "parallelism": f"data parallel x{world}, gradient all-reduce over NCCL" if world > 1 else "single",
                   "l2": "inputs larger than L2 (z and act alone 537 MB)"},
        "roofline": roofline,
        "e2e": {"value": n * world * args.steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * x_host.numel() * 4, "d2h_bytes_per_step": loss_host.numel() * 8},
        "gpu_launches": (10 if tc else 8) * args.steps, "device_errors": runtime.device_errors(),
        "clocks": clocks.summary(),
        "loss_last": float(loss_host),
    }


def decode_arm(args, workload: dict, rank: int, world: int, local: int, device) -> dict | None:
    """The decode FFN step of the Pythia-410M shape: 24 layers (C4: d_model 1024, d_ff 4096, 50 % supports, bf16),
    8 tokens per call, one call per layer, through ``PreparedRuntime`` (the decode path: prepared per (layer, N),
    the cooperative kernels), the 24 calls of a step replayed as one CUDA graph. Every layer has its own copy of the
    compact arrays in HBM (403 MB of edge streams per step, above L2: no flush needed). HBM-bound: the roofline is
    the algorithmic bytes of the 48 kernels (edges, offsets, biases, x, act, y) per step over the step time. Replicas
    only: with N > 1 every rank runs its own copy."""
    import torch
    import torch.distributed as dist

    from hffn_b200 import synth
    from hffn_b200.runtime import HFFNLayer, PreparedRuntime
    from oracle import x86ref
    case = synth.CASES[workload["case"]]
    layers_n, n = workload["layers"], workload["n"]
    layer = synth.make_layer(case)
    t = torch.from_numpy
    kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                     t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                     t(layer.down_val))
    runtime = PreparedRuntime([kl] * layers_n, device, torch.bfloat16)
    d = case.d_model
    x_host = torch.from_numpy(np.stack([rank_input(case, n, rank + 31 * k) for k in range(layers_n)])).to(
        torch.bfloat16).pin_memory()
    x = x_host.to(device)
    stream = torch.cuda.current_stream(device)

    def step():
        for index in range(layers_n):
            runtime.forward(index, x[index])

    step()                                                   # prepares every (layer, N) entry outside the capture
    up, down = runtime.modes(n)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()
        with torch.cuda.graph(graph, stream=side):
            step()
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    for _ in range(args.warmup):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize(device)
        graph_ms = a.elapsed_time(b) / args.steps
        a.record(stream)
        for _ in range(args.steps):
            step()
        b.record(stream)
        torch.cuda.synchronize(device)
        eager_ms = a.elapsed_time(b) / args.steps
    # the two kernels of a layer apart: every layer's up kernel, then every layer's down kernel, eager launches
    from hffn_b200 import _native as native
    handle = stream.cuda_stream
    act = runtime._act.data_ptr()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    marks[0].record(stream)
    for index in range(layers_n):
        st = runtime._structs[index]
        native.check(native.lib.hffn_up(runtime._code, native.UP_CODES[up], x[index].data_ptr(), st.up_offsets,
                                        st.up_idx, st.up_val, st.b_up, act, None, d, case.d_ff, n, handle), "hffn_up")
    marks[1].record(stream)
    for index in range(layers_n):
        st = runtime._structs[index]
        native.check(native.lib.hffn_down(runtime._code, native.DOWN_CODES[down], act, st.out_offsets, st.out_hidden,
                                          st.out_val, st.b_down, runtime._y.data_ptr(), d, case.d_ff, n, handle),
                     "hffn_down")
    marks[2].record(stream)
    torch.cuda.synchronize(device)
    kernel_us = {"up": 1e3 * marks[0].elapsed_time(marks[1]) / layers_n,
                 "down": 1e3 * marks[1].elapsed_time(marks[2]) / layers_n}
    # end to end: the step's 24 inputs copied in from pinned host memory, the 24 outputs copied back, every step
    y_host = torch.empty(layers_n, n, d, dtype=torch.bfloat16).pin_memory()
    e2e = []
    for k in range(args.warmup + args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        x.copy_(x_host, non_blocking=True)
        for index in range(layers_n):
            y_host[index].copy_(runtime.forward(index, x[index]), non_blocking=True)
        b.record(stream)
        b.synchronize()
        if k >= args.warmup:
            e2e.append(a.elapsed_time(b))
    step_s, e2e_s = max_over_ranks(torch, [graph_ms / 1e3, sum(e2e) / len(e2e) / 1e3], world, device)
    pk, pk_source = peaks()
    alg = algorithmic(case, n, 2)
    step_bytes = layers_n * (alg["up"]["bytes"] + alg["down"]["bytes"])
    achieved = step_bytes / step_s / 1e9
    errors = runtime.device_errors()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and x86ref.available():
        threads = len(os.sched_getaffinity(0))
        kernel = x86ref.X86Kernel(layer, threads=threads)
        xs = x_host.float().numpy()
        kernel.forward(xs[0])
        steps, start = 0, time.perf_counter()
        while time.perf_counter() - start < args.cpu_seconds:
            for index in range(layers_n):
                kernel.forward(xs[index])
            steps += 1
        elapsed = time.perf_counter() - start
        cpu = {"value": steps * n * layers_n / elapsed, "unit": "layer-tokens/s", "cores": threads,
               "kind": "reference", "sample": f"{steps} decode steps (24 calls of 8 tokens, float32: the reference "
                                              f"kernel's only type), {elapsed:.1f} s"}
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {
        "metric": "HFFN FFN layer tokens/s (decode, bf16)", "value": n * layers_n * world / step_s,
        "unit": "layer-tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{case.name}: Pythia-410M FFN shape, {layers_n} layers x {n} tokens per decode step "
                               f"(one call per layer, CUDA graph)", "modes": [up, down],
                   "parallelism": "single" if world == 1 else f"replicas x{world}",
                   "l2": f"inputs larger than L2 (edge streams {step_bytes / 1e6:.0f} MB per step)"},
        "roofline": {"bound": "hbm", "kernel": f"whole decode step ({up} + {down}, {2 * layers_n} launches)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "traffic": None, "algorithmic_bytes": step_bytes, "peak_source": pk_source},
        "eager_ms_per_step": eager_ms,
        "kernel_us_eager": kernel_us,
        "e2e": {"value": n * layers_n * world / e2e_s, "unit": "layer-tokens/s",
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 2},
        "gpu_launches": 2 * layers_n * args.steps, "device_errors": errors, "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }


def pythia_arm(args, workload: dict, rank: int, world: int, local: int, device) -> dict | None:
    """The Pythia-410M architecture (random init, 50 % HFFN FFNs, bfloat16): prefill of batch x prompt tokens, then
    greedy decode steps with the KV cache; the HFFN arm and the dense arm (the model's own MLP with the same weights
    on the support) timed back to back on the same prompts."""
    import tempfile

    import torch

    from hffn_b200 import pythia
    root = Path(tempfile.gettempdir()) / "hffn_bench_pythia410m"
    if not (root / "model" / "model.safetensors").exists():
        pythia.make_random_pythia(root / "model", root / "export", pythia.PYTHIA_410M, support=512, seed=3004)
    b, t, steps = workload["batch"], workload["prompt"], workload["decode"]
    g = torch.Generator().manual_seed(3004)
    prompt = torch.randint(0, 50277, (b, t), generator=g).to(device)
    stream = torch.cuda.current_stream(device)
    results = {}
    for arm in ("hffn", "dense"):
        model = pythia.load_pythia(root / "model", root / "export", arm, device, torch.bfloat16)

        @torch.inference_mode()
        def run():
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record(stream)
            out = model(input_ids=prompt, use_cache=True)
            e[1].record(stream)
            cache, token = out.past_key_values, out.logits[:, -1:].argmax(-1)
            for _ in range(steps):
                out = model(input_ids=token, past_key_values=cache, use_cache=True)
                cache, token = out.past_key_values, out.logits[:, -1:].argmax(-1)
            e[2].record(stream)
            e[2].synchronize()
            return e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])

        for _ in range(args.warmup):
            run()
        prefill, decode = zip(*[run() for _ in range(args.steps)])
        results[arm] = {"prefill_ms": statistics.median(prefill), "decode_ms": statistics.median(decode)}
        if arm == "hffn":
            results[arm]["device_errors"] = model.hffn_runtime.device_errors()
            results[arm]["ffn_calls"] = {f"{u}/{d}": c for (u, d), c in model.hffn_runtime.calls.items()}
        del model
        torch.cuda.empty_cache()
    h, d = results["hffn"], results["dense"]
    tokens = b * t + b * steps
    return {"metric": "Pythia-410M (50 % HFFN FFNs, bf16) tokens/s: prefill 8 x 512 + 128 greedy decode steps",
            "value": tokens / ((h["prefill_ms"] + h["decode_ms"]) / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random init, uniform token ids)",
            "config": {"workload": "pythia-410m architecture, 24 layers, d_model 1024, d_ff 4096, 512-of-1024 supports"},
            "prefill_tokens_per_s": {"hffn": b * t / (h["prefill_ms"] / 1e3), "dense": b * t / (d["prefill_ms"] / 1e3)},
            "decode_tokens_per_s": {"hffn": b * steps / (h["decode_ms"] / 1e3), "dense": b * steps / (d["decode_ms"] / 1e3)},
            "arms_ms": results}


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("hffn", "reference"), default="hffn")
    parser.add_argument("--workload", choices=tuple(WORKLOADS), default="fwd")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--ref-tokens", type=int, default=512)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--segments", type=int, default=None, help="sharded forward: pipeline segments per step")
    parser.add_argument("--comm-sms", type=int, default=0, help="sharded forward: SMs left to the collectives")
    parser.add_argument("--transport", choices=("nccl", "peer"), default="nccl",
                        help="sharded forward: NCCL collectives or NVLink peer memory (tensor cores)")
    parser.add_argument("--push", choices=("copy", "store"), default="copy",
                        help="peer sharded forward: partial outputs pushed by copy engines or by the GEMM epilogue")
    parser.add_argument("--path", choices=("auto", "cuda_cores", "tensor_cores"), default="auto",
                        help="forward kernels: the runtime policy, the CUDA-core gather kernels, or the tcgen05 path")
    args = parser.parse_args()
    workload = WORKLOADS[args.workload]
    rank, world, _ = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(reference_arm(args, workload)), flush=True)
        return 0
    line = gpu_arm(args, workload)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
