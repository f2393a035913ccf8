"""Benchmark of the HFFN sparse FFN hot path on B200: one JSON line on rank 0.

Default (``--workload all``): every configuration of the benchmark plan that one run can time, one record each; the
line's own fields are the headline record, the others sit under ``workloads``:
- headline, ``c2_fwd_fp32``: the Pythia-410M-shape synthetic layer (d_model 1024, d_ff 4096, 512-of-1024 supports,
  50 %), N = 4096 tokens per GPU per step, float32 (the reference's own precision). A step is one forward: the up
  kernel (+ bias + GELU) then the down kernel, launched through the C ABI on inputs resident in HBM;
- ``c2_fwd_bf16``: the same layer and batch in bfloat16 storage;
- ``c1_fwd_fp32`` (one GPU): d_model 512, d_ff 2048, 128-of-512 supports, N = 256 (the reference's CPU-runnable case);
- ``c3_train_fp32``: the training step, d_model 2048, d_ff 8192, 1638-of-2048 supports (80 %), N = 8192 tokens per
  GPU, MSE loss, backward and AdamW (data parallel over the GPUs, gradient all-reduce);
- ``c4_decode_bf16``: 24 Pythia-410M-shape FFN layers x 8 tokens per step, the prepared decode path in a CUDA graph
  (HBM-bound; replicas when N > 1);
- ``c5_pythia1b_bf16``: the Pythia-1B architecture (random init, 20 % HFFN FFNs, bf16), prefill of 64 x 2048 tokens,
  every FFN neuron-sharded over the N GPUs (strong scaling: the same batch at every N).
Single workloads: ``--workload fwd | fwd_bf16 | c1 | train | train_small | decode | pythia410m | c5`` (c5: Pythia-1B
bf16 prefill of 64 x 2048 tokens with every FFN neuron-sharded over the GPUs, the plan's 8-GPU configuration).

Every record carries: ``value`` (tokens/s of the whole job, inputs resident in HBM), ``roofline`` (the dominant kernel
against the measured peaks of ``MEASURED_PEAKS.json``), ``e2e`` (the same metric through the public API with host
batches: pinned host inputs copied in and outputs copied back every step, median of three windows, beside the
host-link roof: the same copies alone on all GPUs at once), ``parity`` (this run's outputs against the float64 oracle
on a subset of token rows, or the data-parallel gradients against the float64 oracle of the concatenated batch),
``cpu_baseline`` (one GPU: the reference's own x86 kernels on this host's cores, a bounded sample), ``clocks``.

Timing: W warm-up steps, then exactly K timed steps bracketed by a barrier and a device synchronisation; every step is
timed with CUDA events on the launching stream and the L2 is flushed (a 512 MiB write) between steps, outside the
events (workloads whose per-step inputs exceed L2 say so instead). Multi-GPU (torchrun, one process per GPU): the
forward is neuron-sharded (each rank holds a slice of the hidden neurons and sends every rank's batch through it:
NCCL all-gather / reduce-scatter, or ``--transport peer`` for the NVLink peer-memory pipeline); training is
data-parallel with a gradient all-reduce; decode runs replicas. Weak scaling: each rank brings its own batch; the time
is the max over ranks.

``--impl reference`` times the reference's own x86 AVX2 kernel (compiled from the reference sources into
``oracle/_ref``) on this host's cores, on the headline workload, 512-token slices of its batch per step (rank 0 only;
the same protocol as the headline's ``cpu_baseline``).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 512 << 20
PARITY_ROWS = 64
FP32_RELATIVE, BF16_RELATIVE = 1e-5, 2e-2
CPU_SLICE = 512
WORKLOADS = {
    "fwd": {"case": "c2_1024_4096_k512", "n": 4096, "dtype": "fp32"},
    "fwd_bf16": {"case": "c2_1024_4096_k512", "n": 4096, "dtype": "bf16"},
    "c1": {"case": "c1_512_2048_k128", "n": 256, "dtype": "fp32"},
    "train": {"case": "c3_2048_8192_k1638", "n": 8192, "dtype": "fp32"},
    "train_small": {"case": "c3_2048_8192_k1638", "n": 1024, "dtype": "fp32"},
    "pythia410m": {"case": "c4_1024_4096_k512", "n": 8 * 512, "dtype": "bf16", "batch": 8, "prompt": 512,
                   "decode": 128},
    "decode": {"case": "c4_1024_4096_k512", "n": 8, "dtype": "bf16", "layers": 24},
    "c5": {"case": "c5_2048_8192_k410", "dtype": "bf16", "batch": 64, "prompt": 2048, "support": 410, "seed": 3005},
}
COMPOSITE = (("c2_fwd_fp32", "fwd"), ("c2_fwd_bf16", "fwd_bf16"), ("c1_fwd_fp32", "c1"), ("c3_train_fp32", "train"),
             ("c4_decode_bf16", "decode"), ("c5_pythia1b_bf16", "c5"))
# DRAM bytes (read + write) per launch of the dominant kernel from one `ncu --set full` capture of the same workload
# on a B200 (dram__bytes_read.sum + dram__bytes_write.sum); the command and the figures are in the named summary under
# profiles/. Keyed by (workload, kernel, operand format); a kernel without a capture reports null.
NCU_TRAFFIC = {
    ("fwd", "tc_gemm_up", "f16x3"): (34.428e6 + 25.815e6, "profiles/fwd_tensor_cores_c2_fp32_f16x3.md"),
    ("fwd", "tc_gemm_up", "tf32x3"): (142.489e6 + 96.618e6, "profiles/fwd_tensor_cores_c2_fp32_tf32x3.md"),
    ("fwd_bf16", "tc_gemm_up", "bf16"): (16.834e6 + 0.433e6, "profiles/fwd_tensor_cores_c2_bf16.md"),
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


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


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


# -- CPU legs: the reference's own kernels on this host --------------------------------------------------------------
def reference_arm(args, workload: dict) -> dict:
    """The reference x86 kernel on this host's cores: each step one 512-token slice of the headline workload's batch
    (tokens are independent, so tokens/s of a slice is that of the batch)."""
    from hffn_b200 import synth
    from oracle import x86ref
    metric = f"HFFN FFN layer tokens/s (forward, {workload['dtype']})"
    if not x86ref.available():
        return {"impl": "reference", "unavailable": "oracle/_ref not built (make -C oracle)", "metric": metric}
    if workload["dtype"] != "fp32" or workload["case"] != WORKLOADS["fwd"]["case"]:
        return {"impl": "reference", "metric": metric,
                "unavailable": "the reference x86 kernel is float32 inference only; its arm times the headline workload"}
    case = synth.CASES[workload["case"]]
    layer = synth.make_layer(case)
    threads = host_threads()
    kernel = x86ref.X86Kernel(layer, threads=threads)
    sample = min(CPU_SLICE, workload["n"])
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
    return {"metric": metric, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload["case"], "tokens_per_step": sample,
                       "sample": f"{sample} of the workload's {workload['n']} tokens per step (tokens are independent)",
                       "parallelism": f"{threads} host threads"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": f"{sample}-token slices of the workload's batch, dual route, <=96-token chunks"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_forward_baseline(case, x: np.ndarray, seconds: float, slice_tokens: int = CPU_SLICE) -> dict | None:
    """The reference x86 kernel on all host cores over slices of the workload's batch for about ``seconds``."""
    from hffn_b200 import synth
    from oracle import x86ref
    if not x86ref.available():
        return None
    threads = host_threads()
    kernel = x86ref.X86Kernel(synth.make_layer(case), threads=threads)
    chunk = min(slice_tokens, x.shape[0])
    kernel.forward(x[:chunk])
    tokens, start = 0, time.perf_counter()
    while time.perf_counter() - start < seconds:
        lo = tokens % (x.shape[0] - chunk + 1)
        kernel.forward(x[lo:lo + chunk])
        tokens += chunk
    elapsed = time.perf_counter() - start
    return {"value": tokens / elapsed, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{tokens} tokens in {chunk}-token slices of the workload's batch, {elapsed:.1f} s "
                      f"(the reference x86 AVX2 kernel, float32)"}


def cpu_train_baseline(case, layer, tokens: int, steps: int) -> dict | None:
    """The reference's G4 training step (forward, MSE gradient, backward, AdamW; 4 workers) on a slice of the batch."""
    from hffn_b200 import synth
    from oracle import x86train
    if not x86train.available():
        return None
    step = x86train.G4Step(layer, tokens)
    x, target = synth.make_input(case, tokens), synth.make_target(case, tokens)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step.step_mse(x, target)
        times.append(time.perf_counter() - t0)
    return {"value": tokens * steps / sum(times), "unit": "tokens/s", "cores": x86train.GROUPS, "kind": "reference",
            "sample": f"{steps} steps of {tokens} tokens (the reference's G4 CPU training step: x86 forward with z, "
                      f"G4 backward and AdamW, its fixed 4 workers), {sum(times):.1f} s"}


# -- shared GPU context -----------------------------------------------------------------------------------------------
def rank_input(case, n: int, rank: int) -> np.ndarray:
    """Rank 0's batch is the workload's seeded input; rank k > 0 draws its own from [seed, n, 1000 + k]."""
    from hffn_b200 import synth
    if rank == 0:
        return synth.make_input(case, n)
    rng = np.random.default_rng([case.seed, n, 1000 + rank])
    return np.ascontiguousarray(rng.standard_normal((n, case.d_model)).astype(np.float32))


def rank_target(case, n: int, rank: int) -> np.ndarray:
    from hffn_b200 import synth
    if rank == 0:
        return synth.make_target(case, n)
    return rank_input(case, n, rank + 500)


def canonical(layer, torch) -> dict:
    return {k: torch.from_numpy(getattr(layer, k).copy()) for k in
            ("b_up", "up_offsets", "up_idx", "up_val", "b_down", "down_offsets", "down_idx", "down_val")}


def kernel_layer(layer, torch):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


class Context:
    """Process-wide state of one bench run: ranks, device, the L2 flush buffer, measured GEMM peaks."""

    def __init__(self, args) -> None:
        import datetime

        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.args = torch, dist, args
        self.rank, self.world, self.local = dist_env()
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", device_id=self.device, timeout=datetime.timedelta(seconds=300))
        self.stream = torch.cuda.current_stream(self.device)
        self.flush = torch.empty(L2_FLUSH_BYTES // 4, device=self.device)
        self._gemm_peaks: dict | None = None

    def barrier(self) -> None:
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize(self.device)

    def max_over_ranks(self, values: list[float]) -> list[float]:
        t = self.torch.tensor(values, device=self.device, dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(v) for v in t]

    def events(self, k: int, marks: int = 2):
        return [[self.torch.cuda.Event(enable_timing=True) for _ in range(marks)] for _ in range(k)]

    def gemm_peaks(self) -> dict:
        """cuBLAS float32 GEMMs 8192^3 measured in this run (best of 5, CUDA events): TF32 off (the CUDA-core SGEMM)
        and TF32 on (the tensor pipe at tf32, the peak of one 3xTF32 pass). Rank 0 only."""
        if self._gemm_peaks is None:
            torch = self.torch
            a = torch.randn(8192, 8192, device=self.device)
            b = torch.randn(8192, 8192, device=self.device)
            c = a @ b
            out = {}
            for name, tf32 in (("fp32_simt_tflops", False), ("tf32_tflops", True)):
                torch.backends.cuda.matmul.allow_tf32 = tf32
                torch.mm(a, b, out=c)
                best = float("inf")
                for _ in range(5):
                    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    start.record()
                    torch.mm(a, b, out=c)
                    end.record()
                    end.synchronize()
                    best = min(best, start.elapsed_time(end) / 1e3)
                out[name] = 2 * 8192 ** 3 / best / 1e12
            torch.backends.cuda.matmul.allow_tf32 = False
            out["source"] = "cuBLAS float32 GEMM 8192^3 in this run, best of 5 (TF32 off / on)"
            self._gemm_peaks = out
            del a, b, c
        return self._gemm_peaks

    def close(self) -> None:
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def bf16_rounded(a: np.ndarray, torch) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).float().numpy()


def bf16_held(layer, torch):
    """The layer as a bf16 runtime holds it: the four value arrays rounded to bf16."""
    import dataclasses
    return dataclasses.replace(layer, up_val=bf16_rounded(layer.up_val, torch), b_up=bf16_rounded(layer.b_up, torch),
                               down_val=bf16_rounded(layer.down_val, torch),
                               b_down=bf16_rounded(layer.b_down, torch))


def relative_error(y: np.ndarray, expected: np.ndarray) -> float:
    """max |y - y_float64| / max(1, |y_float64|), the reference's parity measure."""
    return float(np.max(np.abs(np.asarray(y, np.float64) - expected) / np.maximum(1.0, np.abs(expected))))


def host_link_roof(ctx: Context, x_host, x_dev, y_host, y_dev, steps: int) -> float:
    """Seconds for ``steps`` pipelined copy pairs alone (pinned host -> device of x, device -> pinned host of y, on two
    streams), all ranks at once, max over ranks: the floor of any end-to-end step that moves these bytes."""
    torch = ctx.torch
    streams = [torch.cuda.Stream(ctx.device), torch.cuda.Stream(ctx.device)]
    ctx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(ctx.stream)
    for s in streams:
        s.wait_event(start)
    for _ in range(steps):
        with torch.cuda.stream(streams[0]):
            x_dev.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(streams[1]):
            y_host.copy_(y_dev, non_blocking=True)
    for s in streams:
        ctx.stream.wait_stream(s)
    end.record(ctx.stream)
    end.synchronize()
    return ctx.max_over_ranks([start.elapsed_time(end) / 1e3])[0]


# -- the forward -----------------------------------------------------------------------------------------------------
def algorithmic(case, n: int, elem: int) -> dict:
    """Algorithmic bytes and FLOPs of the two forward kernels per launch (minimal traffic of each kernel)."""
    e_up = case.d_ff * case.up_degree
    e_down = case.d_ff * case.down_degree
    up_bytes = n * case.d_model * elem + e_up * (2 + elem) + case.d_ff * (elem + 4) + 4 + case.d_ff * n * elem
    down_bytes = case.d_ff * n * elem + e_down * (2 + elem) + case.d_model * (elem + 4) + 4 + n * case.d_model * elem
    return {"up": {"bytes": up_bytes, "flops": 2.0 * e_up * n}, "down": {"bytes": down_bytes, "flops": 2.0 * e_down * n}}


def forward_record(ctx: Context, name: str, cpu_seconds: float) -> dict | None:
    torch, args = ctx.torch, ctx.args
    from hffn_b200 import _native as native
    from hffn_b200 import synth
    from hffn_b200.distributed import sharded_runtime
    from hffn_b200.pipeline import HostPipeline, runtime_forward
    from hffn_b200.runtime import HFFNRuntime
    from oracle import forward64

    workload = WORKLOADS[name]
    rank, world, device, stream = ctx.rank, ctx.world, ctx.device, ctx.stream
    case = synth.CASES[workload["case"]]
    n = workload["n"]
    dtype = torch.float32 if workload["dtype"] == "fp32" else torch.bfloat16
    elem = 4 if dtype == torch.float32 else 2
    layer = synth.make_layer(case)
    tensor_cores = False if args.path == "cuda_cores" else None
    if world == 1:
        runtime = HFFNRuntime([kernel_layer(layer, torch)], device, dtype, tensor_cores=tensor_cores,
                              tc_format=args.tc_format if dtype == torch.float32 else None)
        shard, (lo, hi) = None, (0, case.d_ff)
    else:
        runtime, shard, (lo, hi) = sharded_runtime(case.d_model, canonical(layer, torch), device, dtype,
                                                   tensor_cores=tensor_cores, segments=args.segments,
                                                   comm_sms=args.comm_sms, transport=args.transport, push=args.push,
                                                   schedule=args.schedule,
                                                   tc_format=args.tc_format if dtype == torch.float32 else None)
    if args.path == "tensor_cores":
        runtime.force("tc", "tc")
    d, f_local = case.d_model, hi - lo
    n_kernel = n * world                       # a shard runs every rank's batch through its neurons
    x_np = rank_input(case, n, rank)
    x = torch.from_numpy(x_np).to(dtype).to(device)
    x_all = torch.from_numpy(np.concatenate([rank_input(case, n, k) for k in range(world)])).to(dtype).to(device) \
        if world > 1 else x
    runtime.forward(0, x_all)
    up, down = runtime.modes(n_kernel)
    code, struct = runtime._code, runtime._structs[0]
    handle = stream.cuda_stream
    tc = up == "tc"
    ptr = lambda v: None if v is None else v.data_ptr()  # noqa: E731
    if tc:
        tc_format, dense_struct = runtime.forward_operands(0)
        dense, work, err = runtime._dense[0], runtime._tc_work.data_ptr(), runtime._err.data_ptr()
        if tc_format == "tf32x3":
            x_split, act_hi = work, work + 2 * n_kernel * d * 4
            act_lo = act_hi + n_kernel * f_local * 4
        else:
            x_split, act_hi, act_lo = None, work, None

    def kernels(marks):
        """The two kernels of one forward of the local runtime over x_all, an event between them."""
        if tc and tc_format == "f16x3":
            native.check(native.lib.hffn_up_f16x3(x_all.data_ptr(), dense_struct, struct.b_up, None, work, err, d,
                                                  f_local, n_kernel, handle), "hffn_up_f16x3")
            marks[1].record(stream)
            native.check(native.lib.hffn_down_f16x3(work, dense_struct, struct.b_down, runtime._y.data_ptr(), err, d,
                                                    f_local, n_kernel, handle), "hffn_down_f16x3")
            return
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

    # kernel loop: the local forward's two kernels with per-kernel events (the roofline's timing). The timed step is
    # the product call without the middle event (one GPU: runtime.forward, whose float32 tensor-core kernels are
    # chained by programmatic dependent launches that an event between them would serialise; several GPUs: the
    # sharded forward)
    for marks in ctx.events(args.warmup, 3):
        ctx.flush.zero_()
        marks[0].record(stream)
        kernels(marks)
    kernel_events = ctx.events(args.steps, 3)
    ctx.barrier()
    step_events, step_ms_pipelined = None, None
    with ClockSampler(ctx.local) as clocks:
        for marks in kernel_events:
            ctx.flush.zero_()
            marks[0].record(stream)
            kernels(marks)
            marks[2].record(stream)
        torch.cuda.synchronize(device)
        if world == 1:
            for _ in range(args.warmup):
                ctx.flush.zero_()
                runtime.forward(0, x)
            step_events = ctx.events(args.steps)
            for marks in step_events:
                ctx.flush.zero_()
                marks[0].record(stream)
                runtime.forward(0, x)
                marks[1].record(stream)
            torch.cuda.synchronize(device)
        elif world > 1 and args.transport == "peer":
            # the sharded steps as one pipelined stream of batches (forward_many): batch k's gathers and batch
            # k - 2's deliveries run on the copy engines during batch k - 1's GEMMs; each step's working set
            # (gathered batches, activations, partial outputs) exceeds L2, which is not flushed inside the stream
            shard.forward_many([x] * args.warmup)
            ctx.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            shard.forward_many([x] * args.steps)
            b.record(stream)
            torch.cuda.synchronize(device)
            step_ms_pipelined = a.elapsed_time(b) / args.steps
        elif world > 1:
            # the sharded step: gather / compute / reduce pipeline over the ranks' batches
            for _ in range(args.warmup):
                ctx.flush.zero_()
                shard.forward(x)
            step_events = ctx.events(args.steps)
            ctx.barrier()
            for marks in step_events:
                ctx.flush.zero_()
                marks[0].record(stream)
                shard.forward(x)
                marks[1].record(stream)
            torch.cuda.synchronize(device)
    ctx.barrier()
    up_ms = [e[0].elapsed_time(e[1]) for e in kernel_events]
    down_ms = [e[1].elapsed_time(e[2]) for e in kernel_events]
    if step_ms_pipelined is not None:
        step_ms = [step_ms_pipelined] * args.steps
    elif step_events is not None:
        step_ms = [e[0].elapsed_time(e[1]) for e in step_events]
    else:
        step_ms = [e[0].elapsed_time(e[2]) for e in kernel_events]

    # parity: this rank's output rows against the float64 oracle (tokens are independent: a subset of rows). bf16
    # storage: the oracle of what the runtime holds (weights and inputs rounded to bf16), so the bound measures the
    # kernels' arithmetic; the distance to the float32 layer's oracle is reported beside it
    y_dev = runtime.forward(0, x) if world == 1 else shard.forward(x)
    rows = min(PARITY_ROWS, n)
    got = y_dev[:rows].float().cpu().numpy()
    if elem == 4:
        error, error_fp32_layer = relative_error(got, forward64.forward(layer, x_np[:rows])), None
    else:
        error = relative_error(got, forward64.forward(bf16_held(layer, torch), bf16_rounded(x_np[:rows], torch)))
        error_fp32_layer = relative_error(got, forward64.forward(layer, x_np[:rows]))
    bound = FP32_RELATIVE if elem == 4 else BF16_RELATIVE

    # end to end through the public API: every step copies its batch from pinned host memory to the device, runs the
    # forward and copies the output back to pinned host memory; HostPipeline overlaps step k's kernels with the copy
    # in of step k + 1 and the copy out of step k - 1. Timed from the first copy in to the last copy out. Three
    # windows as a user runs it and three with the 512 MiB L2 flush queued before every step's kernels (the flush's own
    # time included), alternating; the medians are reported.
    if world == 1:
        device_forward = runtime_forward(runtime, 0)
    else:
        def device_forward(x_dev, out):
            out.copy_(shard.forward(x_dev))
    x_hosts = [torch.from_numpy(rank_input(case, n, rank + 97 * k)).to(dtype).pin_memory() for k in range(2)]
    y_hosts = [torch.empty(n, d, dtype=dtype).pin_memory() for _ in range(max(args.steps, args.warmup))]

    def e2e_window(flushed: bool) -> float:
        forward = device_forward
        if flushed:
            def forward(x_dev, out):
                ctx.flush.zero_()
                device_forward(x_dev, out)
        pipe = HostPipeline(forward, d, d, n, dtype, device)
        pipe.run([x_hosts[k % 2] for k in range(args.warmup)], y_hosts[:args.warmup])
        ctx.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        pipe.run([x_hosts[k % 2] for k in range(args.steps)], y_hosts[:args.steps], wait=False)
        b.record(stream)
        b.synchronize()
        return ctx.max_over_ranks([a.elapsed_time(b) / 1e3])[0]

    windows = {False: [], True: []}
    for k in range(6):
        windows[k % 2 == 1].append(e2e_window(k % 2 == 1))
    e2e_ok = all(torch.equal(y_hosts[k], y_hosts[k % 2]) for k in range(2, args.steps))
    y_dev_buf = torch.empty(n, d, dtype=dtype, device=device)
    roof_s = host_link_roof(ctx, x_hosts[0], torch.empty_like(x_hosts[0], device=device), y_hosts[0], y_dev_buf,
                            args.steps)
    total_s, error, error_fp32_layer = ctx.max_over_ranks([sum(step_ms) / 1e3, error, error_fp32_layer or 0.0])
    errors = runtime.device_errors()
    cpu = cpu_forward_baseline(case, x_np, cpu_seconds) if rank == 0 and world == 1 and cpu_seconds > 0 else None
    gemm = ctx.gemm_peaks() if rank == 0 else None
    ctx.barrier()
    if rank != 0:
        return None

    pk, pk_source = peaks()
    local_case = type(case)(case.name, d, f_local, case.up_degree, case.down_degree, False, case.seed)
    alg = algorithmic(local_case, n_kernel, elem)
    kernel_ms = {"up": statistics.mean(up_ms), "down": statistics.mean(down_ms)}
    top = max(kernel_ms, key=kernel_ms.get)
    seconds = kernel_ms[top] / 1e3
    achieved_gbs = alg[top]["bytes"] / seconds / 1e9
    achieved_tflops = alg[top]["flops"] / seconds / 1e12
    hbm = {"achieved_gbs": achieved_gbs, "peak_gbs": pk["hbm_gbs"], "frac": achieved_gbs / pk["hbm_gbs"],
           "algorithmic_bytes": alg[top]["bytes"], "note": "of measured"}
    if tc:
        passes = 3 if elem == 4 else 1
        dense_flops = 2.0 * n_kernel * f_local * d * passes
        tf32 = tc_format == "tf32x3"
        pipe_peak = gemm["tf32_tflops"] if tf32 else pk["bf16_tflops"]
        traffic, traffic_source = NCU_TRAFFIC.get((name, f"tc_gemm_{top}", tc_format), (None, None)) \
            if world == 1 else (None, None)
        roofline = {"bound": "tensor", "kernel": f"tc_gemm_{top}", "achieved": achieved_tflops,
                    "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved_tflops / pk["bf16_tflops"],
                    "traffic": traffic, "traffic_source": traffic_source,
                    "algorithmic_flops": alg[top]["flops"], "launch_ms": kernel_ms[top], "peak_source": pk_source,
                    "note": "useful sparse FLOPs (2 per edge per token) of measured dense bf16 burst",
                    "tensor_pipe": {"kind": {"tf32x3": "tf32 x3 (3xTF32 split)",
                                             "f16x3": "f16 x3 (scaled fp16 hi / lo split, three products)",
                                             "bf16": "bf16"}[tc_format],
                                    "executed_tflops": dense_flops / seconds / 1e12, "peak_tflops": pipe_peak,
                                    "peak_source": gemm["source"] + ", TF32 on" if tf32 else
                                    "MEASURED_PEAKS.json dense bf16 burst (the f16 rate)",
                                    "frac": dense_flops / seconds / 1e12 / pipe_peak},
                    "hbm": hbm}
        launches = 3 if elem == 4 else 2
    else:
        roofline = {"bound": "hbm", "kernel": f"{top}_{up if top == 'up' else down}", "achieved": achieved_gbs,
                    "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved_gbs / pk["hbm_gbs"], "traffic": None,
                    "algorithmic_bytes": alg[top]["bytes"], "launch_ms": kernel_ms[top], "peak_source": pk_source,
                    "fp32_cuda_cores": {"achieved_tflops": achieved_tflops, "peak_tflops": gemm["fp32_simt_tflops"],
                                        "frac": achieved_tflops / gemm["fp32_simt_tflops"], "peak_source": gemm["source"]}}
        launches = 2
    if world == 1:
        parallelism = "single"
    elif args.transport == "peer":
        parallelism = (f"neuron-sharded x{world} (NVLink peer memory, pipelined over batches: copy-engine gathers, "
                       f"partial outputs delivered into the owners' slots by "
                       f"{'the down GEMM epilogue' if args.push == 'store' else 'copy engines'})")
    else:
        parallelism = (f"neuron-sharded x{world} (all-gather / reduce-scatter pipeline over NCCL, {shard.segments} "
                       f"segments, {shard.comm_sms} SMs left to NCCL)" if shard.schedule == "collective" else
                       f"neuron-sharded x{world} (own tokens first while the inputs cross by NCCL point-to-point, "
                       f"then the peers' tokens and their partial outputs sent to their owners, summed in rank "
                       f"order; {shard.comm_sms} SMs left to NCCL during the first call)")
    e2e_s = statistics.median(windows[False])
    bytes_in, bytes_out = x_hosts[0].numel() * elem, y_hosts[0].numel() * elem
    tokens = n * world * args.steps
    record = {
        "metric": f"HFFN FFN layer tokens/s (forward, {workload['dtype']})",
        "value": tokens / total_s, "unit": "tokens/s", "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total_s / args.steps, "dtype": "f32" if elem == 4 else "bf16",
        "config": {"workload": f"{case.name}: d_model {d}, d_ff {case.d_ff}, support {case.up_degree} of {d}, "
                               f"N {n} tokens per GPU per step", "modes": [up, down], "parallelism": parallelism,
                   "l2": "flushed between steps (512 MiB write)"},
        "roofline": roofline,
        "kernels_ms": kernel_ms,
        "e2e": {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_out,
                "pipelined": "copy in of step k+1 and copy out of step k-1 overlap step k's kernels (HostPipeline)",
                "windows_s": windows[False], "l2": "not flushed: every step's batch arrives by a fresh host-to-device "
                                                   "copy and the step's working set exceeds L2",
                "value_l2_flushed": tokens / statistics.median(windows[True]),
                "host_link_roof": tokens / roof_s, "frac_of_roof": roof_s / e2e_s,
                "roof_note": "the same pinned copies alone (in and out on two streams) on all GPUs at once",
                "outputs_repeatable": e2e_ok},
        "parity": {"max_rel": error, "bound": bound, "ok": error <= bound and e2e_ok,
                   "against": f"float64 oracle on {rows} token rows of every rank's batch"
                              + ("" if elem == 4 else " (layer and inputs as held in bf16)")},
        "gpu_launches": launches * args.steps,
        "device_errors": errors,
        "clocks": clocks.summary(),
    }
    if elem == 2:
        record["parity"]["max_rel_vs_fp32_layer"] = error_fp32_layer
    record["kernel_loop_ms_per_step"] = statistics.mean(a + b for a, b in zip(up_ms, down_ms))
    if cpu is not None:
        record["cpu_baseline"] = cpu
    return record


# -- the training step -------------------------------------------------------------------------------------------
def train_parity(ctx: Context) -> dict:
    """The data-parallel tensor-core step (one GPU: the plain step) on 256 tokens per rank of a reference test layer,
    its compact gradients (after the all-reduce) against the float64 oracle of the concatenated batch."""
    torch = ctx.torch
    from hffn_b200 import synth
    from hffn_b200.distributed import DataParallelTrainer
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    from oracle import train64
    case = synth.TEST_CASES["homog_512_2048"]
    layer = synth.make_layer(case)
    n = 256
    xs = [rank_input(case, n, r) for r in range(ctx.world)]
    ts = [rank_target(case, n, r) for r in range(ctx.world)]
    train = HFFNTrainRuntime(HFFNRuntime([kernel_layer(layer, torch)], ctx.device), **train64.HYPER, max_tokens=n,
                             tensor_cores=True)
    x, t = (torch.from_numpy(a[ctx.rank]).to(ctx.device) for a in (xs, ts))
    if ctx.world > 1:
        DataParallelTrainer(train).step_mse(0, x, t)
    else:
        train.step_mse(0, x, t)
    grads = {k: v.double().cpu().numpy() for k, v in train.gradients(0).items()}
    ref = train64.step_groups(layer, np.concatenate(xs), train64.mse_upstream(np.concatenate(ts), n * ctx.world))
    perm = np.argsort(layer.down_idx.astype(np.int64), kind="stable")
    expected = {"up_val": ref["g_up"], "b_up": ref["gb_up"], "out_val": ref["g_down"][perm], "b_down": ref["gb_down"]}
    error = max(float(np.max(np.abs(grads[k] - expected[k])) / np.abs(expected[k]).max()) for k in expected)
    error = ctx.max_over_ranks([error])[0]
    return {"max_rel": error, "bound": FP32_RELATIVE, "ok": error <= FP32_RELATIVE,
            "against": f"float64 oracle of the {ctx.world} x {n}-token concatenated batch ({case.name}, tensor-core "
                       f"step{', data parallel: gradients after the all-reduce' if ctx.world > 1 else ''}): the four "
                       f"compact gradients, max |g - g64| / max |g64|"}


def train_record(ctx: Context, name: str, cpu_tokens: int) -> dict | None:
    """The MSE training step (d_model 2048, d_ff 8192, 80 %, N per GPU), data parallel over ranks."""
    torch, args = ctx.torch, ctx.args
    from hffn_b200 import synth
    from hffn_b200.distributed import DataParallelTrainer
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime

    workload = WORKLOADS[name]
    rank, world, device, stream = ctx.rank, ctx.world, ctx.device, ctx.stream
    case = synth.CASES[workload["case"]]
    n = workload["n"]
    layer = synth.make_layer(case)
    runtime = HFFNRuntime([kernel_layer(layer, torch)], device, tensor_cores=False if args.path == "cuda_cores" else None,
                          tc_format=args.tc_format)
    train = HFFNTrainRuntime(runtime, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, max_tokens=n,
                             store_gradients=world > 1,
                             tensor_cores={"cuda_cores": False, "tensor_cores": True}.get(args.path))
    tc = train.uses_tensor_cores(0, n)
    tc_format = runtime.tc_format
    train.reserve(n)
    x_host = torch.from_numpy(rank_input(case, n, rank)).pin_memory()
    target_host = torch.from_numpy(rank_target(case, n, rank)).pin_memory()
    x, target = x_host.to(device), target_host.to(device)
    dp = DataParallelTrainer(train) if world > 1 else None
    step = (lambda: dp.step_mse(0, x, target)) if dp else (lambda: train.step_mse(0, x, target))
    for _ in range(args.warmup):
        step()
    marks = ctx.events(args.steps)
    ctx.barrier()
    with ClockSampler(ctx.local) as clocks:
        for a, b in marks:
            a.record(stream)
            loss = step()
            b.record(stream)
        torch.cuda.synchronize(device)
    ctx.barrier()
    step_ms = [a.elapsed_time(b) for a, b in marks]
    # end to end: every step copies its batch and target in from pinned host memory and reads the loss back
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
    total_s, e2e_step_s = ctx.max_over_ranks([sum(step_ms) / 1e3, statistics.median(e2e_ms) / 1e3])
    errors = runtime.device_errors()
    del train, runtime, dp
    torch.cuda.empty_cache()
    parity = train_parity(ctx)
    cpu = cpu_train_baseline(case, layer, cpu_tokens, 2) if rank == 0 and world == 1 and cpu_tokens > 0 else None
    gemm = ctx.gemm_peaks() if rank == 0 else None
    ctx.barrier()
    if rank != 0:
        return None
    pk, pk_source = peaks()
    e = case.d_ff * case.up_degree
    flops = 12.0 * e * n                       # forward 2 x 2En, backward 2x the forward
    step_bytes = (4 * n * case.d_model * 4      # x, target, gy, gx
                  + 2 * case.d_ff * n * 4 * 2   # z written and read
                  + 2 * e * 6 * 2               # both supports (index + value), forward and backward
                  + 2 * e * 24)                 # AdamW: p, m, v read and written, both value arrays
    seconds = total_s / args.steps
    achieved = step_bytes / seconds / 1e9
    hbm = {"achieved_gbs": achieved, "peak_gbs": pk["hbm_gbs"], "frac": achieved / pk["hbm_gbs"],
           "algorithmic_bytes": step_bytes}
    simt = {"achieved_tflops": flops / seconds / 1e12, "peak_tflops": gemm["fp32_simt_tflops"],
            "frac": flops / seconds / 1e12 / gemm["fp32_simt_tflops"], "peak_source": gemm["source"]}
    if tc:
        dense_flops = 6 * 2.0 * case.d_model * case.d_ff * n * 3      # six GEMMs, three passes each
        if tc_format == "f16x3":
            # four GEMMs (up, down + MSE, W_down^T gy, W_up^T gz) run at the f16 rate, the two sampled weight-gradient
            # GEMMs at the tf32 rate: the pipe's peak for this mix is the harmonic blend (each GEMM a sixth of the work)
            pipe_peak = 1.0 / ((2 / 3) / pk["bf16_tflops_sustained"] + (1 / 3) / gemm["tf32_tflops"])
            pipe = {"kind": "f16 x3 (up, down + MSE, W_down^T gy, W_up^T gz) and tf32 x3 (the two sampled "
                            "weight-gradient GEMMs)",
                    "peak_source": "blend of MEASURED_PEAKS.json dense bf16 sustained (f16 rate) for 2/3 of the work and "
                                   + gemm["source"] + ", TF32 on, for 1/3"}
        else:
            pipe_peak = gemm["tf32_tflops"]
            pipe = {"kind": "tf32 x3 (3xTF32 split)", "peak_source": gemm["source"] + ", TF32 on"}
        pipe.update(executed_tflops=dense_flops / seconds / 1e12, peak_tflops=pipe_peak,
                    frac=dense_flops / seconds / 1e12 / pipe_peak)
        roofline = {"bound": "tensor", "kernel": "whole step (six tcgen05 GEMMs)", "achieved": flops / seconds / 1e12,
                    "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                    "frac": flops / seconds / 1e12 / pk["bf16_tflops_sustained"], "traffic": None,
                    "algorithmic_flops": flops, "peak_source": pk_source,
                    "note": "useful sparse FLOPs of measured dense bf16 sustained (a step of milliseconds)",
                    "tensor_pipe": pipe, "hbm": hbm, "fp32_cuda_cores": simt}
    else:
        roofline = {"bound": "hbm", "kernel": "whole step", "achieved": achieved, "peak": pk["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": None,
                    "algorithmic_bytes": step_bytes, "peak_source": pk_source, "fp32_cuda_cores": simt}
    record = {
        "metric": "HFFN FFN layer tokens/s (train step, fp32)", "value": n * world * args.steps / total_s,
        "unit": "tokens/s", "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * seconds, "dtype": "f32",
        "config": {"workload": f"{case.name}: d_model {case.d_model}, d_ff {case.d_ff}, support {case.up_degree} of "
                               f"{case.d_model}, N {n} tokens per GPU per step, MSE loss, AdamW",
                   "path": "tensor_cores" if tc else "cuda_cores",
                   "parallelism": f"data parallel x{world}, gradient all-reduce over NCCL" if world > 1 else "single",
                   "l2": "inputs larger than L2 (z and act alone 537 MB)"},
        "roofline": roofline,
        "e2e": {"value": n * world / e2e_step_s, "unit": "tokens/s", "h2d_bytes_per_step": 2 * x_host.numel() * 4,
                "d2h_bytes_per_step": loss_host.numel() * 4, "step": "copies in, the step, the loss read back; median"},
        "parity": parity,
        "gpu_launches": (10 if tc else 8) * args.steps, "device_errors": errors, "clocks": clocks.summary(),
        "loss_last": float(loss_host),
    }
    if cpu is not None:
        record["cpu_baseline"] = cpu
    return record


# -- decode ----------------------------------------------------------------------------------------------------------
def decode_record(ctx: Context, name: str, cpu_seconds: float) -> dict | None:
    """The decode FFN step of the Pythia-410M shape: 24 layers (C4: d_model 1024, d_ff 4096, 50 % supports, bf16),
    8 tokens per call, one call per layer, through ``PreparedRuntime`` (the decode path: prepared per (layer, N),
    the cooperative kernels), the 24 calls of a step replayed as one CUDA graph. Every layer has its own copy of the
    compact arrays in HBM (403 MB of edge streams per step, above L2: no flush needed). HBM-bound: the roofline is
    the algorithmic bytes of the 48 kernels (edges, offsets, biases, x, act, y) per step over the step time. Replicas
    only: with N > 1 every rank runs its own copy."""
    torch, args = ctx.torch, ctx.args
    from hffn_b200 import _native as native
    from hffn_b200 import synth
    from hffn_b200.runtime import PreparedRuntime
    from oracle import forward64, x86ref
    workload = WORKLOADS[name]
    rank, world, device, stream = ctx.rank, ctx.world, ctx.device, ctx.stream
    case = synth.CASES[workload["case"]]
    layers_n, n = workload["layers"], workload["n"]
    layer = synth.make_layer(case)
    runtime = PreparedRuntime([kernel_layer(layer, torch)] * layers_n, device, torch.bfloat16)
    d = case.d_model
    x_host = torch.from_numpy(np.stack([rank_input(case, n, rank + 31 * k) for k in range(layers_n)])).to(
        torch.bfloat16).pin_memory()
    x = x_host.to(device)

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
    ctx.barrier()
    with ClockSampler(ctx.local) as clocks:
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
    # parity: layer 0's output against the float64 oracle of the layer and input the runtime holds (bf16 values)
    held = bf16_held(layer, torch)
    first = runtime.forward(0, x[0]).clone()
    repeat = bool(torch.equal(first, runtime.forward(0, x[0])))
    error = relative_error(first.float().cpu().numpy(), forward64.forward(held, x_host[0].float().numpy()))
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
    step_s, e2e_s, error = ctx.max_over_ranks([graph_ms / 1e3, statistics.median(e2e) / 1e3, error])
    errors = runtime.device_errors()
    cpu = None
    if rank == 0 and world == 1 and cpu_seconds > 0 and x86ref.available():
        threads = host_threads()
        kernel = x86ref.X86Kernel(layer, threads=threads)
        xs = x_host.float().numpy()
        kernel.forward(xs[0])
        steps, start = 0, time.perf_counter()
        while time.perf_counter() - start < cpu_seconds:
            for index in range(layers_n):
                kernel.forward(xs[index])
            steps += 1
        elapsed = time.perf_counter() - start
        cpu = {"value": steps * n * layers_n / elapsed, "unit": "layer-tokens/s", "cores": threads,
               "kind": "reference", "sample": f"{steps} decode steps (24 calls of 8 tokens, float32: the reference "
                                              f"kernel's only type), {elapsed:.1f} s"}
    ctx.barrier()
    if rank != 0:
        return None
    pk, pk_source = peaks()
    alg = algorithmic(case, n, 2)
    step_bytes = layers_n * (alg["up"]["bytes"] + alg["down"]["bytes"])
    achieved = step_bytes / step_s / 1e9
    record = {
        "metric": "HFFN FFN layer tokens/s (decode, bf16)", "value": n * layers_n * world / step_s,
        "unit": "layer-tokens/s", "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "dtype": "bf16",
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
        "parity": {"max_rel": error, "bound": BF16_RELATIVE, "ok": error <= BF16_RELATIVE and repeat,
                   "against": "float64 oracle of the bf16-held layer 0 on its 8 tokens, same bits on repeat"},
        "gpu_launches": 2 * layers_n * args.steps, "device_errors": errors, "clocks": clocks.summary(),
    }
    if cpu is not None:
        record["cpu_baseline"] = cpu
    return record


# -- the model ---------------------------------------------------------------------------------------------------------
def pythia_record(ctx: Context, name: str) -> dict | None:
    """The Pythia-410M architecture (random init, 50 % HFFN FFNs, bfloat16): prefill of batch x prompt tokens, then
    greedy decode steps with the KV cache; the HFFN arm and the dense arm (the model's own MLP with the same weights
    on the support) timed back to back on the same prompts."""
    import tempfile
    torch, args = ctx.torch, ctx.args
    from hffn_b200 import pythia
    workload = WORKLOADS[name]
    device, stream = ctx.device, ctx.stream
    root = Path(tempfile.gettempdir()) / "hffn_bench_pythia410m"
    if not (root / "model" / "model.safetensors").exists():
        pythia.make_random_pythia(root / "model", root / "export", pythia.PYTHIA_410M, support=512, seed=3004)
    b, t, steps = workload["batch"], workload["prompt"], workload["decode"]
    g = torch.Generator().manual_seed(3004)
    prompt = torch.randint(0, 50277, (b, t), generator=g).to(device)
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
            "value": tokens / ((h["prefill_ms"] + h["decode_ms"]) / 1e3), "unit": "tokens/s",
            "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
            "config": {"workload": "pythia-410m architecture, 24 layers, d_model 1024, d_ff 4096, 512-of-1024 supports"},
            "prefill_tokens_per_s": {"hffn": b * t / (h["prefill_ms"] / 1e3), "dense": b * t / (d["prefill_ms"] / 1e3)},
            "decode_tokens_per_s": {"hffn": b * steps / (h["decode_ms"] / 1e3), "dense": b * steps / (d["decode_ms"] / 1e3)},
            "arms_ms": results} if ctx.rank == 0 else None


def c5_record(ctx: Context, name: str) -> dict | None:
    """Pythia-1B architecture (random init, 20 % HFFN FFNs, bfloat16), prefill of 64 x 2048 tokens; with N ranks every
    FFN is neuron-sharded 1/N per GPU (``load_pythia(group=...)``: the rank's shard on the tensor cores, the partial
    outputs all-reduced over NCCL) and the rest of the model replicated, every rank running the same batch (strong
    scaling: the job's throughput is the batch over the step). Beside the step: the shard's two FFN kernels timed alone
    on the step's FFN input shape (the roofline), one all-reduce of an FFN output, and the parity of the sharded layer-0
    FFN on 64 token rows against the float64 oracle of the layer as held in bf16."""
    import tempfile
    torch, args = ctx.torch, ctx.args
    from hffn_b200 import pythia, synth
    from oracle import forward64
    workload = WORKLOADS[name]
    rank, world, device, stream = ctx.rank, ctx.world, ctx.device, ctx.stream
    b, t = workload["batch"], workload["prompt"]
    arch = pythia.PYTHIA_1B
    root = Path(tempfile.gettempdir()) / "hffn_bench_pythia1b"
    if rank == 0 and not (root / "model" / "hffn_random_init.json").exists():
        pythia.make_random_pythia(root / "model", root / "export", arch, support=workload["support"],
                                  seed=workload["seed"])
    ctx.barrier()
    group = ctx.dist.group.WORLD if world > 1 else None
    model = pythia.load_pythia(root / "model", root / "export", "hffn", device, torch.bfloat16, group=group)
    prompt_host = torch.randint(0, 50277, (b, t), generator=torch.Generator().manual_seed(workload["seed"])).pin_memory()
    prompt = prompt_host.to(device)
    logits_host = torch.empty(b, 1, arch["vocab_size"], dtype=torch.bfloat16).pin_memory()

    @torch.inference_mode()
    def step(ids):
        return model(input_ids=ids, use_cache=False, logits_to_keep=1).logits

    for _ in range(args.warmup):
        step(prompt)
    marks = ctx.events(args.steps)
    ctx.barrier()
    with ClockSampler(ctx.local) as clocks:
        for a, e in marks:
            a.record(stream)
            step(prompt)
            e.record(stream)
        torch.cuda.synchronize(device)
    step_ms = [a.elapsed_time(e) for a, e in marks]
    e2e = []
    for _ in range(args.steps):               # token ids in from pinned host memory, last-position logits back
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        prompt.copy_(prompt_host, non_blocking=True)
        logits_host.copy_(step(prompt), non_blocking=True)
        e.record(stream)
        e.synchronize()
        e2e.append(a.elapsed_time(e))
    # the rank's FFN kernels alone (layer 0's runtime, the step's FFN input shape), and one all-reduce of its output
    runtime = model.hffn_runtime
    x = torch.randn(b * t, arch["hidden_size"], generator=torch.Generator().manual_seed(7)).to(device, torch.bfloat16)
    runtime.forward(0, x)
    kernel_ms, reduce_ms = [], []
    for _ in range(3):
        a, m, e = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(stream)
        y = runtime.forward(0, x)
        m.record(stream)
        if world > 1:
            ctx.dist.all_reduce(y, op=ctx.dist.ReduceOp.SUM)
        e.record(stream)
        e.synchronize()
        kernel_ms.append(a.elapsed_time(m))
        reduce_ms.append(m.elapsed_time(e))
    # parity: the (sharded) layer-0 FFN on 64 rows against the float64 oracle of the layer as held in bf16
    case0 = synth.Case("pythia_layer0", arch["hidden_size"], arch["intermediate_size"], workload["support"],
                       workload["support"], False, workload["seed"], 0.02)
    rows = torch.randn(PARITY_ROWS, arch["hidden_size"], generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    with torch.inference_mode():
        y_rows = model.gpt_neox.layers[0].mlp(rows.to(device).unsqueeze(0)).squeeze(0).float().cpu().numpy()
    error = relative_error(y_rows, forward64.forward(bf16_held(synth.make_layer(case0), torch), rows.float().numpy())) \
        if rank == 0 else 0.0
    total_s, e2e_s, kernel_s, reduce_s, error = ctx.max_over_ranks(
        [sum(step_ms) / 1e3, statistics.median(e2e) / 1e3, statistics.median(kernel_ms) / 1e3,
         statistics.median(reduce_ms) / 1e3, error])
    errors = runtime.device_errors()
    ctx.barrier()
    if rank != 0:
        return None
    pk, pk_source = peaks()
    shard_edges = sum(int(s.numel()) for s in (runtime._tensors[0]["up_val"], runtime._tensors[0]["out_val"]))
    flops = 2.0 * shard_edges * b * t                       # useful: 2 per edge per token, both projections
    achieved = flops / kernel_s / 1e12
    tokens = b * t
    return {
        "metric": "Pythia-1B (20 % HFFN FFNs, bf16) prefill tokens/s: 64 x 2048 tokens, FFNs neuron-sharded over the GPUs",
        "value": tokens * args.steps / total_s, "unit": "tokens/s", "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total_s / args.steps, "dtype": "bf16", "scaling": "strong",
        "config": {"workload": f"pythia-1b architecture (random init), {arch['num_hidden_layers']} layers, d_model "
                               f"{arch['hidden_size']}, d_ff {arch['intermediate_size']}, {workload['support']}-of-"
                               f"{arch['hidden_size']} supports; prefill {b} x {t}, last-position logits",
                   "parallelism": "single" if world == 1 else
                   f"every FFN neuron-sharded 1/{world} per GPU, partial outputs all-reduced over NCCL; attention, "
                   f"embeddings and head replicated", "l2": "inputs larger than L2 (hidden states 537 MB per layer)"},
        "roofline": {"bound": "tensor", "kernel": "the rank's FFN shard (tc_gemm up + down, layer 0, the step's shape)",
                     "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["bf16_tflops"], "traffic": None, "launch_ms": kernel_s * 1e3,
                     "peak_source": pk_source, "note": "useful sparse FLOPs (2 per edge per token) of measured dense "
                                                       "bf16 burst; the dense tiles execute 1 / density of that"},
        "all_reduce": {"ms": reduce_s * 1e3, "bytes": tokens * arch["hidden_size"] * 2,
                       "bus_gbs": (2 * (world - 1) / world * tokens * arch["hidden_size"] * 2 / reduce_s / 1e9)
                       if world > 1 else None},
        "ffn_ms_per_step": (kernel_s + reduce_s) * 1e3 * arch["num_hidden_layers"],
        "e2e": {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": prompt_host.numel() * 8,
                "d2h_bytes_per_step": logits_host.numel() * 2},
        "parity": {"max_rel": error, "bound": BF16_RELATIVE, "ok": error <= BF16_RELATIVE,
                   "against": "float64 oracle of layer 0 (as held in bf16) on 64 token rows, through the sharded FFN"},
        "gpu_launches": 2 * arch["num_hidden_layers"] * args.steps, "device_errors": errors,
        "clocks": clocks.summary(),
    }


# -- driver ------------------------------------------------------------------------------------------------------------
def single(ctx: Context, name: str) -> dict | None:
    args = ctx.args
    if name.startswith("train"):
        return train_record(ctx, name, 0 if args.no_cpu_baseline else args.cpu_train_tokens)
    if name == "decode":
        return decode_record(ctx, name, 0 if args.no_cpu_baseline else args.cpu_seconds / 2)
    if name == "pythia410m":
        return pythia_record(ctx, name)
    if name == "c5":
        return c5_record(ctx, name)
    return forward_record(ctx, name, 0 if args.no_cpu_baseline else args.cpu_seconds)


def finish(ctx: Context, record: dict) -> dict:
    """The line's contract fields around a record."""
    line = {"metric": record["metric"], "value": record["value"], "unit": record["unit"], "n_gpus": ctx.world,
            "steps": record["steps"], "warmup": record["warmup"], "ms_per_step": record.get("ms_per_step"),
            "higher_is_better": True, "scaling": record.get("scaling", "weak"), "vs_baseline": None,
            "dtype": record["dtype"],
            "data": "synthetic (seeded supports, weights and inputs of the benchmark plan's shapes)"}
    line.update({k: v for k, v in record.items() if k not in line})
    return line


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("hffn", "reference"), default="hffn")
    parser.add_argument("--workload", choices=("all", *WORKLOADS), default="all")
    parser.add_argument("--cpu-seconds", type=float, default=8.0, help="forward CPU baselines: seconds per sample")
    parser.add_argument("--cpu-train-tokens", type=int, default=256, help="training CPU baseline: tokens per step")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--segments", type=int, default=None, help="sharded forward: pipeline segments per step")
    parser.add_argument("--schedule", choices=("collective", "own_first"), default="collective",
                        help="sharded forward: gather / reduce-scatter, or own tokens first with point-to-point sends")
    parser.add_argument("--comm-sms", type=int, default=0, help="sharded forward: SMs left to the collectives")
    parser.add_argument("--transport", choices=("nccl", "peer"), default="nccl",
                        help="sharded forward: NCCL collectives or NVLink peer memory (tensor cores)")
    parser.add_argument("--push", choices=("copy", "store"), default="copy",
                        help="peer sharded forward: partial outputs pushed by copy engines or by the GEMM epilogue")
    parser.add_argument("--tc-format", choices=("f16x3", "tf32x3"), default=None,
                        help="operand format of the float32 tensor-core forward and of the training step's up and "
                             "down + MSE GEMMs (default: f16x3)")
    parser.add_argument("--path", choices=("auto", "cuda_cores", "tensor_cores"), default="auto",
                        help="forward kernels: the runtime policy, the CUDA-core gather kernels, or the tcgen05 path")
    args = parser.parse_args()
    rank, world, _ = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(reference_arm(args, WORKLOADS["fwd"])), flush=True)
        return 0
    ctx = Context(args)
    try:
        if args.workload == "all":
            records = {}
            for key, name in COMPOSITE:
                if name == "c1" and ctx.world > 1:
                    continue                 # the reference's CPU-sized case: one GPU only
                if key == "c2_fwd_fp32":     # the headline: its failure is the run's
                    records[key] = single(ctx, name)
                    continue
                try:                         # a secondary record that fails (alike on every rank) leaves the others
                    records[key] = single(ctx, name)
                except Exception as error:   # noqa: BLE001
                    traceback.print_exc()
                    records[key] = {"error": f"{type(error).__name__}: {error}"}
                ctx.torch.cuda.empty_cache()
            if ctx.rank == 0:
                line = finish(ctx, records.pop("c2_fwd_fp32"))
                line["workloads"] = records
                line["parity_all_ok"] = line["parity"]["ok"] and all(r.get("parity", {}).get("ok", False)
                                                                     for r in records.values())
                print(json.dumps(line), flush=True)
        else:
            record = single(ctx, args.workload)
            if ctx.rank == 0:
                print(json.dumps(finish(ctx, record)), flush=True)
    finally:
        ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
