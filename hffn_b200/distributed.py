"""Multi-GPU HFFN on one box: hidden neurons sharded across ranks for inference, data parallelism for training.

One process per GPU, ``torch.distributed`` for the plumbing (NCCL over NVLink on GPUs; gloo on CPU for the tests).

Inference (the north star's natural shard). Rank k owns a contiguous range of hidden neurons, balanced by edge
count (up + down slots) and rounded to multiples of 8 so that every shard keeps the tensor-core path: its up slots
and biases, and the down edges of its neurons only (re-sorted output-major by ``HFFNLayer.from_hidden_major``).
``b_down`` is added by rank 0 only, so the sum over ranks of the partial outputs is the layer's output. Two forms:
- ``forward_replicated(x)``: x identical on every rank (already broadcast); partial y all-reduced; every rank gets y.
- ``forward(x_local)``: weak scaling, each rank holds its own batch. Per segment of the batch: all-gather of every
  rank's sub-batch, one call of the rank's shard over all of them, reduce-scatter of the partial outputs back to
  their ranks; the collectives are asynchronous, so the gather of the next segment and the reduction of the previous
  one overlap the compute of the current one. Every rank returns y of its own batch.
Training: data parallel over tokens with full compact replicas (``DataParallelTrainer``): forward, MSE loss on the
rank's tokens, backward with the gradients stored, one all-reduce (sum) of the four compact gradient arrays scaled
by 1 / world (the mean over all tokens), then AdamW. The fused backward + AdamW of one GPU does not apply: the update
must wait for the exchange.

Every rank calls the same collectives in the same order, in warm-up and in timing.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

GRANULE = 8


def balanced_partition(cost: torch.Tensor, parts: int, granule: int = GRANULE) -> list[int]:
    """Offsets ``[0 = b_0 <= b_1 <= ... <= b_parts = len(cost)]`` of contiguous groups of nearly equal total cost; inner
    boundaries are multiples of ``granule`` (the last group takes the remainder)."""
    count = int(cost.numel())
    cumulative = torch.cumsum(cost.to(torch.float64), 0)
    total = float(cumulative[-1]) if count else 0.0
    bounds = [0]
    for k in range(1, parts):
        target = total * k / parts
        cut = int(torch.searchsorted(cumulative, torch.tensor(target, dtype=torch.float64))) + 1
        cut = min(count, max(bounds[-1], int(round(cut / granule)) * granule))
        bounds.append(cut)
    bounds.append(count)
    return bounds


def shard_hidden_major(d_model: int, arrays: dict, lo: int, hi: int, with_bias: bool) -> dict:
    """The canonical hidden-major arrays of neurons ``[lo, hi)``: offsets rebased to 0, ``b_down`` zeroed unless
    ``with_bias``. ``arrays`` holds ``b_up, up_offsets, up_idx, up_val, b_down, down_offsets, down_idx, down_val``."""
    up_off, dn_off = arrays["up_offsets"], arrays["down_offsets"]
    u0, u1 = int(up_off[lo]), int(up_off[hi])
    d0, d1 = int(dn_off[lo]), int(dn_off[hi])
    b_down = arrays["b_down"].clone() if with_bias else torch.zeros_like(arrays["b_down"])
    return {"d_model": d_model, "d_ff": hi - lo, "b_up": arrays["b_up"][lo:hi].clone(),
            "up_offsets": (up_off[lo:hi + 1] - u0).to(torch.int32), "up_idx": arrays["up_idx"][u0:u1].clone(),
            "up_val": arrays["up_val"][u0:u1].clone(), "b_down": b_down,
            "down_offsets": (dn_off[lo:hi + 1] - d0).to(torch.int32), "down_idx": arrays["down_idx"][d0:d1].clone(),
            "down_val": arrays["down_val"][d0:d1].clone()}


def neuron_partition(arrays: dict, world: int) -> list[int]:
    cost = arrays["up_offsets"].diff().long() + arrays["down_offsets"].diff().long()
    return balanced_partition(cost, world)


class ShardedFFN:
    """The collectives of the neuron-sharded forward around a rank-local forward ``local_forward(x, out)`` that writes
    the partial y of the rank's neuron shard (``b_down`` on rank 0 only) into ``out``. ``group`` None: the default
    process group."""

    def __init__(self, local_forward: Callable[[torch.Tensor, torch.Tensor], None], d_model: int, group=None,
                 segments: int | None = None, comm_sms: int = 0, packets=None, schedule: str = "collective") -> None:
        if schedule not in ("collective", "own_first"):
            raise ValueError("schedule must be 'collective' or 'own_first'")
        self.schedule = schedule
        self.local_forward = local_forward
        # packets: the rank-local fp16x3 runtime when its forward can start from token packets: each rank then splits
        # its own tokens and the packets are gathered (the same bytes as float32 x), instead of every rank splitting
        # the whole gathered batch
        self.packets = packets
        self.d_model = d_model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        # One segment by default: measured on B200 with the fp16x3 forward (C2, 4096 tokens per rank), 1 / 2 / 3 / 4
        # segments took 336 / 350 / 428 / 504 us per step on 2 GPUs and 1 / 2 / 4 took 662 / 703 / 743 us on 8: the
        # collectives of a later segment wait for SMs the persistent GEMMs hold, so cutting the batch adds launches
        # and latency without overlap (leaving 8 to 32 SMs to NCCL did not change that).
        self.segments = segments or 1
        self.comm_sms = comm_sms
        self._cuda = False
        self._buffers: dict = {}
        # The reduce-scatters run on a second communicator of the same ranks, so that they proceed concurrently with
        # the gathers (the other NVLink direction) instead of queueing behind them on one NCCL stream.
        ranks = [dist.get_global_rank(group, k) if group is not None else k for k in range(self.world)]
        self.scatter_group = dist.new_group(ranks=ranks) if self.world > 1 else group
        self._ranks = [dist.get_global_rank(group, k) if group is not None else k for k in range(self.world)]

    def forward_replicated(self, x: torch.Tensor) -> torch.Tensor:
        """``y`` of an ``x`` that every rank holds: partial outputs all-reduced (sum)."""
        y = torch.empty(x.shape[0], self.d_model, dtype=x.dtype, device=x.device)
        self.local_forward(x, y)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y

    def _limit_ctas(self, on: bool) -> None:
        """While the pipeline runs, the persistent tensor-core GEMMs leave ``comm_sms`` SMs to the NCCL kernels."""
        if self.comm_sms and x_is_cuda(self):
            from . import _native as native
            count = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
            native.lib.hffn_set_tc_max_ctas(count - self.comm_sms if on else 0)

    def forward(self, x_local: torch.Tensor, segments: int | None = None) -> torch.Tensor:
        """``y`` of this rank's own batch ``x_local`` (every rank passes a batch of the same shape).

        The batch is cut into ``segments`` sub-batches; for each, every rank's sub-batch is all-gathered, this rank's
        neuron shard runs on all of them in one call, and the partial outputs are reduce-scattered back to their
        ranks. The collectives are queued asynchronously, so the gather of segment s + 1 and the reduction of
        segment s - 1 overlap the compute of segment s."""
        if self.schedule == "own_first" and self.world > 1:
            return self._forward_own_first(x_local)
        n, d = x_local.shape[0], self.d_model
        segments = max(1, min(segments or self.segments, n))
        bounds = [n * k // segments for k in range(segments + 1)]
        packed = self.packets is not None and x_local.is_cuda and all(
            self.packets.uses_packets(self.world * (bounds[s + 1] - bounds[s])) for s in range(segments))
        key = (n, segments, x_local.dtype, x_local.device, packed)
        if key not in self._buffers:     # exchange buffers, reused by every call of this shape
            device = x_local.device
            row = (self.packets.packet_bytes(),) if packed else (d,)
            kind = torch.uint8 if packed else x_local.dtype
            self._buffers[key] = [(torch.empty(self.world * (bounds[s + 1] - bounds[s]), *row, dtype=kind,
                                               device=device),
                                   torch.empty(self.world * (bounds[s + 1] - bounds[s]), d, dtype=x_local.dtype,
                                               device=device),
                                   torch.empty(bounds[s + 1] - bounds[s], *row, dtype=kind, device=device)
                                   if packed else None) for s in range(segments)]
        buffers = self._buffers[key]
        self._cuda = x_local.is_cuda
        if segments > 1:
            self._limit_ctas(True)
        gathers = []
        for s in range(segments):
            part = x_local[bounds[s]:bounds[s + 1]]
            if packed:
                self.packets.split_packets(0, part, buffers[s][2])
                part = buffers[s][2]
            gathers.append(dist.all_gather_into_tensor(buffers[s][0], part, group=self.group, async_op=True))
        out = torch.empty(n, d, dtype=x_local.dtype, device=x_local.device)
        scatters = []
        for s in range(segments):
            gathers[s].wait()
            if packed:
                self.packets.forward_packets(0, buffers[s][0], buffers[s][1])
            else:
                self.local_forward(buffers[s][0], buffers[s][1])
            scatters.append(self._reduce_scatter(out[bounds[s]:bounds[s + 1]], buffers[s][1]))
        for work in scatters:
            if work is not None:
                work.wait()
        if segments > 1:
            self._limit_ctas(False)
        return out

    def _run(self, packed: bool, inputs: torch.Tensor, out: torch.Tensor) -> None:
        if packed:
            self.packets.forward_packets(0, inputs, out)
        else:
            self.local_forward(inputs, out)

    def _forward_own_first(self, x_local: torch.Tensor) -> torch.Tensor:
        """The ``own_first`` schedule: the rank's inputs (token packets on the fp16x3 path, else x) go to every peer
        by point-to-point sends while the shard runs on the rank's own tokens; then the shard runs on the peers'
        tokens (one call over all of them) and each peer is sent the partial outputs of its own tokens; the rank sums
        the partials of its tokens in rank order (fixed, whatever the arrival order). The same bytes cross NVLink as
        with the gather / reduce-scatter pair, but the gather overlaps the first call."""
        n, d, world, rank = x_local.shape[0], self.d_model, self.world, self.rank
        peers = [(rank + j) % world for j in range(1, world)]
        packed = self.packets is not None and x_local.is_cuda and self.packets.uses_packets(n) \
            and self.packets.uses_packets((world - 1) * n)
        key = ("own_first", n, x_local.dtype, x_local.device, packed)
        device = x_local.device
        if key not in self._buffers:
            row = (self.packets.packet_bytes(),) if packed else (d,)
            kind = torch.uint8 if packed else x_local.dtype
            self._buffers[key] = {
                "own": torch.empty(n, *row, dtype=kind, device=device) if packed else None,
                "peer_in": torch.empty((world - 1) * n, *row, dtype=kind, device=device),
                "peer_out": torch.empty((world - 1) * n, d, dtype=x_local.dtype, device=device),
                "slots": torch.empty(world, n, d, dtype=x_local.dtype, device=device)}
        buf = self._buffers[key]
        self._cuda = x_local.is_cuda
        own = x_local.contiguous()
        if packed:
            self.packets.split_packets(0, own, buf["own"])
            own = buf["own"]
        ops = []
        for j, k in enumerate(peers):
            ops.append(dist.P2POp(dist.isend, own, self._ranks[k], group=self.group))
            ops.append(dist.P2POp(dist.irecv, buf["peer_in"][j * n:(j + 1) * n], self._ranks[k], group=self.group))
        self._limit_ctas(True)
        works = dist.batch_isend_irecv(ops)
        self._run(packed, own, buf["slots"][rank])
        for work in works:
            work.wait()
        self._limit_ctas(False)
        self._run(packed, buf["peer_in"], buf["peer_out"])
        ops = []
        for j, k in enumerate(peers):
            ops.append(dist.P2POp(dist.isend, buf["peer_out"][j * n:(j + 1) * n], self._ranks[k], group=self.group))
            ops.append(dist.P2POp(dist.irecv, buf["slots"][k], self._ranks[k], group=self.group))
        for work in dist.batch_isend_irecv(ops):
            work.wait()
        return sum_in_rank_order(buf["slots"])

    def _reduce_scatter(self, out: torch.Tensor, partial: torch.Tensor):
        if dist.get_backend(self.group) == "gloo":      # gloo has no reduce-scatter: all-reduce and keep the slice
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.scatter_group)
            m = out.shape[0]
            out.copy_(partial[self.rank * m:(self.rank + 1) * m])
            return None
        return dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=self.scatter_group, async_op=True)


def sum_in_rank_order(slots: torch.Tensor) -> torch.Tensor:
    """slots[0] + slots[1] + ... in that order (float32 accumulation; ``hffn_sum_slots`` on the device)."""
    if not slots.is_cuda:
        out = slots[0].clone()
        for k in range(1, slots.shape[0]):
            out += slots[k]
        return out
    from . import _native as native
    out = torch.empty(slots.shape[1:], dtype=slots.dtype, device=slots.device)
    code = native.F32 if slots.dtype == torch.float32 else native.BF16
    native.check(native.lib.hffn_sum_slots(code, slots.data_ptr(), slots.shape[0], out.numel(), out.data_ptr(),
                                           native.stream_handle(slots.device)), "hffn_sum_slots")
    return out


def x_is_cuda(ffn: "ShardedFFN") -> bool:
    return ffn._cuda


def sharded_runtime(d_model: int, arrays: dict, device, dtype=torch.float32, tensor_cores=None, group=None,
                    segments: int | None = None, comm_sms: int = 0, transport: str = "nccl", push: str = "copy",
                    tc_format: str | None = None, schedule: str = "collective"):
    """The rank's ``HFFNRuntime`` over its neuron shard and the sharded forward around it: ``transport="nccl"`` a
    ``ShardedFFN`` (collective kernels), ``"peer"`` a ``PeerShardedFFN`` (NVLink peer memory and copy engines,
    pipelined over batches, tensor cores only, ``push`` its delivery mode)."""
    if transport not in ("nccl", "peer"):
        raise ValueError("transport must be 'nccl' or 'peer'")
    from .runtime import HFFNLayer, HFFNRuntime
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    bounds = neuron_partition(arrays, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    if hi <= lo:
        raise ValueError(f"rank {rank} owns no hidden neuron (d_ff {arrays['b_up'].numel()} over {world} ranks)")
    shard = shard_hidden_major(d_model, arrays, lo, hi, with_bias=rank == 0)
    layer = HFFNLayer.from_hidden_major(shard["d_model"], shard["d_ff"], shard["b_up"], shard["up_offsets"],
                                        shard["up_idx"], shard["up_val"], shard["b_down"], shard["down_offsets"],
                                        shard["down_idx"], shard["down_val"])
    if transport == "peer" and dtype == torch.float32:
        tc_format = "tf32x3"          # the peer pipeline's GEMMs run on the tf32 pairs
    runtime = HFFNRuntime([layer], device, dtype, tensor_cores=tensor_cores, tc_format=tc_format)
    if transport == "peer":
        return runtime, PeerShardedFFN(runtime, d_model, group, push=push), (lo, hi)
    packets = None
    if runtime.tensor_cores and runtime.tc_format == "f16x3":
        # every shard reads the packets every rank makes: their activation scales use the whole layer's bound
        l1 = torch.zeros(arrays["b_up"].numel(), dtype=torch.float64).index_add_(
            0, torch.repeat_interleave(torch.arange(arrays["b_up"].numel()), arrays["up_offsets"].cpu().diff().long()),
            arrays["up_val"].cpu().double().abs())
        runtime.up_bound_floor = torch.tensor([float(l1.max()), float(arrays["b_up"].cpu().double().abs().max())],
                                              dtype=torch.float32)
        packets = runtime
    ffn = ShardedFFN(lambda x, out: runtime.forward(0, x, out=out), d_model, group, segments=segments,
                     comm_sms=comm_sms, packets=packets, schedule=schedule)
    return runtime, ffn, (lo, hi)


class DataParallelTrainer:
    """Data-parallel MSE training step over an ``HFFNTrainRuntime`` replica per rank."""

    def __init__(self, train, group=None) -> None:
        self.train = train
        self.group = group
        self.world = dist.get_world_size(group)
        self._loss = torch.zeros(1, dtype=torch.float64, device=train.runtime.device)

    def step_mse(self, index: int, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One step on this rank's tokens; returns the mean loss over all ranks' tokens (before the update)."""
        from . import _native as native
        train = self.train
        n = train._check_tokens(target, "target")
        if train.uses_tensor_cores(index, n):
            # gradients of the mean over all ranks' tokens (n_total = world n): summed, not averaged
            train.step_mse_tc(index, x, target, n_total=n * self.world, apply=False)
            grads = train.gradients(index)
            for name in ("up_val", "b_up", "out_val", "b_down"):
                dist.all_reduce(grads[name], op=dist.ReduceOp.SUM, group=self.group)
            train.apply_adamw(index)
            self._loss.copy_(train._loss)
            dist.all_reduce(self._loss, op=dist.ReduceOp.SUM, group=self.group)
            return self._loss / self.world
        y = train.forward(index, x, train._z)
        gy = train._gy[:n]
        native.check(native.lib.hffn_mse(y.data_ptr(), target.data_ptr(), gy.data_ptr(), train._loss.data_ptr(), n,
                                         train.d_model, train._work.data_ptr(),
                                         native.stream_handle(train.runtime.device)), "hffn_mse")
        train.backward(index, gy)
        grads = train.gradients(index)
        for name in ("up_val", "b_up", "out_val", "b_down"):
            dist.all_reduce(grads[name], op=dist.ReduceOp.SUM, group=self.group)
            grads[name].mul_(1.0 / self.world)
        train.adamw(index)
        self._loss.copy_(train._loss)
        dist.all_reduce(self._loss, op=dist.ReduceOp.SUM, group=self.group)
        return self._loss / self.world


class PeerShardedFFN:
    """The neuron-sharded forward over a stream of batches, its exchange through NVLink peer memory and copy engines
    instead of collective kernels, pipelined across batches (the native loop ``hffn_peer_pipeline_run``).

    Every rank holds its neuron shard and hands in batches [n, d] (all ranks the same n and count). Batch k of rank
    r is staged into r's gather buffer, pulled by copy engines into every other rank's gather buffer, run through
    every rank's shard (one up + down call over all ranks' batches), and each rank's partial outputs for the tokens
    of rank p are delivered into p's receive slot for it: by copy engines from a local buffer (``push="copy"``) or by
    the down GEMM's epilogue storing into the peer's slot over NVLink (``push="store"``); every rank sums its slots
    in rank order (a fixed summation order, whatever the timing). Iteration k stages batch k, waits for the pulls of
    batch k - 1 and the deliveries of batch k - 3, passes a barrier over signal pads in peer memory (bounded waits: a
    dead or late peer ends in error flag 201, never a hang), starts the pulls of batch k, runs batch k - 1, starts
    its deliveries and sums batch k - 3: the copy engines move one batch in and another out while the SMs run a third.

    Buffers live in symmetric memory (``torch.distributed._symmetric_memory``, plain peer mappings, no multicast
    object); no collective kernel runs beside the GEMMs and no load with multicast is issued. Requires the
    tensor-core runtime.
    """

    def __init__(self, runtime, d_model: int, group=None, push: str = "copy") -> None:
        if not runtime.tensor_cores:
            raise ValueError("the peer-memory sharded forward runs on the tensor-core path")
        if push not in ("store", "copy"):
            raise ValueError("push must be 'store' or 'copy'")
        self.runtime = runtime
        self.d_model = d_model
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one box)")
        self.push = push
        self._state: dict = {}

    def _setup(self, n: int, dtype: torch.dtype, device) -> dict:
        import os

        import torch.distributed._symmetric_memory as symm_mem

        from . import _native as native
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")   # plain peer mappings: no multicast object
        d, w, r = self.d_model, self.world, self.rank
        runtime = self.runtime
        elem = torch.empty(0, dtype=dtype).element_size()
        order = [(r + j) % w for j in range(w)]        # position j: rank (r + j) % w
        cfg = native.PeerConfig()
        cfg.world, cfg.rank, cfg.tokens, cfg.dtype = w, r, n, runtime._code
        keep = []
        for b in range(2):
            buf = symm_mem.empty(w * n, d, dtype=dtype, device=device)
            handle = symm_mem.rendezvous(buf, self.group)
            keep += [buf, handle]
            cfg.gather[b] = buf.data_ptr()
            for j, p in enumerate(order):
                cfg.gather_peer[b][j] = int(handle.buffer_ptrs[p])
        slots = []
        for b in range(3):
            buf = symm_mem.empty(w, n, d, dtype=dtype, device=device)
            handle = symm_mem.rendezvous(buf, self.group)
            keep += [buf, handle]
            slots.append(buf)
            cfg.slots[b] = buf.data_ptr()
            for j, p in enumerate(order):
                cfg.slot_peer[b][j] = int(handle.buffer_ptrs[p]) + r * n * d * elem
        signal = symm_mem.empty(w, dtype=torch.int32, device=device)
        signal_handle = symm_mem.rendezvous(signal, self.group)
        keep += [signal, signal_handle]
        signal.zero_()
        cfg.signal = signal.data_ptr()
        for j, p in enumerate(order):
            cfg.signal_peer[j] = int(signal_handle.buffer_ptrs[p])
        partial = [torch.empty(w * n, d, dtype=dtype, device=device) for _ in range(2)] if self.push == "copy" else []
        for b, buf in enumerate(partial):
            cfg.partial[b] = buf.data_ptr()
        work = torch.empty(int(native.lib.hffn_forward_tc_workspace(runtime._code, runtime._structs[0], w * n)),
                           dtype=torch.uint8, device=device)
        cfg.work = work.data_ptr()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)                # every rank's pad is zeroed before any signal
        if runtime._dense_stale[0]:
            runtime._densify(0)
        pipeline = ctypes.c_void_p()
        native.check(native.lib.hffn_peer_pipeline_create(ctypes.byref(cfg), ctypes.byref(runtime._structs[0]),
                                                          ctypes.byref(runtime._dense_structs[0]),
                                                          runtime._err.data_ptr(), ctypes.byref(pipeline)),
                     "hffn_peer_pipeline_create")
        return {"pipeline": pipeline, "config": cfg, "keep": keep, "slots": slots, "partial": partial, "work": work}

    def close(self) -> None:
        """Release the native pipelines (their buffers go with this object)."""
        from . import _native as native
        for state in self._state.values():
            native.lib.hffn_peer_pipeline_destroy(state["pipeline"])
        self._state.clear()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        """One batch: ``forward_many([x_local])[0]``."""
        return self.forward_many([x_local])[0]

    def forward_many(self, xs: list[torch.Tensor], outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
        """The layer's output for each batch of ``xs`` (this rank's tokens), every rank calling with the same number
        of batches of the same shape. ``outs``: contiguous [n, d] tensors to write (else allocated)."""
        from . import _native as native
        runtime = self.runtime
        if not xs:
            return []
        n, d = xs[0].shape[0], self.d_model
        for x in xs:
            runtime._check_input(x)
            if x.shape[0] != n:
                raise ValueError("every batch of one call has the same token count")
        if outs is None:
            outs = [torch.empty(n, d, dtype=xs[0].dtype, device=xs[0].device) for _ in xs]
        elif len(outs) != len(xs) or any(o.shape != (n, d) or o.dtype != xs[0].dtype or not o.is_contiguous()
                                         or o.device != xs[0].device for o in outs):
            raise ValueError("outs: one contiguous [n, d] tensor of the input dtype and device per batch")
        key = (n, xs[0].dtype)
        if key not in self._state:
            self._state[key] = self._setup(n, xs[0].dtype, xs[0].device)
        if runtime._dense_stale[0]:
            runtime._densify(0)
        count = len(xs)
        x_ptrs = (ctypes.c_void_p * count)(*(x.data_ptr() for x in xs))
        out_ptrs = (ctypes.c_void_p * count)(*(o.data_ptr() for o in outs))
        native.check(native.lib.hffn_peer_pipeline_run(self._state[key]["pipeline"], x_ptrs, out_ptrs, count,
                                                       native.stream_handle(xs[0].device)), "hffn_peer_pipeline_run")
        runtime.calls["tc", "tc"] += count
        return outs
