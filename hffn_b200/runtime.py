"""HFFN forward runtime for a stack of FFNs of one shape, on B200: the drop-in of the reference's
``runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py`` (``HFFNLayer``, ``HFFNRuntime``, ``up_mode``, ``down_mode``,
``UP_MODES``, ``DOWN_MODES``, ``MAX_TOKENS``).

One call runs the whole block of N tokens of one FFN through ``libhffn_b200.so``: the fused up + bias + GELU kernel,
then the down kernel, on the caller's current CUDA stream (any ``cuda:i``, any stream; the reference accepts only
cuda:0 and the default stream, ``runtime.py:79-82``). The policy (``modes``): the decode kernels for N <= 8; from 9
tokens the tcgen05 GEMMs over the densified supports (float32 in the fp16x3 operand format unless ``tc_format`` says
otherwise), when d_model and d_ff are multiples of 8; the CUDA-core kernels otherwise or when forced. Model arrays are
compact and stay on the device (the dense tensor-core operands are built from them on first use); the work buffers
(``act`` hidden-major ``[d_ff, N]``, the tensor-core workspace and ``y``) are shared by all layers, sized for the
largest N seen and reused. The output is a view of the runtime's buffer, overwritten by the next call, as in the
reference (``runtime.py:118-121``). Storage is float32 (the reference's only type) or bfloat16 (``dtype=``); the
kernels accumulate in float32 in both.

Errors follow the reference: ``ValueError`` for a bad shape, dtype, device, contiguity, token count or mode;
``hffn_b200._native.NativeError`` (a RuntimeError) when CUDA fails.
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass

import torch

from . import _native as native

UP_MODES = ("coop", "lane", "tile")
DOWN_MODES = ("coop", "tiled", "blocked")
TC = "tc"                   # the tensor-core path: up and down together, force("tc", "tc")
# The policy's tensor-core threshold (dense operands available): every N above the decode kernels' range (N <= 8).
# Measured on B200 against the CUDA-core tile / blocked kernels, N 9 .. 255: the tensor cores (narrow token tiles for
# small N) were faster at every N on the C1, C2 / C4 and C5 layer shapes in float32 and bfloat16, from 1.6x (C1 fp32,
# N 9-64) to 30x (C5 bf16, N 255); C2 fp32: 77-79 us against 248-903 us.
TC_MIN_TOKENS = 9
MAX_TOKENS = 1 << 24        # the kernels index tokens with 32-bit ints and act with 64-bit offsets
BLOCK = 512                 # threads of the tiled kernels
UP_TILE = 32                # largest token tile of the up kernel
DOWN_TILE = 32              # largest token tile of the down kernel
DTYPES = {torch.float32: native.F32, torch.bfloat16: native.BF16}


def up_mode(n: int, d_model: int = 0) -> str:
    """The up kernel the policy runs for N tokens (``hffn_up_mode``): coop for N <= 8, else tile."""
    return UP_MODES[native.lib.hffn_up_mode(n, d_model)]


def down_mode(n: int, d_ff: int = 0) -> str:
    """The down kernel the policy runs for N tokens (``hffn_down_mode``): coop for N <= 8, else blocked."""
    return DOWN_MODES[native.lib.hffn_down_mode(n, d_ff)]


@dataclass(frozen=True)
class HFFNLayer:
    """The kernel arrays of one FFN: up slots per hidden neuron, down edges in output order (``runtime.py:41-53``)."""
    d_model: int
    d_ff: int
    b_up: torch.Tensor         # [d_ff]
    up_offsets: torch.Tensor   # int32[d_ff + 1]
    up_idx: torch.Tensor       # int16[nnz_up], input feature of each slot
    up_val: torch.Tensor       # [nnz_up]
    b_down: torch.Tensor       # [d_model]
    out_offsets: torch.Tensor  # int32[d_model + 1]
    out_hidden: torch.Tensor   # int16[nnz_down], hidden neuron of each edge
    out_val: torch.Tensor      # [nnz_down]

    @classmethod
    def from_hidden_major(cls, d_model: int, d_ff: int, b_up: torch.Tensor, up_offsets: torch.Tensor,
                          up_idx: torch.Tensor, up_val: torch.Tensor, b_down: torch.Tensor, down_offsets: torch.Tensor,
                          down_idx: torch.Tensor, down_val: torch.Tensor) -> "HFFNLayer":
        """From the canonical hidden-major storage (neuron r owns ``[offsets[r], offsets[r + 1])`` on both sides).

        The up arrays are kept as given; the down slots are put in output-major order by a stable sort of their
        output feature, so that the edges of one output keep ascending neuron order, the order the reference fixes
        (``runtime.py:55-67``); ``out_offsets`` counts the edges of each output. CUDA tensors: the sort runs on their
        device (``layout_device.out_major``, the same bits) and the layer's arrays stay there."""
        if down_idx.is_cuda:
            from . import layout_device
            out_offsets, out_hidden, out_val = layout_device.out_major(d_model, d_ff, down_offsets, down_idx, down_val)
            return cls(d_model, d_ff, b_up, up_offsets, up_idx, up_val, b_down, out_offsets, out_hidden, out_val)
        output = down_idx.long().cpu()
        order = torch.argsort(output, stable=True)
        out_offsets = torch.zeros(d_model + 1, dtype=torch.int32)
        out_offsets[1:] = torch.cumsum(torch.bincount(output, minlength=d_model), 0)
        owner = torch.repeat_interleave(torch.arange(d_ff), down_offsets.cpu().diff().long())
        return cls(d_model, d_ff, b_up, up_offsets, up_idx, up_val, b_down, out_offsets,
                   owner[order].to(torch.int16), down_val.cpu()[order].contiguous())

    def model_bytes(self) -> int:
        return sum(v.numel() * v.element_size() for v in vars(self).values() if isinstance(v, torch.Tensor))

    def validate(self) -> None:
        """Refuse offsets that do not cover their arrays or indices out of range (ValueError)."""
        for side, offsets, index, values, count, bound in (
                ("up", self.up_offsets, self.up_idx, self.up_val, self.d_ff, self.d_model),
                ("down", self.out_offsets, self.out_hidden, self.out_val, self.d_model, self.d_ff)):
            offsets, index = offsets.cpu(), index.cpu()
            if offsets.dtype != torch.int32 or index.dtype != torch.int16:
                raise ValueError(f"{side}: offsets must be int32 and indices int16")
            if offsets.numel() != count + 1 or int(offsets[0]) != 0 or int(offsets[-1]) != values.numel() \
                    or index.numel() != values.numel():
                raise ValueError(f"{side}: offsets do not cover the compact arrays")
            if bool((offsets.diff() < 0).any()):
                raise ValueError(f"{side}: offsets decrease")
            if index.numel() and (int(index.min()) < 0 or int(index.max()) >= bound):
                raise ValueError(f"{side}: index out of range")
        if self.b_up.numel() != self.d_ff or self.b_down.numel() != self.d_model:
            raise ValueError("bias dimensions do not match d_model / d_ff")


ARRAYS = ("b_up", "up_offsets", "up_idx", "up_val", "b_down", "out_offsets", "out_hidden", "out_val")
VALUES = ("b_up", "up_val", "b_down", "out_val")


def layer_struct(tensors: dict, d_model: int, d_ff: int) -> native.Layer:
    """The ``hffn_layer`` of the device tensors of one layer (pointers only; the tensors own the memory)."""
    return native.Layer(d_model, d_ff, tensors["up_val"].numel(), tensors["out_val"].numel(),
                        *(tensors[name].data_ptr() for name in ARRAYS))


class HFFNRuntime:
    def __init__(self, layers: list[HFFNLayer], device: str | torch.device = "cuda",
                 dtype: torch.dtype = torch.float32, tensor_cores: bool | None = None,
                 tc_format: str | None = None) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the HFFN runtime runs on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if dtype not in DTYPES:
            raise ValueError("dtype must be torch.float32 or torch.bfloat16")
        self.dtype, self._code = dtype, DTYPES[dtype]
        self.layers = layers
        self.d_model, self.d_ff = layers[0].d_model, layers[0].d_ff
        if any((layer.d_model, layer.d_ff) != (self.d_model, self.d_ff) for layer in layers):
            raise ValueError("all layers of a runtime share d_model and d_ff")
        if self.d_model % 16:
            raise ValueError("d_model must be a multiple of 16")
        for layer in layers:
            layer.validate()
        # The device tensors own the memory; the structs hold their pointers for the native calls.
        self._tensors = [{name: (getattr(layer, name).to(self.device, dtype) if name in VALUES
                                 else getattr(layer, name).to(self.device)).contiguous() for name in ARRAYS}
                         for layer in layers]
        self._structs = [layer_struct(t, self.d_model, self.d_ff) for t in self._tensors]
        # Tensor-core operands: the supports densified (W_up [d_ff, d_model], W_down [d_model, d_ff], zeros off the
        # support), built on first use and rebuilt after the compact values change. Two formats: ``_dense`` (bfloat16;
        # float32 as tf32 hi / lo pairs, the operands of the 3xTF32 training step and of the peer pipeline) and
        # ``_dense16`` (float32 as scaled fp16 hi / lo pairs, the fp16x3 format of the float32 forward, the default;
        # ``tc_format="tf32x3"`` runs the float32 forward on the tf32 pairs instead).
        compatible = self.d_model % 8 == 0 and self.d_ff % 8 == 0
        if tensor_cores and not compatible:
            raise ValueError("the tensor-core path needs d_model and d_ff multiples of 8")
        self.tensor_cores = compatible if tensor_cores is None else bool(tensor_cores)
        if dtype == torch.bfloat16:
            if tc_format not in (None, "bf16"):
                raise ValueError("bfloat16 layers have one tensor-core format")
            self.tc_format = "bf16"
        else:
            if tc_format not in (None, "f16x3", "tf32x3"):
                raise ValueError("tc_format must be 'f16x3' or 'tf32x3'")
            self.tc_format = tc_format or "f16x3"
        count = len(layers)
        self._dense: list[dict | None] = [None] * count
        self._dense_structs: list = [None] * count
        self._dense_stale: list[bool] = [True] * count
        self._dense16: list[dict | None] = [None] * count
        self._dense16_structs: list = [None] * count
        self._dense16_stale: list[bool] = [True] * count
        # A floor of the fp16x3 up bound {max row L1 norm, max |b_up|}: a neuron shard whose token packets are read
        # by the other shards of the same layer sets the whole layer's bound (sharded_runtime)
        self.up_bound_floor: torch.Tensor | None = None
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.forced_up: str | None = None
        self.forced_down: str | None = None
        self.calls: Counter = Counter()
        self._tokens = 0
        self._reserve(1)

    def _alloc_dense(self) -> dict:
        f, d = self.d_ff, self.d_model
        split = self.dtype == torch.float32
        make = lambda rows, cols: torch.empty(rows, cols, device=self.device, dtype=self.dtype)  # noqa: E731
        return {"up_hi": make(f, d), "up_lo": make(f, d) if split else None,
                "down_hi": make(d, f), "down_lo": make(d, f) if split else None}

    def _densify(self, index: int) -> None:
        """(Re)build the tf32-pair (float32) or bfloat16 tensor-core operands of layer ``index`` from its compact
        arrays."""
        if self._dense[index] is None:
            dense = self._dense[index] = self._alloc_dense()
            self._dense_structs[index] = native.Dense(*(None if dense[k] is None else dense[k].data_ptr()
                                                        for k in ("up_hi", "up_lo", "down_hi", "down_lo")))
        t, dense, stream = self._tensors[index], self._dense[index], native.stream_handle(self.device)
        ptr = lambda v: None if v is None else v.data_ptr()  # noqa: E731
        native.check(native.lib.hffn_densify(self._code, t["up_offsets"].data_ptr(), t["up_idx"].data_ptr(),
                                             t["up_val"].data_ptr(), self.d_ff, self.d_model, ptr(dense["up_hi"]),
                                             ptr(dense["up_lo"]), stream), "hffn_densify up")
        native.check(native.lib.hffn_densify(self._code, t["out_offsets"].data_ptr(), t["out_hidden"].data_ptr(),
                                             t["out_val"].data_ptr(), self.d_model, self.d_ff, ptr(dense["down_hi"]),
                                             ptr(dense["down_lo"]), stream), "hffn_densify down")
        self._dense_stale[index] = False

    def _densify16(self, index: int) -> None:
        """(Re)build the fp16x3 operands of float32 layer ``index``: per projection the scaled fp16 hi / lo parts, the
        rows' inverse scales and, for up, the bound of |z| per unit of max|x| (``hffn_densify_f16x3``)."""
        f, d, device = self.d_ff, self.d_model, self.device
        if self._dense16[index] is None:
            half = lambda rows, cols: torch.empty(rows, cols, device=device, dtype=torch.float16)  # noqa: E731
            dense = self._dense16[index] = {
                "up_hi": half(f, d), "up_lo": half(f, d), "up_scale": torch.empty(f, device=device),
                "down_hi": half(d, f), "down_lo": half(d, f), "down_scale": torch.empty(d, device=device),
                "up_bound": torch.empty(2, device=device)}
            self._dense16_structs[index] = native.DenseF16x3(*(dense[k].data_ptr() for k in (
                "up_hi", "up_lo", "up_scale", "down_hi", "down_lo", "down_scale", "up_bound")))
        t, dense, stream = self._tensors[index], self._dense16[index], native.stream_handle(device)
        native.check(native.lib.hffn_densify_f16x3(t["up_offsets"].data_ptr(), t["up_idx"].data_ptr(),
                                                   t["up_val"].data_ptr(), t["b_up"].data_ptr(), f, d,
                                                   dense["up_hi"].data_ptr(), dense["up_lo"].data_ptr(),
                                                   dense["up_scale"].data_ptr(), dense["up_bound"].data_ptr(), stream),
                     "hffn_densify_f16x3 up")
        native.check(native.lib.hffn_densify_f16x3(t["out_offsets"].data_ptr(), t["out_hidden"].data_ptr(),
                                                   t["out_val"].data_ptr(), None, d, f, dense["down_hi"].data_ptr(),
                                                   dense["down_lo"].data_ptr(), dense["down_scale"].data_ptr(), None,
                                                   stream), "hffn_densify_f16x3 down")
        if self.up_bound_floor is not None:
            torch.maximum(dense["up_bound"], self.up_bound_floor.to(device), out=dense["up_bound"])
        self._dense16_stale[index] = False

    def forward_operands(self, index: int):
        """The ``(format, struct)`` of the dense operands the tensor-core forward of layer ``index`` runs on, built or
        rebuilt first if needed: ``("f16x3", DenseF16x3)`` or ``("tf32x3" / "bf16", Dense)``."""
        if self.tc_format == "f16x3":
            if self._dense16_stale[index]:
                self._densify16(index)
            return self.tc_format, self._dense16_structs[index]
        if self._dense_stale[index]:
            self._densify(index)
        return self.tc_format, self._dense_structs[index]

    def packet_bytes(self) -> int:
        """Bytes per token of the fp16x3 token packets (``hffn_f16x3_packet_bytes``)."""
        return int(native.lib.hffn_f16x3_packet_bytes(self.d_model))

    def uses_packets(self, n: int) -> bool:
        """Whether a call on ``n`` tokens runs the fp16x3 tensor-core forward, which can start from token packets."""
        return self.tc_format == "f16x3" and self.modes(n)[0] == TC

    def split_packets(self, index: int, x: torch.Tensor, packets: torch.Tensor) -> None:
        """x [N, d_model] (float32, contiguous, on the device) -> packets (uint8 [N, packet_bytes()]): each token's
        fp16x3 parts and scales (``hffn_split_f16x3``), the input of ``forward_packets`` here or on another rank
        holding another shard of the same layer (the up bound of every shard must be that of the whole layer)."""
        n = self._check_input(x)
        if packets.dtype != torch.uint8 or packets.shape != (n, self.packet_bytes()) or not packets.is_contiguous():
            raise ValueError("packets must be a contiguous uint8 [N, packet_bytes()] tensor")
        _, dense = self.forward_operands(index)
        native.check(native.lib.hffn_split_f16x3(x.data_ptr(), dense, packets.data_ptr(), self.d_model, self.d_ff, n,
                                                 native.stream_handle(self.device)), "hffn_split_f16x3")

    def forward_packets(self, index: int, packets: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """``forward`` from token packets (``split_packets``): y [N, d_model] into ``out`` (float32, contiguous)."""
        n = packets.shape[0]
        if packets.dtype != torch.uint8 or packets.dim() != 2 or packets.shape[1] != self.packet_bytes() \
                or not packets.is_contiguous() or packets.device != self._y.device:
            raise ValueError("packets must be a contiguous uint8 [N, packet_bytes()] tensor on the runtime's device")
        if out.shape != (n, self.d_model) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError("out must be a contiguous float32 [N, d_model] tensor")
        if self.tc_format != "f16x3":
            raise ValueError("token packets belong to the fp16x3 format")
        if n > self._tokens:
            self._reserve(n)
        _, dense = self.forward_operands(index)
        native.check(native.lib.hffn_forward_f16x3_packets(self._structs[index], dense, packets.data_ptr(),
                                                           out.data_ptr(), None, self._tc_work.data_ptr(),
                                                           self._err.data_ptr(), n, native.stream_handle(self.device)),
                     "hffn_forward_f16x3_packets")
        self.calls[TC, TC] += 1
        return out

    def mark_updated(self, index: int, refreshed: str | None = None) -> None:
        """The compact values of layer ``index`` changed (an optimiser step): the dense operands are rebuilt lazily,
        except those of format ``refreshed`` (``"tf32x3"``: the 3xTF32 training step refreshed them in place)."""
        if self.tensor_cores:
            if refreshed != "tf32x3":
                self._dense_stale[index] = True
            self._dense16_stale[index] = True

    def force(self, up: str | None, down: str | None) -> None:
        """Diagnostic: fix the up and/or the down kernel regardless of N (None: the policy). ``("tc", "tc")`` forces the
        tensor-core path, whose up and down run together."""
        if (up == TC) != (down == TC):
            raise ValueError("the tensor-core path is forced as the pair (\"tc\", \"tc\")")
        if up == TC and not self.tensor_cores:
            raise ValueError("this runtime has no tensor-core operands")
        if up not in (None, TC, *UP_MODES) or down not in (None, TC, *DOWN_MODES):
            raise ValueError("unknown kernel mode")
        self.forced_up, self.forced_down = up, down

    def _reserve(self, n: int) -> None:
        self._tokens = n
        self._act = torch.empty(self.d_ff * n, device=self.device, dtype=self.dtype)   # [d_ff, n]
        self._y = torch.empty(n, self.d_model, device=self.device, dtype=self.dtype)
        self._tc_work = None
        if self.tensor_cores:
            if self.tc_format == "f16x3":
                size = int(native.lib.hffn_forward_f16x3_workspace(self._structs[0], n))
            else:
                size = int(native.lib.hffn_forward_tc_workspace(self._code, self._structs[0], n))
            self._tc_work = torch.empty(size, dtype=torch.uint8, device=self.device)

    def workspace_bytes(self) -> int:
        extra = self._tc_work.numel() if self._tc_work is not None else 0
        return self._act.element_size() * (self._act.numel() + self._y.numel()) + extra

    def device_errors(self) -> int:
        """The error flags of the tensor-core kernels and of the decode kernels (0: none; the code of a wait that
        timed out otherwise). Synchronises."""
        code = int(self._err.item())
        if code:
            return code
        flag = native.ctypes.c_int32(0)
        with torch.cuda.device(self.device):
            native.check(native.lib.hffn_decode_error(native.ctypes.byref(flag), 0), "hffn_decode_error")
        return int(flag.value)

    def _check_input(self, x: torch.Tensor) -> int:
        if x.dim() != 2 or x.shape[1] != self.d_model or x.dtype != self.dtype or x.device != self._y.device \
                or not x.is_contiguous():
            raise ValueError(f"expected a contiguous {self.dtype} [N, d_model] tensor on the runtime's device")
        n = x.shape[0]
        if not 1 <= n <= MAX_TOKENS:
            raise ValueError("unsupported token count")
        return n

    def forward(self, index: int, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[N, d_model] of layer ``index`` for x[N, d_model]: a view of the runtime's output buffer (overwritten by
        the next call), or ``out`` (contiguous [N, d_model] of the runtime's dtype and device) when given."""
        n = self._check_input(x)
        if out is not None and (out.shape != (n, self.d_model) or out.dtype != self.dtype or out.device != self._y.device
                                or not out.is_contiguous()):
            raise ValueError("out must be a contiguous [N, d_model] tensor of the runtime's dtype and device")
        if n > self._tokens:
            self._reserve(n)
        up, down = self._launch(index, x, n, None, out)
        self.calls[up, down] += 1
        return self._y[:n] if out is None else out

    def modes(self, n: int, hidden_major: bool = False) -> tuple[str, str]:
        """The (up, down) modes of a call on N tokens. ``hidden_major``: the caller needs the hidden-major activations
        and z of the CUDA-core kernels (the training step), so the tensor-core pair is not taken."""
        up, down = self.forced_up, self.forced_down
        if hidden_major and up == TC:
            up = down = None
        if up is None and down is None and not hidden_major and self.tensor_cores and n >= TC_MIN_TOKENS:
            return TC, TC
        return up or up_mode(n, self.d_model), down or down_mode(n, self.d_ff)

    def _launch(self, index: int, x: torch.Tensor, n: int, z: torch.Tensor | None,
                out: torch.Tensor | None = None) -> tuple[str, str]:
        """Queue the up then the down kernel of layer ``index`` for the ``n`` tokens of ``x`` (validated, buffers
        reserved); ``z`` (float32, >= d_ff * n entries) also receives the pre-activations, hidden-major (the CUDA-core
        kernels then run whatever the policy). Returns the modes."""
        up, down = self.modes(n, hidden_major=z is not None)
        y = self._y if out is None else out
        if up == TC:
            fmt, dense = self.forward_operands(index)
            stream = native.stream_handle(self.device)
            if fmt == "f16x3":
                status = native.lib.hffn_forward_f16x3(self._structs[index], dense, x.data_ptr(), y.data_ptr(), None,
                                                       self._tc_work.data_ptr(), self._err.data_ptr(), n, stream)
            else:
                status = native.lib.hffn_forward_tc(self._code, self._structs[index], dense, x.data_ptr(),
                                                    y.data_ptr(), None, self._tc_work.data_ptr(),
                                                    self._err.data_ptr(), n, stream)
            native.check(status, "hffn_forward_tc")
            return up, down
        status = native.lib.hffn_forward(self._code, self._structs[index], x.data_ptr(), y.data_ptr(),
                                         self._act.data_ptr(), None if z is None else z.data_ptr(), n,
                                         native.UP_CODES[up], native.DOWN_CODES[down],
                                         native.stream_handle(self.device))
        native.check(status, "hffn_forward")
        return up, down


class PreparedRuntime(HFFNRuntime):
    """``HFFNRuntime`` whose small-batch calls (the decode steps) skip the per-call resolution: the drop-in of the
    reference's ``runtime/gpu/nvidia/llm/inference/hffn_pythia_cuda/prepared_runtime.py:34-82``.

    A call with N <= ``PREPARED_MAX_TOKENS`` tokens and no forced mode looks up a prepared entry of (layer, N): the
    layer's struct, the kernel mode codes and the device pointers of the runtime's ``act`` and ``y`` buffers, resolved
    once; the call then checks ``x`` and issues one ``hffn_forward``. ``_reserve`` (buffers moved) and ``force`` drop
    every entry. Every other call is ``HFFNRuntime.forward``. The kernels allocate nothing and run on the caller's
    current stream, so a prepared call can be captured in a CUDA graph (after one call outside the capture).
    """

    PREPARED_MAX_TOKENS = 8

    def _reserve(self, n: int) -> None:
        super()._reserve(n)
        self._prepared: dict = {}

    def force(self, up, down) -> None:
        super().force(up, down)
        self._prepared = {}

    def forward(self, index: int, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        n = x.shape[0] if x.dim() == 2 else 0
        if out is not None or self.forced_up or self.forced_down or not 1 <= n <= self.PREPARED_MAX_TOKENS:
            return super().forward(index, x, out)
        entry = self._prepared.get((index, n))
        if entry is None:
            self._check_input(x)
            if n > self._tokens:
                self._reserve(n)
            up, down = self.modes(n)
            entry = (self._structs[index], native.UP_CODES[up], native.DOWN_CODES[down], self._act.data_ptr(),
                     self._y.data_ptr(), (up, down))
            self._prepared[(index, n)] = entry
        elif x.dtype != self.dtype or x.shape[1] != self.d_model or x.device != self._y.device or not x.is_contiguous():
            raise ValueError(f"expected a contiguous {self.dtype} [N, d_model] tensor on the runtime's device")
        struct, up_code, down_code, act, y, modes = entry
        native.check(native.lib.hffn_forward(self._code, struct, x.data_ptr(), y, act, None, n, up_code, down_code,
                                             native.stream_handle(self.device)), "hffn_forward")
        self.calls[modes] += 1
        return self._y[:n]
