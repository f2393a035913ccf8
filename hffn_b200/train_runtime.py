"""HFFN training step on B200 over the forward runtime: the drop-in of the reference's
``runtime/gpu/nvidia/ffn/training/train_runtime.py`` (``HFFNTrainRuntime``, ``transposed_supports``, ``PARAMETERS``,
``SUPPORTS``).

The wrapped ``HFFNRuntime`` keeps its compact arrays, its dispatch policy and its work buffers; the step reads and
updates them in place. Added here, allocated at construction or by ``reserve(n)``:
- compact, per layer: the gradients of ``up_val``, ``b_up``, ``out_val``, ``b_down`` and their two AdamW moments, each
  of the length and order of its array (``out_val`` output-major); the two transposed supports as positions into the
  runtime's arrays;
- dense, shared by the layers, sized for the largest N reserved: ``z``, ``gz`` ``[d_ff, N]``, ``gx`` ``[N, d_model]``
  and the float32 workspace of ``hffn_backward`` (the transposed x and gy, and the token-group partials of the
  weight gradients, at most 16 groups whatever N).
No dense ``W_up``, ``W_down``, gradient or moment exists. ``step`` runs the fused backward + AdamW of
``hffn_backward``: each gradient entry is applied by AdamW in the kernel that completes it (and also stored, so that
``gradients()`` reads the step's gradients, unless ``store_gradients=False``). ``backward`` + ``adamw`` are the
reference's two separate phases. Nothing allocates once ``reserve(n)`` has run for the largest N.

``backward(index, gy)`` uses the state of the last ``forward(index, x, z)`` with a ``z`` buffer and must follow it
with no other forward of the runtime in between (checked, ``RuntimeError``), as in the reference.
"""
from __future__ import annotations

import math
from collections import Counter

import torch

from . import _native as native
from .runtime import MAX_TOKENS, TC, HFFNLayer, HFFNRuntime

# The training step's tensor-core threshold (the forward's is lower): the tensor-core MSE step contracts over the
# tokens in its weight-gradient GEMMs and its gates run at 257 to 2100 tokens; below 256 the CUDA-core step runs.
TC_MIN_TOKENS = 256

PARAMETERS = ("up_val", "b_up", "out_val", "b_down")
SUPPORTS = ("in_offsets", "in_pos", "in_hidden", "hid_offsets", "hid_pos", "hid_output")
PARTIAL_MAX_TOKENS = 2048
GRAD_TILE = 256          # tokens per tile of the reference's partial workspace (kernels_train.py:85)


def grad_tiles(n: int) -> int:
    """Tiles of GRAD_TILE tokens the reference's gradient kernels cut N into."""
    return -(-n // GRAD_TILE)


def transposed_supports(layer: HFFNLayer) -> dict[str, torch.Tensor]:
    """Up slots input-major and down edges hidden-major, as positions into the runtime's arrays (host, once).

    Stable sorts, so the up slots of one input keep ascending neuron order and the down edges of one neuron ascending
    output order: the summation orders of ``gx`` and ``gz`` (``train_runtime.py:39-56`` of the reference). A layer
    whose arrays are CUDA tensors is sorted on its device (``layout_device.supports``, the same bits)."""
    if layer.out_hidden.is_cuda:
        from . import layout_device
        return layout_device.supports(layer.d_model, layer.d_ff, layer.up_offsets, layer.up_idx, layer.out_offsets,
                                      layer.out_hidden)
    up_offsets, up_idx = layer.up_offsets.cpu().long(), layer.up_idx.cpu().long()
    out_offsets, out_hidden = layer.out_offsets.cpu().long(), layer.out_hidden.cpu().long()
    up_owner = torch.repeat_interleave(torch.arange(layer.d_ff), up_offsets.diff())
    by_input = torch.argsort(up_idx, stable=True)
    in_offsets = torch.zeros(layer.d_model + 1, dtype=torch.int32)
    in_offsets[1:] = torch.cumsum(torch.bincount(up_idx, minlength=layer.d_model), 0)
    out_owner = torch.repeat_interleave(torch.arange(layer.d_model), out_offsets.diff())
    by_hidden = torch.argsort(out_hidden, stable=True)
    hid_offsets = torch.zeros(layer.d_ff + 1, dtype=torch.int32)
    hid_offsets[1:] = torch.cumsum(torch.bincount(out_hidden, minlength=layer.d_ff), 0)
    return {"in_offsets": in_offsets, "in_pos": by_input.to(torch.int32),
            "in_hidden": up_owner[by_input].to(torch.int16),
            "hid_offsets": hid_offsets, "hid_pos": by_hidden.to(torch.int32),
            "hid_output": out_owner[by_hidden].to(torch.int16)}


def up_slots_ascending(layer: HFFNLayer) -> bool:
    """Whether the up slots of every neuron are in strictly ascending input order (the tensor-core training step
    walks each neuron's slots against the columns of its gradient tile)."""
    idx = layer.up_idx.cpu().long()
    if idx.numel() < 2:
        return True
    step = idx[1:] - idx[:-1]
    starts = layer.up_offsets.cpu().long()[1:-1]          # a slot that starts a neuron may step down
    ok = step > 0
    boundary = torch.zeros(idx.numel(), dtype=torch.bool)
    boundary[starts[(starts > 0) & (starts < idx.numel())]] = True
    return bool((ok | boundary[1:]).all())


def adamw_scalars(lr: float, betas: tuple[float, float], eps: float, weight_decay: float, k: int) -> native.AdamWStep:
    """The step scalars of update k, in float64 on the host, passed as float32 (``train_runtime.py:195-207``)."""
    beta1, beta2 = betas
    return native.AdamWStep(lr * weight_decay, beta1, 1.0 - beta1, beta2, 1.0 - beta2, lr / (1.0 - beta1 ** k),
                            math.sqrt(1.0 - beta2 ** k), eps)


class HFFNTrainRuntime:
    def __init__(self, runtime: HFFNRuntime, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2, max_tokens: int = PARTIAL_MAX_TOKENS,
                 store_gradients: bool = True, tensor_cores: bool | None = None) -> None:
        if runtime.dtype != torch.float32:
            raise ValueError("training runs on a float32 runtime (float32 master weights)")
        self.runtime = runtime
        self.d_model, self.d_ff = runtime.d_model, runtime.d_ff
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.store_gradients = store_gradients
        # the MSE step on the tensor cores: None = from TC_MIN_TOKENS tokens when possible, True / False = always / never
        self.tensor_cores = tensor_cores
        self._tc_layers = [runtime.tensor_cores and self.d_model % 32 == 0 and self.d_ff % 32 == 0
                           and up_slots_ascending(layer) for layer in runtime.layers]
        if tensor_cores and not all(self._tc_layers):
            raise ValueError("tensor-core training needs dense operands, d_model and d_ff multiples of 32 and ascending "
                             "up slots per neuron")
        self._tc_work = None
        self._tc_tokens = 0
        device = runtime.device
        self._supports, self._grads, self._moments = [], [], []
        self._support_structs, self._param_structs = [], []
        for layer, params in zip(runtime.layers, runtime._tensors):
            supports = {name: t.to(device) for name, t in transposed_supports(layer).items()}
            grads = {name: torch.zeros_like(params[name]) for name in PARAMETERS}
            moments = {name: (torch.zeros_like(params[name]), torch.zeros_like(params[name])) for name in PARAMETERS}
            self._supports.append(supports)
            self._grads.append(grads)
            self._moments.append(moments)
            self._support_structs.append(native.Supports(*(supports[name].data_ptr() for name in SUPPORTS)))
            self._param_structs.append(native.TrainParams(*(
                native.Param(params[name].data_ptr(), grads[name].data_ptr(), moments[name][0].data_ptr(),
                             moments[name][1].data_ptr(), params[name].numel()) for name in PARAMETERS)))
        self._fused_structs = [native.TrainParams(*(
            native.Param(p.value, p.grad if store_gradients else None, p.m, p.v, p.count)
            for p in (s.up_val, s.b_up, s.out_val, s.b_down))) for s in self._param_structs]
        # Columns of the partial workspace per layer, the reference's layout (train_runtime.py:79-89): g_down [0, c1),
        # gb_down [c1, c2), g_up [c2, c3), gb_up [c3, S); hffn_backward's token-group partials use the same columns.
        self._columns = []
        for params in runtime._tensors:
            for offsets, values in (("out_offsets", "out_val"), ("up_offsets", "up_val")):
                if int(params[offsets][0]) != 0 or int(params[offsets][-1]) != params[values].numel():
                    raise ValueError(f"{offsets} must cover {values} exactly (partial workspace columns)")
            c1 = params["out_val"].numel()
            c2 = c1 + self.d_model
            c3 = c2 + params["up_val"].numel()
            self._columns.append((c1, c2, c3, c3 + self.d_ff))
        self.steps = [0] * len(runtime.layers)
        self.calls: Counter = Counter()
        self._saved: tuple | None = None
        self._tokens = 0
        self._work_tokens = 0
        self.growths = 0
        self.reserve(1)
        self._reserve_partials(max_tokens)
        self.growths = 0

    # -- buffers -------------------------------------------------------------------------------------------------
    def reserve(self, n: int) -> None:
        """Size every dense buffer for N tokens; allocates only when N grows (call it with the largest N).

        ``growths`` counts each buffer family that had to grow (the runtime's forward buffers, this step's
        activation buffers, the backward workspace): a timed window must leave it unchanged."""
        if n > self.runtime._tokens:             # forward buffers (act, y, the tensor-core workspace)
            self.runtime._reserve(n)
            self._grown()
        if n > self._tokens:                     # this step's token-sized buffers
            self._tokens = n
            make = lambda *shape: torch.empty(*shape, device=self.runtime.device)  # noqa: E731
            self._z, self._gz = make(self.d_ff * n), make(self.d_ff * n)
            self._gx, self._gy = make(n, self.d_model), make(n, self.d_model)
            self._loss = torch.zeros(1, device=self.runtime.device)
            self._grown()
        self._reserve_partials(n)

    def _grown(self) -> None:
        """A buffer was replaced: count it, and forget the forward state the backward would read from the old one."""
        self.growths += 1
        self._saved = None

    def _reserve_partials(self, n: int) -> None:
        """Size the backward workspace for N tokens (grows only with N).

        Refuses (ValueError) an N at which the reference's partial workspace, ``grad_tiles(N)`` rows of the widest
        layer's columns, would pass 32-bit indexing (``train_runtime.py:119-127``): the drop-in accepts the token
        range the reference accepts. This build's workspace holds at most 16 token groups and is indexed with 64-bit
        offsets, so the bound is the reference's contract rather than a limit of these kernels."""
        stride = max(c[3] for c in self._columns)
        if grad_tiles(n) * stride >= 2 ** 32:
            raise ValueError(f"partial workspace of {grad_tiles(n)} tiles x {stride} columns exceeds 32-bit indexing")
        if n <= self._work_tokens:
            return
        floats = max(int(native.lib.hffn_backward_workspace(s, n)) for s in self.runtime._structs)
        floats = max(floats, 1024)
        self._work_tokens = n
        self.growths += 1
        self._work = torch.empty(floats, device=self.runtime.device)

    def _check_tokens(self, t: torch.Tensor, what: str) -> int:
        if (t.dim() != 2 or t.shape[1] != self.d_model or t.dtype != torch.float32 or t.device != self.runtime._y.device
                or not t.is_contiguous()):
            raise ValueError(f"expected a contiguous float32 [N, d_model] tensor {what} on the runtime's device")
        if not 1 <= t.shape[0] <= MAX_TOKENS:
            raise ValueError("unsupported token count")
        return t.shape[0]

    # -- the step and its pieces ---------------------------------------------------------------------------------
    def forward(self, index: int, x: torch.Tensor, z: torch.Tensor | None = None) -> torch.Tensor:
        """y[N, d_model] of layer ``index`` (a view of the runtime's output). With ``z`` (contiguous float32, at
        least d_ff * N entries): the same kernels also write ``z`` hidden-major and the state of the backward is kept."""
        runtime = self.runtime
        if z is None:
            return runtime.forward(index, x)
        n = self._check_tokens(x, "x")
        if z is self._z:          # the step's own buffer: sized here for N (reserve may replace it)
            self.reserve(n)
            z = self._z
        if z.dtype != torch.float32 or z.device != runtime._y.device or not z.is_contiguous() or z.numel() < self.d_ff * n:
            raise ValueError("z must be a contiguous float32 device tensor of at least d_ff * N entries")
        self.reserve(n)
        up, down = runtime._launch(index, x, n, z)
        runtime.calls[up, down] += 1
        self.calls[up, down] += 1
        self._saved = (index, n, z, x, sum(runtime.calls.values()))
        return runtime._y[:n]

    def _backward(self, index: int, gy: torch.Tensor, fused: native.AdamWStep | None) -> torch.Tensor:
        runtime = self.runtime
        if self._saved is None or self._saved[0] != index or self._saved[4] != sum(runtime.calls.values()):
            raise RuntimeError("backward must follow a forward of the same layer with a z buffer, with no forward in between")
        _, n, z, x, _ = self._saved
        if self._check_tokens(gy, "gy") != n:
            raise ValueError("gy must have the N of the forward")
        params = self._fused_structs[index] if fused is not None else self._param_structs[index]
        status = native.lib.hffn_backward(runtime._structs[index], self._support_structs[index], x.data_ptr(),
                                          gy.data_ptr(), z.data_ptr(), runtime._act.data_ptr(), self._gz.data_ptr(),
                                          self._gx.data_ptr(), params, fused, self._work.data_ptr(), n,
                                          native.stream_handle(runtime.device))
        native.check(status, "hffn_backward")
        return self._gx[:n]

    def backward(self, index: int, gy: torch.Tensor) -> torch.Tensor:
        """Compact gradients of layer ``index`` (see ``gradients``) and gx[N, d_model] (a view of the step's buffer)
        for the upstream gradient gy[N, d_model] of the last forward with a ``z`` buffer."""
        return self._backward(index, gy, None)

    def _next_step(self, index: int) -> native.AdamWStep:
        self.steps[index] += 1
        return adamw_scalars(self.lr, self.betas, self.eps, self.weight_decay, self.steps[index])

    def adamw(self, index: int) -> None:
        """One AdamW update of the four compact arrays of layer ``index`` from the gradients of the last backward."""
        scalars = self._next_step(index)
        stream = native.stream_handle(self.runtime.device)
        params = self._param_structs[index]
        for name in PARAMETERS:
            native.check(native.lib.hffn_adamw(getattr(params, name), scalars, stream), "hffn_adamw")
        self.runtime.mark_updated(index)

    def step(self, index: int, x: torch.Tensor, gy: torch.Tensor) -> torch.Tensor:
        """Forward (z stored in the step's buffer), then the fused backward + AdamW. Returns gx (a view)."""
        self.forward(index, x, self._z)
        gx = self._backward(index, gy, self._next_step(index))
        self.runtime.mark_updated(index)
        return gx

    def uses_tensor_cores(self, index: int, n: int) -> bool:
        if not self._tc_layers[index]:
            return False
        return self.tensor_cores if self.tensor_cores is not None else n >= TC_MIN_TOKENS

    def step_mse(self, index: int, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        """One step on the MSE loss ``mean((y - target)^2)``: forward, loss and its gradient
        ``gy = 2 (y - target) / (N d_model)``, fused backward + AdamW. Returns the loss (a 1-element device view,
        the loss of the parameters before the update). From ``TC_MIN_TOKENS`` tokens (``tensor_cores``) the whole
        step runs on the tensor cores (``hffn_train_step_tc``); gx is then ``self._gx`` and y the runtime's output."""
        n = self._check_tokens(target, "target")
        if self.uses_tensor_cores(index, n):
            return self.step_mse_tc(index, x, target)
        y = self.forward(index, x, self._z)
        if n != y.shape[0]:
            raise ValueError("target must have the N of x")
        gy = self._gy[:n]
        native.check(native.lib.hffn_mse(y.data_ptr(), target.data_ptr(), gy.data_ptr(), self._loss.data_ptr(), n,
                                         self.d_model, self._work.data_ptr(), native.stream_handle(self.runtime.device)),
                     "hffn_mse")
        self._backward(index, gy, self._next_step(index))
        self.runtime.mark_updated(index)
        return self._loss

    def _reserve_tc(self, n: int) -> None:
        self.reserve(n)
        if n > self._tc_tokens:
            size = int(native.lib.hffn_train_step_tc_workspace(self.runtime._structs[0], n))
            self._tc_work = torch.empty(size, dtype=torch.uint8, device=self.runtime.device)
            self._tc_tokens = n
            self.growths += 1

    def step_mse_tc(self, index: int, x: torch.Tensor, target: torch.Tensor, n_total: int | None = None,
                    apply: bool = True) -> torch.Tensor:
        """The MSE step on the tensor cores. ``n_total``: tokens of the loss mean (all ranks' for data parallelism).
        ``apply=False``: gradients stored, nothing updated (the caller exchanges them, then ``apply_adamw``)."""
        runtime = self.runtime
        n = self._check_tokens(x, "x")
        if self._check_tokens(target, "target") != n:
            raise ValueError("target must have the N of x")
        self._reserve_tc(n)
        # fp16x3 runtimes: four of the step's GEMMs run on the fp16x3 operands (rebuilt from the current values when
        # stale, as after every applied step) and its transposes, and the step reads no tf32 pair: those are built
        # once (the entry takes their addresses) and otherwise left stale for whoever needs them next
        f16 = runtime.tc_format == "f16x3"
        if runtime._dense_stale[index] and not (f16 and runtime._dense[index] is not None):
            runtime._densify(index)
        dense16 = runtime.forward_operands(index)[1] if f16 else None
        params = self._fused_structs[index] if apply else self._param_structs[index]
        status = native.lib.hffn_train_step_tc(runtime._structs[index], runtime._dense_structs[index], dense16,
                                               x.data_ptr(),
                                               target.data_ptr(), runtime._y.data_ptr(), self._gx.data_ptr(), params,
                                               self._next_step(index) if apply else None, self._loss.data_ptr(),
                                               self._tc_work.data_ptr(), runtime._err.data_ptr(), n, n_total or n,
                                               native.stream_handle(runtime.device))
        native.check(status, "hffn_train_step_tc")
        if apply:                 # the 3xTF32 step refreshed the tf32 pairs in place; the fp16x3 step refreshes none
            runtime.mark_updated(index, refreshed=None if dense16 is not None else "tf32x3")
        self._saved = None
        runtime.calls[TC, TC] += 1
        self.calls[TC, TC] += 1
        return self._loss

    def apply_adamw(self, index: int) -> None:
        """AdamW from the stored gradients (after a data-parallel exchange); the dense operands are rebuilt lazily."""
        self.adamw(index)

    # -- stacks of layers: every call keeps its own activations ---------------------------------------------------
    def forward_saved(self, index: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """``(y, z, act)`` of layer ``index`` for x[N, d_model], each a new tensor (z and act hidden-major
        ``[d_ff * N]``): the state its ``backward_saved`` needs, kept by the caller, so that a stack of layers can run
        all its forwards first and its backwards later in reverse order (the runtime's shared work buffers serve one
        layer at a time). The CUDA-core kernels (hidden-major activations); allocates through torch's caching
        allocator."""
        runtime = self.runtime
        n = self._check_tokens(x, "x")
        up, down = runtime.modes(n, hidden_major=True)
        device = runtime.device
        y = torch.empty(n, self.d_model, device=device)
        z = torch.empty(self.d_ff * n, device=device)
        act = torch.empty(self.d_ff * n, device=device)
        native.check(native.lib.hffn_forward(runtime._code, runtime._structs[index], x.data_ptr(), y.data_ptr(),
                                             act.data_ptr(), z.data_ptr(), n, native.UP_CODES[up],
                                             native.DOWN_CODES[down], native.stream_handle(device)), "hffn_forward")
        runtime.calls[up, down] += 1
        self.calls[up, down] += 1
        return y, z, act

    def backward_saved(self, index: int, x: torch.Tensor, gy: torch.Tensor, z: torch.Tensor,
                       act: torch.Tensor) -> torch.Tensor:
        """gx[N, d_model] (a new tensor) for the upstream gradient gy of a ``forward_saved`` call (its x, z, act);
        the layer's compact gradients (``gradients(index)``) are overwritten with this call's. ``adamw(index)``
        applies them."""
        runtime = self.runtime
        n = self._check_tokens(gy, "gy")
        if self._check_tokens(x, "x") != n or z.numel() < self.d_ff * n or act.numel() < self.d_ff * n:
            raise ValueError("x, z and act must come from the forward of the same N tokens")
        self._reserve_partials(n)
        device = runtime.device
        gz = torch.empty(self.d_ff * n, device=device)
        gx = torch.empty(n, self.d_model, device=device)
        native.check(native.lib.hffn_backward(runtime._structs[index], self._support_structs[index], x.data_ptr(),
                                              gy.data_ptr(), z.data_ptr(), act.data_ptr(), gz.data_ptr(), gx.data_ptr(),
                                              self._param_structs[index], None, self._work.data_ptr(), n,
                                              native.stream_handle(device)), "hffn_backward")
        return gx

    # -- read access for the checks (views, no copy) -------------------------------------------------------------
    def parameters(self, index: int) -> dict[str, torch.Tensor]:
        """The compact values of layer ``index`` (views: a caller may write through them, as the reference's checks
        do to restore a state, so the layer's dense tensor-core operands are marked for a rebuild)."""
        self.runtime.mark_updated(index)
        return {name: self.runtime._tensors[index][name] for name in PARAMETERS}

    def gradients(self, index: int) -> dict[str, torch.Tensor]:
        """Keyed by parameter: ``up_val`` hidden-major slot order, ``out_val`` output-major edge order."""
        return self._grads[index]

    def moments(self, index: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return self._moments[index]

    def supports(self, index: int) -> dict[str, torch.Tensor]:
        return self._supports[index]

    def activations(self, n: int) -> dict[str, torch.Tensor]:
        """z, h, gz hidden-major [d_ff, N] and gx [N, d_model] of the last step on N tokens."""
        return {"z": self._z[:self.d_ff * n].view(self.d_ff, n),
                "h": self.runtime._act[:self.d_ff * n].view(self.d_ff, n),
                "gz": self._gz[:self.d_ff * n].view(self.d_ff, n), "gx": self._gx[:n]}

    def nbytes(self, index: int) -> dict[str, int]:
        """Device bytes by role for layer ``index``: its compact values, gradients, moments and index arrays, and the
        buffers shared by the layers (forward work buffers with this step's activations; backward workspace)."""
        def total(*groups) -> int:
            return sum(t.numel() * t.element_size() for group in groups for t in group)
        own = self.runtime._tensors[index]
        return {"values": total(own[k] for k in PARAMETERS),
                "gradients": total(self._grads[index].values()),
                "moments": total(*self._moments[index].values()),
                "indices": total((own[k] for k in ("up_offsets", "up_idx", "out_offsets", "out_hidden")),
                                 self._supports[index].values()),
                "workspace": self.runtime.workspace_bytes() + total((self._z, self._gz, self._gx, self._gy)),
                "partials": total((self._work,))}


class HFFNFunction(torch.autograd.Function):
    """One HFFN layer as a torch autograd function: ``HFFNFunction.apply(x, train, index)`` -> y. The forward keeps
    the call's x, z and activations for its backward (``forward_saved`` / ``backward_saved``), so stacks of layers and
    whole models train through torch autograd; the backward returns gx and leaves the layer's compact gradients in
    ``train.gradients(index)`` (one backward per layer between two ``train.adamw(index)``)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, train: "HFFNTrainRuntime", index: int) -> torch.Tensor:
        y, z, act = train.forward_saved(index, x.contiguous())
        ctx.save_for_backward(x, z, act)
        ctx.train, ctx.index = train, index
        return y

    @staticmethod
    def backward(ctx, gy: torch.Tensor):
        x, z, act = ctx.saved_tensors
        return ctx.train.backward_saved(ctx.index, x.contiguous(), gy.contiguous(), z, act), None, None
